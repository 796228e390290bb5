"""Multi-rank host logic on CPU: world_size-2 `gloo` process groups.

The GPU path shards segments over ranks with no data-path collective; what
crosses ranks is control traffic (barriers, the max over ranks of a time,
checksums) and each rank's output slice lands in one shared host buffer.
Here each rank computes its segments with the oracle (the CPU stand-in for
its GPU) and the gathered buffer is checked against a single-process run.
"""

import os
import socket
import uuid

import numpy as np
import pytest
import torch.multiprocessing as mp

from ffai_b200 import partition

SEGMENTS, HEADS, SEQ = 5, 2, 72


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(0)
    shape = (SEGMENTS, HEADS, SEQ, 64)
    q = (rng.standard_normal(shape) * 0.5).astype(np.float32)
    k = (rng.standard_normal(shape) * 0.5).astype(np.float32)
    v = rng.standard_normal(shape).astype(np.float32)
    return q, k, v


def _compute(segs):
    """Attention of segments `segs` with the restated reference kernel."""
    from oracle import oracle
    q, k, v = _inputs()
    out = np.zeros((len(segs), HEADS, SEQ, 64), np.float32)
    for i, s in enumerate(segs):
        out[i] = oracle.flash_rowmajor_k(q[s], k[s], v[s], 0.125, threads=1)
    return out


def _worker(rank, world, port, name, result_q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    group = partition.RankGroup("gloo", timeout_s=60).init()
    try:
        lo, hi = partition.contiguous_ranges(SEGMENTS, world)[rank]
        seg_bytes = HEADS * SEQ * 64 * 4
        buf = partition.open_shared_output(group, name, SEGMENTS * seg_bytes)
        mine = _compute(range(lo, hi))
        buf.view(np.float32, mine.shape, offset=lo * seg_bytes)[...] = mine
        group.barrier()
        whole = buf.view(np.float32, (SEGMENTS, HEADS, SEQ, 64)) if rank == 0 else None
        ok = partition.gather_verified(group, mine, whole)
        t_max = group.max(float(rank + 1))
        n_total = group.sum(float(hi - lo))
        if rank == 0:
            result_q.put((ok, t_max, n_total, np.array(whole)))
        group.barrier()
        buf.close(unlink=rank == 0)
    finally:
        group.close()


def test_two_rank_gather_matches_single_process(oracle):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    name = f"ffai_test_{uuid.uuid4().hex}"
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    ok, t_max, n_total, whole = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert ok is True
    assert t_max == 2.0            # max over ranks of (rank + 1)
    assert n_total == SEGMENTS     # every segment computed exactly once
    ref = _compute(range(SEGMENTS))
    assert np.array_equal(whole, ref)


def test_contiguous_ranges_cover_once():
    for n in (0, 1, 7, 64, 65):
        for w in (1, 2, 3, 8):
            r = partition.contiguous_ranges(n, w)
            assert len(r) == w and r[0][0] == 0 and r[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
            sizes = [b - a for a, b in r]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [1, 2, 8])
def test_ragged_assignment_balances_work(world):
    from ffai_b200 import workloads
    lengths = workloads.ragged_lengths()
    assign, load, tokens = partition.ragged_assignment(lengths, world)
    flat = sorted(i for a in assign for i in a)
    assert flat == list(range(len(lengths)))
    costs = [float(L) ** 2 for L in lengths]
    assert abs(sum(load) - sum(costs)) < 1e-6 * sum(costs)
    lower = max(max(costs), sum(costs) / world)
    assert max(load) <= 4 / 3 * lower          # Graham's LPT bound vs. a lower bound
    assert sum(tokens) == sum(lengths)


def test_checksum_is_order_independent_sum():
    # slices that split on 8-byte boundaries (whole segments do) add up exactly
    b = np.arange(4096, dtype=np.int16)
    halves = [b[:2048], b[2048:]]
    assert partition.checksum(b) == sum(partition.checksum(h) for h in halves) % 2**64
