"""The multi-device host entry (ffai_attn_multi_prefill_host): its chunk
queue on CPU with injected worker failures, and on a GPU with several
worker contexts, with and without a host-side injected fault."""

import ctypes
import os

import pytest
import torch

from ffai_b200 import _abi


def _selftest(workers, chunks, mask):
    owner = (ctypes.c_int32 * max(1, chunks))(*([-1] * max(1, chunks)))
    failed = ctypes.c_int32(-1)
    st = _abi.load().ffai_attn_chunk_queue_selftest(workers, chunks, mask, owner,
                                                   ctypes.byref(failed))
    return st, list(owner)[:chunks], failed.value


@pytest.mark.parametrize("workers,chunks", [(1, 1), (2, 8), (4, 64), (8, 8), (8, 3)])
def test_queue_completes_every_chunk_once(workers, chunks):
    st, owner, failed = _selftest(workers, chunks, 0)
    assert st == _abi.OK and failed == 0
    assert all(0 <= o < workers for o in owner)


@pytest.mark.parametrize("workers,chunks,mask", [(2, 8, 0b01), (4, 16, 0b1010), (8, 64, 0x7F),
                                                 (3, 2, 0b011)])
def test_failed_workers_hand_chunks_back(workers, chunks, mask):
    """A worker that fails retires after handing its chunk back; the others
    complete every chunk, and no chunk is owned by a failed worker."""
    st, owner, failed = _selftest(workers, chunks, mask)
    dead = {w for w in range(workers) if (mask >> w) & 1}
    assert st == _abi.OK
    # worker w starts with chunk w, so every marked worker that has a first
    # chunk fails exactly once
    assert failed == len({w for w in dead if w < chunks})
    assert all(o not in dead and 0 <= o < workers for o in owner)


def test_all_workers_failing_is_an_error():
    st, owner, failed = _selftest(3, 5, 0b111)
    assert st != _abi.OK and failed == 3


def _inputs(B=6, H=8, N=300, seed=3):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, H, N, 64, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, H, N, 64, generator=g) * 0.5).to(torch.bfloat16)
    v = torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16)
    return q.pin_memory(), k.pin_memory(), v.pin_memory()


@pytest.mark.gpu
@pytest.mark.parametrize("chunk", [0, 1, 4])
def test_multi_matches_single_device(chunk):
    from ffai_b200 import attention
    q, k, v = _inputs()
    ref = attention.prefill_host(q, k, v, device=0, scale=0.125, out_dtype=torch.bfloat16)
    devs = [d for d in range(torch.cuda.device_count())] * 2  # two workers per device
    out, failed = attention.multi_prefill_host(q, k, v, devices=devs, scale=0.125,
                                               out_dtype=torch.bfloat16, chunk_segments=chunk)
    assert failed == 0
    assert torch.equal(out, ref)


@pytest.mark.gpu
def test_multi_recovers_from_an_injected_worker_fault(monkeypatch):
    from ffai_b200 import attention
    q, k, v = _inputs(seed=4)
    ref = attention.prefill_host(q, k, v, device=0, scale=0.125, out_dtype=torch.bfloat16)
    monkeypatch.setenv("FFAI_ATTN_FAULT_WORKER", "1")
    out, failed = attention.multi_prefill_host(q, k, v, devices=[0, 0, 0], scale=0.125,
                                               out_dtype=torch.bfloat16, chunk_segments=1)
    assert failed == 1
    assert torch.equal(out, ref)
