"""GPU parity of the split-KV decode kernel (q_len = 1) against the oracle's
restated xattn_head / xattn_head_f16 (flash_attn.rs:602-789), on the decode
workload's shapes: 5 beams x 12 heads over a KV cache of {1, 32, 128, 448}
keys (self-attention) and 1500 keys (cross-attention)."""

import numpy as np
import pytest
import torch

from ffai_b200 import attention, workloads
from helpers import (LSE_TOL, ROWSUM_TOL, assert_bf16_close, assert_f32_close, f32np,
                     rowsum_error)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _oracle_decode(oracle, q, k, v, scale=1.0):
    B, H, _, _ = q.shape
    keys = k.shape[2]
    qn = f32np(q).reshape(B * H, 64) * np.float32(scale)
    ktn = np.ascontiguousarray(np.swapaxes(f32np(k).reshape(B * H, keys, 64), 1, 2))
    vn = f32np(v).reshape(B * H, keys, 64)
    return oracle.xattn_rows(qn, ktn, vn, threads=8).reshape(B, H, 1, 64)


@pytest.mark.parametrize("keys", [1, 7, 8, 32, 128, 448, 1500])
@pytest.mark.parametrize("k_layout", ["heads", "kt"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_decode_parity(oracle, keys, k_layout, dtype):
    q, k, v = workloads.decode_inputs(keys, seed=1, dtype=dtype)
    ref = _oracle_decode(oracle, q, k, v)
    kd = k.transpose(-1, -2).contiguous() if k_layout == "kt" else k
    out, lse = attention.decode(q.to(DEV), kd.to(DEV), v.to(DEV), k_layout=k_layout, with_lse=True)
    got = f32np(out)
    # q stays f32 and products are f32 even over a 16-bit cache, so every
    # cache dtype meets the checked-f32 bar against the oracle.
    assert_f32_close(got, ref, f"decode keys={keys} {k_layout} {dtype}")
    assert_bf16_close(got, ref)
    B, H = q.shape[:2]
    err = rowsum_error(f32np(q).reshape(B * H, 1, 64), f32np(k).reshape(B * H, keys, 64), 1.0,
                       f32np(lse).reshape(B * H, 1))
    assert err <= LSE_TOL, f"LSE off by {err:.2e}"


@pytest.mark.parametrize("keys", [8, 448, 1500])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_decode_rowsums(keys, dtype):
    """Applied softmax weights sum to 1 within 1e-6 (V = ones)."""
    q, k, _ = workloads.decode_inputs(keys, seed=8, dtype=dtype)
    ones = torch.ones(k.shape, dtype=dtype)
    out = attention.decode(q.to(DEV), k.to(DEV), ones.to(DEV))
    err = (out.double() - 1.0).abs().max().item()
    assert err <= ROWSUM_TOL, f"row sums off by {err:.2e}"


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 12, 0])
def test_decode_split_counts(oracle, splits):
    q, k, v = workloads.decode_inputs(1500, seed=2)
    ref = _oracle_decode(oracle, q, k, v)
    out = attention.decode(q.to(DEV), k.to(DEV), v.to(DEV), num_splits=splits)
    assert_f32_close(f32np(out), ref, f"splits={splits}")


def test_decode_cache_prefix(oracle):
    """A cache of capacity 448 attended at its current length 129."""
    q, k, v = workloads.decode_inputs(448, seed=3)
    L = 129
    ref = _oracle_decode(oracle, q, k[:, :, :L], v[:, :, :L])
    for layout in ("heads", "kt"):
        kd = k.transpose(-1, -2).contiguous() if layout == "kt" else k
        out = attention.decode(q.to(DEV), kd.to(DEV), v.to(DEV), k_layout=layout, kv_len=L)
        assert_f32_close(f32np(out), ref, f"prefix {layout}")
    # causal at q_len 1: the query at position q_offset sees keys <= q_offset
    out = attention.decode(q.to(DEV), k.to(DEV), v.to(DEV), causal=True, q_offset=L - 1)
    assert_f32_close(f32np(out), ref, "causal prefix")


def test_decode_scale_and_bf16_out(oracle):
    q, k, v = workloads.decode_inputs(448, seed=4)
    ref = _oracle_decode(oracle, q, k, v, scale=0.125)
    out = attention.decode(q.to(DEV), k.to(DEV), v.to(DEV), scale=0.125, out_dtype=torch.bfloat16)
    assert out.dtype == torch.bfloat16
    assert_bf16_close(f32np(out), ref, "bf16 out")


def test_decode_bf16_query(oracle):
    q, k, v = workloads.decode_inputs(1500, seed=5)
    qb = q.to(torch.bfloat16)
    ref = _oracle_decode(oracle, qb, k, v)
    out = attention.decode(qb.to(DEV), k.to(DEV), v.to(DEV))
    assert_f32_close(f32np(out), ref, "bf16 q")


def test_decode_repeatable_and_ticket_rearmed(oracle):
    """Back-to-back launches reuse the split tickets; results stay bitwise equal."""
    q, k, v = workloads.decode_inputs(1500, seed=6)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    first = attention.decode(qd, kd, vd).clone()
    for _ in range(5):
        again = attention.decode(qd, kd, vd)
        assert torch.equal(first, again)
    attention.sync(0)


def test_decode_beams_independent():
    """Changing one beam's cache changes only that beam's output."""
    q, k, v = workloads.decode_inputs(448, seed=7)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    a = attention.decode(qd, kd, vd).clone()
    kd2 = kd.clone()
    kd2[2] = kd2[2].flip(1)
    vd2 = vd.clone()
    vd2[2] = torch.roll(vd2[2], 5, 1)
    b = attention.decode(qd, kd2, vd2)
    keep = [0, 1, 3, 4]
    assert torch.equal(a[keep], b[keep])
    assert not torch.equal(a[2], b[2])


@pytest.mark.parametrize("keys", [15, 16, 17, 63, 64, 65, 383, 384, 385, 769, 5000])
@pytest.mark.parametrize("beams,heads", [(5, 12), (1, 20), (2, 8), (16, 20)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_decode_row_and_key_counts(oracle, keys, beams, heads, dtype):
    """Ragged key counts around the stage and split boundaries, for row counts
    that take the cluster kernel (>= 19 rows on 148 SMs) and the split kernel."""
    q, k, v = workloads.decode_inputs(keys, seed=9, dtype=dtype, beams=beams, heads=heads)
    ref = _oracle_decode(oracle, q, k, v, scale=0.125)
    out = attention.decode(q.to(DEV), k.to(DEV), v.to(DEV), scale=0.125)
    assert_f32_close(f32np(out), ref, f"keys={keys} rows={beams * heads} {dtype}")


def test_decode_reads_q_written_just_before(oracle):
    """The decode kernel starts while the preceding kernel drains; it must
    still see the q that kernel wrote (no host sync between the launches)."""
    caches = [workloads.decode_inputs(1500, seed=20 + i) for i in range(4)]
    qbuf = torch.zeros(5, 12, 1, 64, device=DEV)
    k = caches[0][1].to(DEV)
    v = caches[0][2].to(DEV)
    qs = [c[0].to(DEV) for c in caches]
    outs = []
    for i in range(4):
        qbuf.copy_(qs[i])          # a kernel on the same stream
        qbuf.mul_(1.0)             # and a second one right before the decode
        outs.append(attention.decode(qbuf, k, v, kv_stable=(i % 2 == 1)))
    torch.cuda.synchronize()
    for i in range(4):
        ref = _oracle_decode(oracle, caches[i][0], caches[0][1], caches[0][2])
        assert_f32_close(f32np(outs[i]), ref, f"q written before decode {i}")


def test_decode_kv_stable_same_bits():
    q, k, v = workloads.decode_inputs(1500, seed=21)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    a = attention.decode(qd, kd, vd).clone()
    b = attention.decode(qd, kd, vd, kv_stable=True)
    assert torch.equal(a, b)


@pytest.mark.parametrize("keys", [1, 64, 65, 200, 448, 1500])
def test_decode_kv_append_only_same_bits(keys):
    # copying the older keys before the dependency wait changes no result
    q, k, v = workloads.decode_inputs(keys, seed=22)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    a = attention.decode(qd, kd, vd).clone()
    b = attention.decode(qd, kd, vd, kv_append_only=True)
    assert torch.equal(a, b)


def test_decode_kv_append_only_sees_the_appended_key(oracle):
    """The self-attention step: the newest key and value are written by a
    kernel on the same stream just before the decode that attends them; with
    kv_append_only the decode copies the older keys early but must see them."""
    keys, cap = 300, 448
    q, k, v = workloads.decode_inputs(cap, seed=23)
    kd, vd = k.to(DEV).clone(), v.to(DEV).clone()
    qd = q.to(DEV)
    outs, refs = [], []
    for step in range(4):
        n = keys + step
        kd[:, :, n - 1].mul_(-2.0)  # a kernel writing key n - 1 only
        vd[:, :, n - 1].add_(1.0)
        outs.append(attention.decode(qd, kd, vd, kv_len=n, kv_append_only=True))
        refs.append((kd[:, :, :n].cpu(), vd[:, :, :n].cpu()))
    torch.cuda.synchronize()
    for step, (o, (kr, vr)) in enumerate(zip(outs, refs)):
        ref = _oracle_decode(oracle, q, kr, vr)
        assert_f32_close(f32np(o), ref, f"append step {step}")


# ------------------------------------------------ next-call L2 prefetch (ffai_attn_decode_prefetch)
@pytest.mark.parametrize("keys,beams,heads,dtype", [
    (1500, 5, 12, torch.bfloat16), (448, 5, 12, torch.bfloat16), (1500, 5, 12, torch.float16),
    (300, 5, 12, torch.float32), (37, 5, 12, torch.bfloat16), (1500, 1, 2, torch.bfloat16)])
def test_decode_prefetch_same_bits(keys, beams, heads, dtype):
    """Prefetching the next call's cache into L2 reads nothing into this call:
    the results are ffai_attn_decode's bit for bit, on the cluster kernel's
    shapes and on one (2 rows) where the hint is ignored."""
    q, k, v = workloads.decode_inputs(keys, seed=31, dtype=dtype, beams=beams, heads=heads)
    _, nk, nv = workloads.decode_inputs(keys, seed=32, dtype=dtype, beams=beams, heads=heads)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    nkd, nvd = nk.to(DEV), nv.to(DEV)
    a, la = attention.decode(qd, kd, vd, with_lse=True)
    a, la = a.clone(), la.clone()
    b, lb = attention.decode(qd, kd, vd, with_lse=True, next_kv=(nkd, nvd), kv_stable=True)
    assert torch.equal(a, b) and torch.equal(la, lb)


def test_decode_prefetch_chain_of_layers(oracle):
    """A step over several layers' caches, each call prefetching the next
    layer's (the last one the first's): every output matches the oracle."""
    layers = 4
    caches = [workloads.decode_inputs(1500, seed=40 + i) for i in range(layers)]
    dev = [(q.to(DEV), k.to(DEV), v.to(DEV)) for q, k, v in caches]
    outs = []
    for i, (q, k, v) in enumerate(dev):
        _, nk, nv = dev[(i + 1) % layers]
        outs.append(attention.decode(q, k, v, next_kv=(nk, nv), kv_stable=True))
    torch.cuda.synchronize()
    for (q, k, v), o in zip(caches, outs):
        assert_f32_close(f32np(o), _oracle_decode(oracle, q, k, v), "prefetch chain")


def test_decode_prefetch_arguments():
    import ctypes
    from ffai_b200 import _abi
    q, k, v = workloads.decode_inputs(1500, seed=33)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    with pytest.raises(ValueError):  # next cache of another shape
        attention.decode(qd, kd, vd, next_kv=(kd[:, :, :100].contiguous(), vd[:, :, :100].contiguous()))
    with pytest.raises(ValueError):  # explicit split counts do not prefetch
        attention.decode(qd, kd, vd, next_kv=(kd, vd), num_splits=4)
    # one of the two pointers alone is an error from the library
    out = torch.empty(5, 12, 1, 64, device=DEV)
    d = _abi.new_desc(batch=5, heads=12, q_len=1, kv_len=1500, kv_capacity=1500,
                      q_dtype=attention._DT[qd.dtype], kv_dtype=attention._DT[kd.dtype],
                      out_dtype=attention._DT[out.dtype], scale=1.0)
    ctx = attention.context(0)
    st = _abi.load().ffai_attn_decode_prefetch(ctx, ctypes.byref(d), qd.data_ptr(), kd.data_ptr(),
                                               vd.data_ptr(), kd.data_ptr(), None,
                                               out.data_ptr(), None, None)
    assert st == _abi.ERR_INVALID
