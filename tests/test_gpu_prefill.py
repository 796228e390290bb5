"""GPU parity of the prefill/encoder kernels against the oracle's restated
flash_head (flash_attn.rs:429-487): the tcgen05 bf16 kernel within
max 1e-2 / mean 1e-3 of the oracle run in f32 on the same bf16-rounded
inputs, the checked f32 kernel within 1e-5 relative, softmax row sums within
1e-6 (through the exported log-sum-exp), on the encoder workloads' shapes and
the edge lengths around every tile boundary."""

import numpy as np
import pytest
import torch

from ffai_b200 import attention, workloads
from helpers import (LSE_TC_TOL, LSE_TOL, ROWSUM_TOL, assert_bf16_close, assert_f32_close, f32np,
                     oracle_encoder, rowsum_error)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
S = workloads.SCALE


def _inputs(B, H, N, dtype=torch.bfloat16, seed=0, M=None):
    g = torch.Generator().manual_seed(seed)
    M = N if M is None else M
    q = (torch.randn(B, H, N, 64, generator=g) * 0.5).to(dtype)
    k = (torch.randn(B, H, M, 64, generator=g) * 0.5).to(dtype)
    v = torch.randn(B, H, M, 64, generator=g).to(dtype)
    return q, k, v


@pytest.mark.parametrize("N", [1, 7, 63, 64, 65, 127, 128, 129, 255, 256, 257, 383, 385, 500, 750])
def test_tc_edge_lengths(oracle, N):
    q, k, v = _inputs(2, 3, N, seed=N)
    ref = oracle_encoder(oracle, q, k, v, S)
    out = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S)
    assert_bf16_close(f32np(out), ref, f"N={N}")


def test_tc_c2_base_encoder_batched(oracle):
    cfg = workloads.C2
    q, k, v = workloads.encoder_inputs(cfg, seed=0)
    ref = oracle_encoder(oracle, q, k, v, S)
    out, lse = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S, with_lse=True)
    mx, mean = assert_bf16_close(f32np(out), ref, "c2")
    print(f"c2 max|err| {mx:.2e} mean|err| {mean:.2e}")
    # row sums through the exported LSE, on a few (segment, head) pairs
    for b, h in [(0, 0), (3, 5), (7, 7)]:
        err = rowsum_error(f32np(q[b, h])[None], f32np(k[b, h])[None], S, f32np(lse[b, h])[None])
        assert err <= LSE_TC_TOL, f"LSE off by {err:.2e} at ({b},{h})"


def test_c1_tiny_encoder_f32(oracle):
    """c1: f32 operands.  Default path: bf16 tensor cores (operands rounded
    on the device); checked path: f32 SIMT kernel at 1e-5 relative."""
    cfg = workloads.C1
    q, k, v = workloads.encoder_inputs(cfg, seed=0)
    ref32 = oracle_encoder(oracle, q, k, v, S)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    chk = attention.prefill(qd, kd, vd, scale=S, checked=True)
    assert_f32_close(f32np(chk), ref32, "c1 checked")
    out = attention.prefill(qd, kd, vd, scale=S)
    rb = [t.to(torch.bfloat16) for t in (q, k, v)]
    ref16 = oracle_encoder(oracle, *rb, S)
    assert_bf16_close(f32np(out), ref16, "c1 bf16 path")


@pytest.mark.parametrize("N", [1, 63, 65, 300])
def test_checked_f32_edges(oracle, N):
    q, k, v = _inputs(1, 2, N, dtype=torch.float32, seed=100 + N)
    ref = oracle_encoder(oracle, q, k, v, S)
    out, lse = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S, checked=True,
                                 with_lse=True)
    assert_f32_close(f32np(out), ref, f"checked N={N}")
    err = rowsum_error(f32np(q).reshape(2, N, 64), f32np(k).reshape(2, N, 64), S,
                       f32np(lse).reshape(2, N))
    assert err <= LSE_TOL


def test_checked_causal_vs_f64(oracle):
    """Causal prefill with a query offset (decoder prompt), checked f32."""
    q, k, v = _inputs(1, 2, 40, dtype=torch.float32, seed=9, M=72)
    out = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S, checked=True, causal=True,
                            q_offset=32)
    ref, _ = oracle.naive_attention_f64(f32np(q), f32np(k), f32np(v), scale=S, causal=True,
                                        q_offset=32)
    assert_f32_close(f32np(out), ref, "causal")


@pytest.mark.parametrize("B,H,Nq,q_offset,cap", [
    (5, 12, 1, 0, 448), (5, 12, 7, 3, 448), (5, 12, 128, 0, 448), (5, 12, 129, 200, 448),
    (2, 12, 300, 100, 448), (1, 12, 448, 0, 448), (1, 4, 1500, 0, 1500), (1, 3, 257, 1200, 1500)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tc_causal_vs_f64(oracle, B, H, Nq, q_offset, cap, dtype):
    """Causal prefill on the tensor-core kernel: decoder prompts over a cache
    of capacity `cap` (keys 0 .. q_offset + Nq - 1 live) and encoder-length
    causal rows; row i sees keys <= q_offset + i."""
    kv = q_offset + Nq
    q, k, v = _inputs(B, H, Nq, dtype=dtype, seed=40 + Nq, M=cap)
    out, lse = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S, causal=True,
                                 q_offset=q_offset, kv_len=kv, with_lse=True)
    ref, ref_lse = oracle.naive_attention_f64(f32np(q), f32np(k)[:, :, :kv], f32np(v)[:, :, :kv],
                                              scale=S, causal=True, q_offset=q_offset)
    assert_bf16_close(f32np(out), ref, f"causal Nq={Nq} off={q_offset}")
    # The kernel's LSE normalises the rounded 16-bit P it applies.  A row with
    # one visible key has one P, rounded by up to 2^-8 (bf16), so its LSE may
    # differ from the exact one by ln(1 + 2^-8) < 4e-3; long rows average out.
    assert np.abs(f32np(lse) - ref_lse).max() <= 4e-3


def test_tc_causal_rowsums():
    """Applied weights of every causal row sum to 1 within 1e-6 (V = ones)."""
    q, k, _ = _inputs(2, 4, 300, seed=44, M=448)
    ones = torch.ones(2, 4, 448, 64, dtype=torch.bfloat16)
    out = attention.prefill(q.to(DEV), k.to(DEV), ones.to(DEV), scale=S, causal=True,
                            q_offset=148, kv_len=448)
    err = (out.double() - 1.0).abs().max().item()
    assert err <= ROWSUM_TOL, f"row sums off by {err:.2e}"


@pytest.mark.parametrize("layout", ["token_in", "token_out", "kt", "all_token"])
def test_tc_layouts(oracle, layout):
    q, k, v = _inputs(2, 4, 300, seed=21)
    ref = oracle_encoder(oracle, q, k, v, S)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    kw = {}
    if layout in ("token_in", "all_token"):
        qd, kd, vd = (t.transpose(1, 2).contiguous() for t in (qd, kd, vd))
        kw.update(q_layout="token", k_layout="token", v_layout="token")
    if layout in ("token_out", "all_token"):
        kw.update(out_layout="token")
    if layout == "kt":
        kd = kd.transpose(-1, -2).contiguous()
        kw.update(k_layout="kt")
    out = attention.prefill(qd, kd, vd, scale=S, **kw)
    if kw.get("out_layout") == "token":
        out = out.transpose(1, 2)
    assert_bf16_close(f32np(out), ref, layout)


def test_tc_f16_and_bf16_out(oracle):
    q, k, v = _inputs(2, 3, 500, dtype=torch.float16, seed=31)
    ref = oracle_encoder(oracle, q, k, v, S)
    out = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S)
    assert_bf16_close(f32np(out), ref, "f16")
    kt = k.transpose(-1, -2).contiguous()
    out2 = attention.prefill(q.to(DEV), kt.to(DEV), v.to(DEV), scale=S, k_layout="kt",
                             out_dtype=torch.bfloat16)
    assert out2.dtype == torch.bfloat16
    assert_bf16_close(f32np(out2), ref, "f16 kt, bf16 out")


def test_tc_cross_shape_kv_capacity(oracle):
    """q_len != kv_len, and a K/V buffer larger than the attended prefix."""
    q, k, v = _inputs(2, 2, 200, seed=41, M=700)
    L = 555
    ref = oracle_encoder(oracle, q, k[:, :, :L], v[:, :, :L], S)
    out = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S, kv_len=L)
    assert_bf16_close(f32np(out), ref, "kv prefix")


def test_tc_lse_rowsums(oracle):
    q, k, v = _inputs(1, 2, 1500, seed=51)
    _, lse = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S, with_lse=True)
    err = rowsum_error(f32np(q).reshape(2, 1500, 64), f32np(k).reshape(2, 1500, 64), S,
                       f32np(lse).reshape(2, 1500))
    assert err <= LSE_TC_TOL, f"LSE off by {err:.2e}"


@pytest.mark.parametrize("path", ["tc_bf16", "tc_f16", "checked_f32"])
def test_softmax_rowsums(path):
    """Row sums of the applied softmax weights within 1e-6: with V = ones,
    every output element is sum_j P_ij / l_i."""
    dtype = {"tc_bf16": torch.bfloat16, "tc_f16": torch.float16, "checked_f32": torch.float32}[path]
    q, k, _ = _inputs(2, 4, 1500, dtype=dtype, seed=55)
    ones = torch.ones(2, 4, 1500, 64, dtype=dtype)
    out = attention.prefill(q.to(DEV), k.to(DEV), ones.to(DEV), scale=S,
                            checked=(path == "checked_f32"))
    err = (out.double() - 1.0).abs().max().item()
    assert err <= ROWSUM_TOL, f"{path}: row sums off by {err:.2e}"


def test_tc_deterministic_and_no_stray_writes():
    q, k, v = _inputs(3, 5, 777, seed=61)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    canary = torch.full((3 * 5 * 777 * 64 + 4096,), 12345.0, device=DEV)
    out = canary[: 3 * 5 * 777 * 64].view(3, 5, 777, 64)
    attention.prefill(qd, kd, vd, scale=S, out=out)
    assert torch.all(canary[3 * 5 * 777 * 64:] == 12345.0), "write past the output"
    first = out.clone()
    again = attention.prefill(qd, kd, vd, scale=S)
    assert torch.equal(first, again)
    attention.sync(0)


def test_tc_segments_independent():
    """Changing one segment changes only that segment's output (content, not shape)."""
    q, k, v = _inputs(3, 2, 400, seed=71)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    a = attention.prefill(qd, kd, vd, scale=S).clone()
    kd[1] = kd[1].flip(1)
    b = attention.prefill(qd, kd, vd, scale=S)
    assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2])
    assert not torch.equal(a[1], b[1])


def test_c4_sampled_parity(oracle):
    """Full c4 batch (64 x 20 x 1500) on the GPU; a sample of (segment, head)
    pairs against the oracle, plus whole-batch sanity: finite, and every
    output row a convex combination of V rows (|o| <= max |v|)."""
    cfg = workloads.C4
    q, k, v = workloads.encoder_inputs(cfg, seed=0, device=DEV)
    out = attention.prefill(q, k, v, scale=S, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert out.float().abs().amax() <= v.float().abs().amax() + 1e-2
    rng = np.random.default_rng(0)
    for b, h in zip(rng.integers(0, cfg.segments, 6), rng.integers(0, cfg.heads, 6)):
        b, h = int(b), int(h)
        sub = [t[b:b + 1, h:h + 1].cpu() for t in (q, k, v)]
        ref = oracle_encoder(oracle, *sub, S)
        assert_bf16_close(f32np(out[b:b + 1, h:h + 1]), ref, f"c4 ({b},{h})")


def _oracle_ragged(oracle, q, k, v, cu, segs):
    outs = {}
    for s in segs:
        a, b = cu[s], cu[s + 1]
        qs = q[a:b].transpose(0, 1)[None]
        ks = k[a:b].transpose(0, 1)[None]
        vs = v[a:b].transpose(0, 1)[None]
        outs[s] = oracle_encoder(oracle, qs, ks, vs, S)[0].transpose(1, 0, 2)
    return outs


def test_varlen_small(oracle):
    lengths = [1, 129, 256, 257, 600, 64, 999, 3]
    q, k, v, cu = workloads.ragged_inputs(lengths, heads=4, seed=3)
    out, lse = attention.varlen(q.to(DEV), k.to(DEV), v.to(DEV), cu, scale=S, with_lse=True)
    refs = _oracle_ragged(oracle, q, k, v, cu, range(len(lengths)))
    for s, ref in refs.items():
        assert_bf16_close(f32np(out[cu[s]:cu[s + 1]]), ref, f"segment {s}")
    s = 6
    a, b = cu[s], cu[s + 1]
    err = rowsum_error(f32np(q[a:b]).transpose(1, 0, 2), f32np(k[a:b]).transpose(1, 0, 2), S,
                       f32np(lse[:, a:b]))
    assert err <= LSE_TC_TOL


def test_varlen_c5_sampled(oracle):
    """c5 at full size: 256 packed segments of 200-1500 frames, 16 heads."""
    lengths = workloads.ragged_lengths()
    q, k, v, cu = workloads.ragged_inputs(lengths, device=DEV)
    out = attention.varlen(q, k, v, cu, scale=S, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    segs = [0, 1, int(np.argmax(lengths)), int(np.argmin(lengths)), 255]
    refs = _oracle_ragged(oracle, q.cpu(), k.cpu(), v.cpu(), cu, segs)
    for s, ref in refs.items():
        assert_bf16_close(f32np(out[cu[s]:cu[s + 1]]), ref, f"c5 segment {s}")


def test_varlen_matches_batched():
    """Equal-length segments through varlen equal the batched kernel bitwise."""
    q, k, v = _inputs(3, 4, 384, seed=81)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    a = attention.prefill(qd, kd, vd, scale=S)
    pack = lambda t: t.transpose(1, 2).reshape(3 * 384, 4, 64).contiguous()
    b = attention.varlen(pack(qd), pack(kd), pack(vd), [0, 384, 768, 1152], scale=S)
    assert torch.equal(pack(a), b)


@pytest.mark.parametrize("dtype,checked", [(torch.bfloat16, False), (torch.float32, False),
                                           (torch.float32, True)])
def test_fused_qkv_views_read_in_place(dtype, checked):
    """q, k, v as the three thirds of one fused projection output
    (B, N, 3, H, 64): read with a token stride of 3*H*64, no copies; equal to
    the result on dense copies."""
    B, N, H = 2, 300, 8
    g = torch.Generator().manual_seed(50)
    qkv = (torch.randn(B, N, 3, H, 64, generator=g) * 0.5).to(dtype).to(DEV)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    assert not q.is_contiguous()
    kw = dict(scale=S, q_layout="token", k_layout="token", v_layout="token", out_layout="token",
              out_dtype=torch.bfloat16, checked=checked)
    got = attention.prefill(q, k, v, **kw)
    ref = attention.prefill(q.contiguous(), k.contiguous(), v.contiguous(), **kw)
    assert torch.equal(got, ref)


def test_fused_qkv_views_varlen():
    g = torch.Generator().manual_seed(51)
    lens = [200, 333, 129]
    T, H = sum(lens), 4
    qkv = (torch.randn(T, 3, H, 64, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    cu = [0, 200, 533, 662]
    got = attention.varlen(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, scale=S)
    ref = attention.varlen(qkv[:, 0].contiguous(), qkv[:, 1].contiguous(),
                           qkv[:, 2].contiguous(), cu, scale=S)
    assert torch.equal(got, ref)


@pytest.mark.parametrize("N", [1, 15, 16, 17, 127, 129, 300, 1500])
@pytest.mark.parametrize("layout", ["heads", "token"])
def test_bf16_output_equals_rounded_f32_output(N, layout):
    """bf16 output (whole 16-row groups go out through the tensor-store
    epilogue, ragged ones through plain stores) is exactly the f32 output
    rounded to bf16, at lengths around the 16-row groups and tiles."""
    q, k, v = _inputs(2, 3, N, seed=60 + N)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    kw = dict(scale=S, out_layout=layout)
    if layout == "token":
        qd, kd, vd = (x.transpose(1, 2).contiguous() for x in (qd, kd, vd))
        kw.update(q_layout="token", k_layout="token", v_layout="token")
    f32 = attention.prefill(qd, kd, vd, out_dtype=torch.float32, **kw)
    b16 = attention.prefill(qd, kd, vd, out_dtype=torch.bfloat16, **kw)
    assert torch.equal(b16, f32.to(torch.bfloat16))


def test_bf16_output_varlen_equals_rounded_f32():
    g = torch.Generator().manual_seed(61)
    lens = [200, 16, 333, 129, 1]
    T, H = sum(lens), 4
    q, k, v = ((torch.randn(T, H, 64, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
               for _ in range(3))
    cu = [0]
    for L in lens:
        cu.append(cu[-1] + L)
    f32 = attention.varlen(q, k, v, cu, scale=S, out_dtype=torch.float32)
    b16 = attention.varlen(q, k, v, cu, scale=S, out_dtype=torch.bfloat16)
    assert torch.equal(b16, f32.to(torch.bfloat16))


def test_inputs_stable_back_to_back_equals_single_launches():
    """Launches over independent batches with FFAI_ATTN_FLAG_INPUTS_STABLE run
    back to back (each reads its operands while the previous one finishes,
    and the work list keeps a short last wave of two-tile units): every
    result equals the same batch launched alone without the flag, bitwise.
    4 x 20 x 1500 is 480 units, a last wave of 36 on 148 SMs."""
    batches = [tuple(t.to(DEV) for t in _inputs(4, 20, 1500, seed=90 + i)) for i in range(4)]
    want = [attention.prefill(*b, scale=S, out_dtype=torch.bfloat16) for b in batches]
    torch.cuda.synchronize()
    for rounds in range(2):
        got = [attention.prefill(*b, scale=S, out_dtype=torch.bfloat16, inputs_stable=True)
               for b in batches]
        torch.cuda.synchronize()
        for i, (g, w) in enumerate(zip(got, want)):
            assert torch.equal(g, w), f"batch {i}, round {rounds}"
    attention.sync(0)


def test_inputs_stable_launch_writes_what_the_previous_launch_reads():
    """Write after read across launches: launch B (stable inputs) writes its
    output into the buffer launch A reads as q.  B may start while A runs, so
    its first store waits for A; A must see the old q."""
    qa, ka, va = (t.to(DEV) for t in _inputs(6, 20, 1500, seed=95))
    qb, kb, vb = (t.to(DEV) for t in _inputs(6, 20, 1500, seed=96))
    want_a = attention.prefill(qa, ka, va, scale=S, out_dtype=torch.bfloat16)
    want_b = attention.prefill(qb, kb, vb, scale=S, out_dtype=torch.bfloat16)
    qa_keep = qa.clone()
    torch.cuda.synchronize()
    got_a = attention.prefill(qa, ka, va, scale=S, out_dtype=torch.bfloat16, inputs_stable=True)
    attention.prefill(qb, kb, vb, scale=S, out=qa, inputs_stable=True)  # overwrites A's q
    torch.cuda.synchronize()
    assert torch.equal(got_a, want_a)
    assert torch.equal(qa, want_b)
    assert not torch.equal(qa, qa_keep)
    attention.sync(0)


@pytest.mark.parametrize("stable", [False, True])
def test_prefill_reads_the_preceding_prefill_output(stable):
    """Read after write: launch B's q is launch A's output, with no flag on B
    (B waits for A before its first load).  With the flag on A only, A still
    waits for the kernel before it before storing."""
    q, k, v = (t.to(DEV) for t in _inputs(6, 20, 1500, seed=97))
    torch.cuda.synchronize()  # the flag on A: nothing pending writes A's inputs
    a = attention.prefill(q, k, v, scale=S, out_dtype=torch.bfloat16, inputs_stable=stable)
    b = attention.prefill(a, k, v, scale=S, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    a_ref = attention.prefill(q, k, v, scale=S, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    b_ref = attention.prefill(a_ref.clone(), k, v, scale=S, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(a, a_ref) and torch.equal(b, b_ref)
    attention.sync(0)


def test_inputs_stable_varlen_and_staged_operands():
    """varlen with the flag equals varlen without; f32 operands (staged by the
    library, so the flag does not apply to the kernel) likewise."""
    lengths = workloads.ragged_lengths()[:64]
    q, k, v, cu = workloads.ragged_inputs(lengths, device=DEV)
    want = attention.varlen(q, k, v, cu, scale=S, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    got = [attention.varlen(q, k, v, cu, scale=S, out_dtype=torch.bfloat16, inputs_stable=True)
           for _ in range(3)]
    torch.cuda.synchronize()
    for g in got:
        assert torch.equal(g, want)
    qf, kf, vf = (t.float().to(DEV) for t in _inputs(2, 6, 700, seed=98))
    want = attention.prefill(qf, kf, vf, scale=S)
    got = attention.prefill(qf, kf, vf, scale=S, inputs_stable=True)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    attention.sync(0)


# ------------------------------------------------ scores that grow after a unit's first block
# Inputs that plant, in later key blocks, keys aligned with chosen queries, so
# a row's maximum jumps by ~`alpha * 2.9` log2 units (|q|^2 ~ 16, scale 1/8)
# while every other row sees a random jump of std ~`alpha * 0.36`.  Each jump
# past 8 moves the row's reference and rescales O in tensor memory; at alpha
# 60 the ordinary keys then sit ~170 log2 units below the reference, where the
# polynomial exp2 (FMA-pipe share of a full block) must clamp its argument
# and still give ~0.


def _growth_inputs(B, H, N, alpha, dtype=torch.bfloat16, seed=0, first_key=300, count=40):
    q, k, v = _inputs(B, H, N, dtype=torch.float32, seed=seed)
    rows = torch.arange(0, min(N, 4 * count), 4)[:count]
    keys = first_key + torch.arange(len(rows)) * 7 % max(1, N - first_key)
    k[:, :, keys] = alpha * q[:, :, rows]
    return q.to(dtype), k.to(dtype), v.to(dtype)


@pytest.mark.parametrize("alpha", [10.0, 60.0])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tc_growth_after_first_block(oracle, alpha, dtype):
    q, k, v = _growth_inputs(2, 3, 700, alpha, dtype=dtype, seed=int(alpha))
    ref = oracle_encoder(oracle, q, k, v, S)
    out, lse = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S, with_lse=True)
    assert_bf16_close(f32np(out), ref, f"growth alpha={alpha}")
    # The planted rows are dominated by one key, whose 16-bit P carries a
    # rounding of up to 2^-8 relative: their LSE may differ from the exact one
    # by up to ln(1 + 2^-8) < 4e-3 (as for a causal row with one visible key).
    err = rowsum_error(f32np(q).reshape(6, 700, 64), f32np(k).reshape(6, 700, 64), S,
                       f32np(lse).reshape(6, 700))
    assert err <= 4e-3, f"LSE off by {err:.2e}"


@pytest.mark.parametrize("alpha", [10.0, 60.0])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tc_growth_rowsums(alpha, dtype):
    """After large jumps of the reference the applied weights of every row
    still sum to 1 (V = ones): the rescales of O in tensor memory and of the
    row sum stay consistent, where a lost or doubled correction would be off
    by orders of magnitude.  The bar is 5e-5, not the 1e-6 of ordinary rows:
    after a jump the remaining keys weigh 2^-20 or less of the running O,
    and the tensor core adds such products to its accumulator with less than
    f32 precision while the f32 row sum keeps more of them (measured up to
    1.7e-5 on these inputs)."""
    q, k, _ = _growth_inputs(2, 4, 1500, alpha, dtype=dtype, seed=3 + int(alpha), first_key=600)
    ones = torch.ones(2, 4, 1500, 64, dtype=dtype)
    out = attention.prefill(q.to(DEV), k.to(DEV), ones.to(DEV), scale=S)
    err = (out.double() - 1.0).abs().max().item()
    assert err <= 5e-5, f"row sums off by {err:.2e}"


@pytest.mark.parametrize("layout", ["all_token", "kt", "fused"])
def test_tc_growth_layouts(oracle, layout):
    """Large jumps under each operand layout."""
    B, H, N = 2, 4, 520
    q, k, v = _growth_inputs(B, H, N, 60.0, seed=77, first_key=260)
    ref = oracle_encoder(oracle, q, k, v, S)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    kw = dict(scale=S)
    if layout == "all_token":
        qd, kd, vd = (t.transpose(1, 2).contiguous() for t in (qd, kd, vd))
        kw.update(q_layout="token", k_layout="token", v_layout="token")
    elif layout == "kt":
        kd = kd.transpose(-1, -2).contiguous()
        kw.update(k_layout="kt")
    else:  # views of one fused projection output (B, N, 3, H, 64)
        qkv = torch.stack([t.transpose(1, 2) for t in (qd, kd, vd)], dim=2).contiguous()
        qd, kd, vd = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        kw.update(q_layout="token", k_layout="token", v_layout="token")
    out = attention.prefill(qd, kd, vd, **kw)
    assert_bf16_close(f32np(out), ref, layout)


def test_tc_growth_causal(oracle):
    B, H, Nq, off, cap = 1, 3, 300, 148, 448
    q, k, v = _growth_inputs(B, H, cap, 60.0, seed=78, first_key=200)
    q = q[:, :, :Nq].contiguous()
    kv = off + Nq
    out = attention.prefill(q.to(DEV), k.to(DEV), v.to(DEV), scale=S, causal=True, q_offset=off,
                            kv_len=kv)
    ref, _ = oracle.naive_attention_f64(f32np(q), f32np(k)[:, :, :kv], f32np(v)[:, :, :kv],
                                        scale=S, causal=True, q_offset=off)
    assert_bf16_close(f32np(out), ref, "causal growth")


def test_tc_growth_varlen(oracle):
    lengths = [700, 129, 1000, 300]
    q, k, v, cu = workloads.ragged_inputs(lengths, heads=4, seed=79)
    q, k, v = q.float(), k.float(), v.float()
    for s, (a, b) in enumerate(zip(cu[:-1], cu[1:])):
        n = b - a
        if n > 300:  # keys past the first block aligned with early queries of the same segment
            rows = torch.arange(a, a + 120, 4)
            keys = a + 260 + (torch.arange(len(rows)) * 11) % (n - 260)
            k[keys] = 60.0 * q[rows]
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    out = attention.varlen(q.to(DEV), k.to(DEV), v.to(DEV), cu, scale=S)
    refs = _oracle_ragged(oracle, q, k, v, cu, range(len(lengths)))
    for s, ref in refs.items():
        assert_bf16_close(f32np(out[cu[s]:cu[s + 1]]), ref, f"segment {s}")
