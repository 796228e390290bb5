"""Generate the golden fixtures under tests/golden/ from the oracle.

The reference (Rust) cannot run in this image, and its own tests hold no
golden vectors for attention, so these fixtures are outputs of the oracle --
the C++ restatement of flash_attn.rs -- on seeded inputs.  They pin the oracle
build (tests/test_golden.py re-runs it and expects the same bits) and give
the GPU tests fixed expected outputs.  Inputs are regenerated from the seed
with numpy's PCG64 (platform-independent), so only outputs are stored.

    python tests/golden/make_golden.py     # rewrites tests/golden/*.npz
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

# name -> (kind, parameters).  Shapes are small versions of the workloads:
# encoder heads at ragged lengths around the 64/128/256-row block edges, the
# c3 decode rows (5 beams x 12 heads) at self- and cross-attention key counts,
# and a packed ragged batch.
CASES = {
    "encoder_f32_h2_n300": ("encoder", dict(heads=2, n=300, seed=11, bf16=False, scale=0.125)),
    "encoder_bf16_h3_n257": ("encoder", dict(heads=3, n=257, seed=12, bf16=True, scale=0.125)),
    "encoder_bf16_h1_n1500": ("encoder", dict(heads=1, n=1500, seed=13, bf16=True, scale=0.125)),
    "decode_bf16_r60_k32": ("decode", dict(rows=60, keys=32, seed=21, cache="bf16")),
    "decode_bf16_r60_k448": ("decode", dict(rows=60, keys=448, seed=22, cache="bf16")),
    "decode_f16_r12_k1500": ("decode", dict(rows=12, keys=1500, seed=23, cache="f16")),
    "decode_f32_r60_k129": ("decode", dict(rows=60, keys=129, seed=24, cache="f32")),
    "ragged_bf16_h2": ("ragged", dict(heads=2, lengths=(200, 333, 129, 256), seed=31,
                                      scale=0.125)),
}


def encoder_inputs(heads, n, seed, bf16, **_):
    from oracle import oracle
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((heads, n, 64)) * 0.5).astype(np.float32)
    k = (rng.standard_normal((heads, n, 64)) * 0.5).astype(np.float32)
    v = rng.standard_normal((heads, n, 64)).astype(np.float32)
    if bf16:
        q, k, v = oracle.bf16_round(q), oracle.bf16_round(k), oracle.bf16_round(v)
    return q, k, v


def decode_inputs(rows, keys, seed, cache, **_):
    """q (rows, 64) f32 ~ N(0, 0.25); K, V (rows, keys, 64) ~ N(0, 1) in `cache` precision."""
    from oracle import oracle
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((rows, 64)) * 0.5).astype(np.float32)
    k = rng.standard_normal((rows, keys, 64)).astype(np.float32)
    v = rng.standard_normal((rows, keys, 64)).astype(np.float32)
    rnd = {"bf16": oracle.bf16_round, "f16": oracle.f16_round, "f32": lambda x: x}[cache]
    return q, rnd(k), rnd(v)


def ragged_inputs(heads, lengths, seed, **_):
    """Packed token-major (T, heads, 64) bf16-rounded q, k, v and cu_seqlens."""
    from oracle import oracle
    rng = np.random.default_rng(seed)
    T = int(sum(lengths))
    q = oracle.bf16_round((rng.standard_normal((T, heads, 64)) * 0.5).astype(np.float32))
    k = oracle.bf16_round((rng.standard_normal((T, heads, 64)) * 0.5).astype(np.float32))
    v = oracle.bf16_round(rng.standard_normal((T, heads, 64)).astype(np.float32))
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    return q, k, v, cu


def expected(kind, p):
    """The oracle's output for one case."""
    from oracle import oracle
    if kind == "encoder":
        q, k, v = encoder_inputs(**p)
        return oracle.flash_rowmajor_k(q, k, v, p["scale"], threads=1)
    if kind == "decode":
        q, k, v = decode_inputs(**p)
        kt = np.ascontiguousarray(np.swapaxes(k, 1, 2))
        if p["cache"] == "f16":
            kb = kt.astype(np.float16).view(np.uint16)
            vb = v.astype(np.float16).view(np.uint16)
            return oracle.xattn_rows_f16(q, kb, vb, threads=1)
        return oracle.xattn_rows(q, kt, v, threads=1)
    if kind == "ragged":
        q, k, v, cu = ragged_inputs(**p)
        out = np.zeros_like(q)
        for s in range(len(cu) - 1):
            a, b = cu[s], cu[s + 1]
            hq = np.ascontiguousarray(np.swapaxes(q[a:b], 0, 1))  # (heads, L, 64)
            hk = np.ascontiguousarray(np.swapaxes(k[a:b], 0, 1))
            hv = np.ascontiguousarray(np.swapaxes(v[a:b], 0, 1))
            o = oracle.flash_rowmajor_k(hq, hk, hv, p["scale"], threads=1)
            out[a:b] = np.swapaxes(o, 0, 1)
        return out
    raise ValueError(kind)


def path(name):
    return os.path.join(HERE, name + ".npz")


def main():
    for name, (kind, p) in CASES.items():
        out = expected(kind, p)
        np.savez_compressed(path(name), out=out)
        print(f"{name}: {out.shape} -> {os.path.getsize(path(name))} bytes")


if __name__ == "__main__":
    main()
