"""The Whisper attention workloads this library is measured on, with seeded
synthetic inputs of their shapes and value distributions (no audio, weights
or dataset is read).

c1  Whisper-tiny encoder self-attention: B=1, H=6, N=1500, f32, seed 0,
    Q and K scaled by 0.5, scale 1/8 (the reference CPU kernel's own shape).
c2  Whisper-base encoder, batched: 8 segments, H=8, N=1500, bf16 N(0,1)*0.5.
c3  Whisper-small decode: 5 beams x 12 heads, q_len 1, bf16 cache of
    {1, 32, 128, 448} keys (self-attention) and 1500 keys (cross-attention);
    K, V ~ N(0,1), Q ~ N(0, 0.25).
c4  Whisper-large-v3 long-form: 64 segments (32 min / 30 s), H=20, N=1500, bf16.
c5  Ragged Whisper-medium: 256 segments, lengths U{200..1500}, H=16, packed.
"""

from __future__ import annotations

import dataclasses

import torch

HD = 64
SCALE = 0.125  # 1/sqrt(64): a power of two, exact in bf16


@dataclasses.dataclass(frozen=True)
class Encoder:
    name: str
    segments: int
    heads: int
    seq: int
    dtype: torch.dtype

    @property
    def flops(self) -> float:
        """4*B*H*N^2*d: QK^T and PV, 2 flops per multiply-add."""
        return 4.0 * self.segments * self.heads * self.seq * self.seq * HD


C1 = Encoder("whisper-tiny-encoder-c1", 1, 6, 1500, torch.float32)
C2 = Encoder("whisper-base-encoder-c2", 8, 8, 1500, torch.bfloat16)
C4 = Encoder("whisper-large-v3-longform-c4", 64, 20, 1500, torch.bfloat16)

C3_BEAMS, C3_HEADS = 5, 12
C3_SELF_KEYS = (1, 32, 128, 448)
C3_CROSS_KEYS = 1500
C5_SEGMENTS, C5_HEADS, C5_MIN, C5_MAX = 256, 16, 200, 1500


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def encoder_inputs(cfg: Encoder, seed: int = 0, device="cpu", segments: int | None = None,
                   first_segment: int = 0):
    """Q, K, V (B,H,N,64) of cfg.dtype; Q and K carry the 0.5 factor.

    Each segment is drawn from its own seed (seed*100003 + segment), so a
    shard of segments [first, first+B) is identical to the same rows of the
    full batch, whichever GPU generates it.
    """
    B = cfg.segments if segments is None else segments
    qs, ks, vs = [], [], []
    for s in range(first_segment, first_segment + B):
        g = _gen(seed * 100003 + s, device)
        shape = (1, cfg.heads, cfg.seq, HD)
        qs.append(torch.randn(shape, generator=g, device=device) * 0.5)
        ks.append(torch.randn(shape, generator=g, device=device) * 0.5)
        vs.append(torch.randn(shape, generator=g, device=device))
    q, k, v = torch.cat(qs), torch.cat(ks), torch.cat(vs)
    return q.to(cfg.dtype), k.to(cfg.dtype), v.to(cfg.dtype)


def decode_inputs(keys: int, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                  beams: int = C3_BEAMS, heads: int = C3_HEADS):
    """q (B,H,1,64) f32 ~ N(0,0.25); K, V (B,H,keys,64) cache of `dtype` ~ N(0,1)."""
    g = _gen(seed * 7919 + keys, device)
    q = torch.randn((beams, heads, 1, HD), generator=g, device=device) * 0.5
    k = torch.randn((beams, heads, keys, HD), generator=g, device=device)
    v = torch.randn((beams, heads, keys, HD), generator=g, device=device)
    return q, k.to(dtype), v.to(dtype)


def ragged_lengths(n: int = C5_SEGMENTS, lo: int = C5_MIN, hi: int = C5_MAX, seed: int = 0):
    g = _gen(seed, "cpu")
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


def ragged_inputs(lengths, heads: int = C5_HEADS, seed: int = 0, device="cpu",
                  dtype=torch.bfloat16):
    """Packed q, k, v (T,H,64) and cu_seqlens for segments of `lengths`."""
    T = int(sum(lengths))
    g = _gen(seed + 17, device)
    q = torch.randn((T, heads, HD), generator=g, device=device) * 0.5
    k = torch.randn((T, heads, HD), generator=g, device=device) * 0.5
    v = torch.randn((T, heads, HD), generator=g, device=device)
    cu = [0]
    for L in lengths:
        cu.append(cu[-1] + int(L))
    return q.to(dtype), k.to(dtype), v.to(dtype), cu


def ragged_segment_inputs(lengths, segments, heads: int = C5_HEADS, seed: int = 0, device="cpu",
                          dtype=torch.bfloat16):
    """Packed q, k, v (T,H,64) and cu_seqlens of the listed `segments` only.

    Segment s is drawn from its own seed (seed*100003 + s), so a rank that
    packs a subset gets the same values as any other packing of s."""
    qs, ks, vs, cu = [], [], [], [0]
    for s in segments:
        L = int(lengths[s])
        g = _gen(seed * 100003 + 7919 + s, device)
        qs.append(torch.randn((L, heads, HD), generator=g, device=device) * 0.5)
        ks.append(torch.randn((L, heads, HD), generator=g, device=device) * 0.5)
        vs.append(torch.randn((L, heads, HD), generator=g, device=device))
        cu.append(cu[-1] + L)
    q, k, v = torch.cat(qs), torch.cat(ks), torch.cat(vs)
    return q.to(dtype), k.to(dtype), v.to(dtype), cu


def ragged_flops(lengths, heads: int = C5_HEADS) -> float:
    return 4.0 * heads * HD * float(sum(int(L) * int(L) for L in lengths))
