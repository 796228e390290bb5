"""Device-resident paged KV cache for beam-search decoding.

Replaces the reference's decoder cache handling: the self-attention cache
grows by Tensor::cat every step and is re-split and transposed for the fused
kernel (DecoderState, text_decoder.rs:1226-1243, :657-664, :841), and beams
are forked by cloning caches (TextDecoder::save/restore, :1363-1381).  Here a
layer's K and V live in two page pools on the device; each beam owns a row of
a block table; a step appends in place (ffai_kv_append) and decodes straight
from the pages (ffai_attn_decode_paged).  Forking beams shares their full
pages; a shared, partly filled last page is copied before either beam writes
to it (copy on write).

The page bookkeeping (free list, reference counts, copy-on-write) is host
logic with no device access, in `PagePlanner`, so it is testable on its own.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _abi
from .attention import _DT, _check, _ptr, _stream, context

PAGE_KEYS = 64


class PagePlanner:
    """Host bookkeeping of one paged cache: which page holds which keys.

    table[b, i] is the page of beam b's keys [64 i, 64 (i + 1)), -1 if none;
    lens[b] the beam's live keys; refs[p] how many table entries name page p.
    """

    def __init__(self, beams: int, max_pages: int, num_pages: int):
        self.max_pages = max_pages
        self.num_pages = num_pages
        self.table = np.full((beams, max_pages), -1, np.int32)
        self.lens = np.zeros(beams, np.int64)
        self.refs = np.zeros(num_pages, np.int64)
        self.free = list(range(num_pages - 1, -1, -1))

    def _take(self) -> int:
        if not self.free:
            raise MemoryError("paged KV cache: no free page")
        p = self.free.pop()
        self.refs[p] = 1
        return p

    def _drop(self, p: int) -> None:
        self.refs[p] -= 1
        if self.refs[p] == 0:
            self.free.append(int(p))

    def plan_append(self):
        """Make every beam's next key position writable and private.

        Returns the (src, dst) page copies that must run before the append
        (copy on write of shared, partly filled pages).  New pages for a
        beam at a page boundary are simply taken from the free list."""
        copies = []
        for b in range(self.table.shape[0]):
            pos = int(self.lens[b])
            slot = pos // PAGE_KEYS
            if slot >= self.max_pages:
                raise ValueError(f"beam {b}: cache is full ({self.max_pages} pages)")
            page = int(self.table[b, slot])
            if page < 0:
                self.table[b, slot] = self._take()
            elif self.refs[page] > 1:
                fresh = self._take()
                copies.append((page, fresh))
                self._drop(page)
                self.table[b, slot] = fresh
        return copies

    def commit_append(self) -> None:
        self.lens += 1

    def reorder(self, src_beams) -> None:
        """Beam b continues beam src_beams[b]'s history (beam-search step):
        the new rows share the old rows' pages."""
        src = np.asarray(src_beams, np.int64)
        table = self.table[src].copy()
        for p in table[table >= 0]:
            self.refs[p] += 1
        for p in self.table[self.table >= 0]:
            self._drop(int(p))
        self.table = table
        self.lens = self.lens[src].copy()


class PagedKVCache:
    """One decoder layer's paged K/V for `beams` sequences of `heads` heads."""

    def __init__(self, beams: int, heads: int, max_len: int, num_pages: int | None = None,
                 dtype=torch.bfloat16, device: int = 0):
        self.beams, self.heads = beams, heads
        self.max_pages = (max_len + PAGE_KEYS - 1) // PAGE_KEYS
        self.num_pages = num_pages or beams * self.max_pages
        self.device = torch.device("cuda", device)
        shape = (self.num_pages, heads, PAGE_KEYS, 64)
        self.k = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v = torch.zeros(shape, dtype=dtype, device=self.device)
        self.plan = PagePlanner(beams, self.max_pages, self.num_pages)
        self.table = torch.full((beams, self.max_pages), -1, dtype=torch.int32, device=self.device)
        self.lens = torch.zeros(beams, dtype=torch.int32, device=self.device)
        self.dtype = dtype

    def _desc(self, **kw):
        return _abi.new_desc(batch=self.beams, heads=self.heads, q_len=1, kv_len=0,
                             kv_dtype=_DT[self.dtype], **kw)

    def _push_table(self):
        self.table.copy_(torch.from_numpy(self.plan.table), non_blocking=False)

    def append(self, k_new, v_new) -> None:
        """k_new, v_new: (beams, heads, 64) of the cache dtype, on the device."""
        copies = self.plan.plan_append()
        ctx = context(self.device.index)
        lib = _abi.load()
        d = self._desc()
        if copies:
            src = torch.tensor([c[0] for c in copies], dtype=torch.int32, device=self.device)
            dst = torch.tensor([c[1] for c in copies], dtype=torch.int32, device=self.device)
            st = lib.ffai_kv_copy_pages(ctx, ctypes.byref(d), _ptr(self.k), _ptr(self.v),
                                        self.num_pages, _ptr(src), _ptr(dst), len(copies),
                                        _stream(self.device))
            _check(st, ctx)
        self._push_table()
        st = lib.ffai_kv_append(ctx, ctypes.byref(d), _ptr(self.k), _ptr(self.v), self.num_pages,
                                _ptr(self.table), _ptr(self.lens), self.max_pages,
                                _ptr(k_new.contiguous()), _ptr(v_new.contiguous()),
                                _stream(self.device))
        _check(st, ctx)
        self.plan.commit_append()

    def reorder(self, src_beams) -> None:
        """Beam-search reordering: beam b continues beam src_beams[b]."""
        self.plan.reorder(src_beams)
        self._push_table()
        self.lens.copy_(torch.from_numpy(self.plan.lens.astype(np.int32)))

    def decode(self, q, *, scale: float = 1.0, out_dtype=torch.float32, with_lse=False, out=None):
        """q (beams, heads, 1, 64) against each beam's live keys."""
        return decode_paged(q, self.k, self.v, self.table, self.lens, scale=scale,
                            out_dtype=out_dtype, with_lse=with_lse, out=out)


def decode_paged(q, k_pool, v_pool, block_table, seq_lens, *, scale: float = 1.0, kv_bound=0,
                 out_dtype=torch.float32, with_lse=False, out=None):
    """ffai_attn_decode_paged on torch tensors: q (B,H,1,64); pools
    (num_pages, H, 64, 64); block_table (B, max_pages) and seq_lens (B,)
    int32 on the device."""
    dev = q.device
    B, H = q.shape[0], q.shape[1]
    if out is None:
        out = torch.empty((B, H, 1, 64), dtype=out_dtype, device=dev)
    lse = torch.empty((B, H), dtype=torch.float32, device=dev) if with_lse else None
    d = _abi.new_desc(batch=B, heads=H, q_len=1, kv_len=kv_bound, q_dtype=_DT[q.dtype],
                      kv_dtype=_DT[k_pool.dtype], out_dtype=_DT[out.dtype], scale=scale)
    ctx = context(dev.index)
    st = _abi.load().ffai_attn_decode_paged(ctx, ctypes.byref(d), _ptr(q), _ptr(k_pool),
                                            _ptr(v_pool), k_pool.shape[0], _ptr(block_table),
                                            _ptr(seq_lens), block_table.shape[1], _ptr(out),
                                            _ptr(lse), _stream(dev))
    _check(st, ctx)
    return (out, lse) if with_lse else out
