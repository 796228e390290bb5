"""Paged KV cache: host page bookkeeping (CPU) and the paged decode, append
and copy-on-write fork on the GPU against the oracle's restated decode
(xattn_head, flash_attn.rs:602-696) over each beam's own key history."""

import numpy as np
import pytest
import torch

from ffai_b200.kvcache import PAGE_KEYS, PagePlanner
from helpers import assert_f32_close

DEV = "cuda:0"


# ----------------------------------------------------------------- host (CPU)
def test_planner_takes_a_page_per_64_keys():
    pl = PagePlanner(beams=3, max_pages=4, num_pages=12)
    for step in range(130):
        assert pl.plan_append() == []
        pl.commit_append()
    # 130 keys -> 3 pages per beam, all distinct
    pages = pl.table[:, :3]
    assert (pages >= 0).all() and len(set(pages.ravel().tolist())) == 9
    assert (pl.table[:, 3] == -1).all()
    assert sorted(pl.free) == sorted(set(range(12)) - set(pages.ravel().tolist()))


def test_planner_fork_shares_then_copies_on_write():
    pl = PagePlanner(beams=2, max_pages=3, num_pages=8)
    for _ in range(70):            # one full page + 6 keys
        pl.plan_append()
        pl.commit_append()
    full0, part0 = pl.table[0, 0], pl.table[0, 1]
    pl.reorder([0, 0])             # both beams continue beam 0
    assert pl.refs[full0] == 2 and pl.refs[part0] == 2
    assert pl.refs[pl.table[1, 0]] == 2  # beam 1's old pages were released
    copies = pl.plan_append()      # the first writer copies the shared partial page;
    assert len(copies) == 1        # the last one keeps the original
    src, dst = copies[0]
    assert src == part0 and dst != part0
    assert pl.table[0, 1] == dst and pl.table[1, 1] == part0
    assert pl.refs[part0] == 1 and pl.refs[dst] == 1
    assert pl.table[0, 0] == pl.table[1, 0] == full0   # full pages stay shared


def test_planner_reports_exhaustion():
    pl = PagePlanner(beams=2, max_pages=1, num_pages=2)
    for _ in range(PAGE_KEYS):
        pl.plan_append()
        pl.commit_append()
    with pytest.raises(ValueError):
        pl.plan_append()
    pl2 = PagePlanner(beams=3, max_pages=2, num_pages=2)
    with pytest.raises(MemoryError):
        pl2.plan_append()


# ----------------------------------------------------------------- device (GPU)
def _oracle_rows(oracle, q, ks, vs, scale):
    """q (R, 64) f32; ks[r], vs[r] (L_r, 64) f32 -> (R, 64) via xattn_rows per row."""
    out = np.zeros((q.shape[0], 64), np.float32)
    for r in range(q.shape[0]):
        L = ks[r].shape[0]
        if L == 0:
            continue
        kt = np.ascontiguousarray(ks[r].T[None])
        out[r] = oracle.xattn_rows(q[r:r + 1] * np.float32(scale), kt, vs[r][None], threads=1)[0]
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_paged_decode_matches_oracle(oracle, dtype):
    from ffai_b200.kvcache import decode_paged
    B, H, max_pages, num_pages = 5, 12, 8, 48
    lens = [1, 63, 64, 129, 448]
    g = torch.Generator().manual_seed(7)
    kp = torch.randn(num_pages, H, PAGE_KEYS, 64, generator=g).to(dtype)
    vp = torch.randn(num_pages, H, PAGE_KEYS, 64, generator=g).to(dtype)
    perm = torch.randperm(num_pages, generator=g)[:B * max_pages].view(B, max_pages)
    table = perm.to(torch.int32)
    q = torch.randn(B, H, 1, 64, generator=g) * 0.5
    out = decode_paged(q.to(DEV), kp.to(DEV), vp.to(DEV), table.to(DEV),
                       torch.tensor(lens, dtype=torch.int32).to(DEV), scale=0.125)
    kf, vf = kp.float().numpy(), vp.float().numpy()
    ks, vs, qs = [], [], []
    for b in range(B):
        pages = table[b, :(lens[b] + 63) // 64].tolist()
        kb = np.concatenate([kf[p] for p in pages], axis=1)[:, :lens[b]]  # (H, L, 64)
        vb = np.concatenate([vf[p] for p in pages], axis=1)[:, :lens[b]]
        for h in range(H):
            ks.append(kb[h]); vs.append(vb[h]); qs.append(q[b, h, 0].numpy())
    ref = _oracle_rows(oracle, np.stack(qs), ks, vs, 0.125)
    assert_f32_close(out.reshape(B * H, 64).cpu().numpy(), ref, f"paged {dtype}")


@pytest.mark.gpu
def test_append_and_fork_match_each_beams_history(oracle):
    """Append keys step by step, fork beams mid-page (copy on write), and
    check every beam's decode against its own dense history."""
    from ffai_b200.kvcache import PagedKVCache
    B, H = 4, 6
    cache = PagedKVCache(B, H, max_len=256, dtype=torch.bfloat16, device=0)
    g = torch.Generator().manual_seed(11)
    hist_k = [[] for _ in range(B)]
    hist_v = [[] for _ in range(B)]

    def step():
        kn = torch.randn(B, H, 64, generator=g).to(torch.bfloat16)
        vn = torch.randn(B, H, 64, generator=g).to(torch.bfloat16)
        cache.append(kn.to(DEV), vn.to(DEV))
        for b in range(B):
            hist_k[b].append(kn[b].float().numpy())
            hist_v[b].append(vn[b].float().numpy())

    def check(tag):
        q = torch.randn(B, H, 1, 64, generator=g) * 0.5
        out = cache.decode(q.to(DEV), scale=0.125)
        ks, vs, qs = [], [], []
        for b in range(B):
            kb = np.stack(hist_k[b], axis=1)  # (H, L, 64)
            vb = np.stack(hist_v[b], axis=1)
            for h in range(H):
                ks.append(kb[h]); vs.append(vb[h]); qs.append(q[b, h, 0].numpy())
        ref = _oracle_rows(oracle, np.stack(qs), ks, vs, 0.125)
        assert_f32_close(out.reshape(B * H, 64).cpu().numpy(), ref, tag)

    for _ in range(70):
        step()
    check("after 70 appends")
    order = [0, 0, 2, 1]                       # beam search: 0 forks, 3 dropped
    cache.reorder(order)
    hist_k = [list(hist_k[s]) for s in order]
    hist_v = [list(hist_v[s]) for s in order]
    for _ in range(60):                        # beams now diverge, crossing a page edge
        step()
    check("after fork and 60 more")
    assert cache.plan.refs.max() <= B


@pytest.mark.gpu
def test_bad_page_id_is_reported_not_read():
    from ffai_b200 import attention
    from ffai_b200.kvcache import decode_paged
    B, H, num_pages = 2, 4, 4
    kp = torch.zeros(num_pages, H, PAGE_KEYS, 64, dtype=torch.bfloat16, device=DEV)
    table = torch.tensor([[0, 1], [2, 99]], dtype=torch.int32, device=DEV)  # 99: outside
    lens = torch.tensor([100, 100], dtype=torch.int32, device=DEV)
    q = torch.zeros(B, H, 1, 64, device=DEV)
    decode_paged(q, kp, kp, table, lens)
    with pytest.raises(attention.AttnError) as e:
        attention.sync(0)
    assert e.value.status == -1  # FFAI_ATTN_ERR_INVALID


@pytest.mark.gpu
def test_length_above_the_bound_is_reported():
    from ffai_b200 import attention
    from ffai_b200.kvcache import decode_paged
    B, H, num_pages = 2, 4, 8
    kp = torch.zeros(num_pages, H, PAGE_KEYS, 64, dtype=torch.bfloat16, device=DEV)
    table = torch.arange(8, dtype=torch.int32, device=DEV).view(2, 4)
    lens = torch.tensor([200, 100], dtype=torch.int32, device=DEV)
    q = torch.zeros(B, H, 1, 64, device=DEV)
    decode_paged(q, kp, kp, table, lens, kv_bound=64)   # bound below beam 0's length
    with pytest.raises(attention.AttnError) as e:
        attention.sync(0)
    assert e.value.status == -1
