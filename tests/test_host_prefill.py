"""The host-buffer prefill entry (ffai_attn_prefill_host): the batch streamed
through the device in sequence chunks with copies and kernels overlapped on
the context's own streams.  Its output and lse equal the device entry's bit
for bit (the same kernel on the same operands), for batches that do and do not
divide into the chunks, with pinned and pageable host buffers."""

import pytest
import torch


def _inputs(B, H, N, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, H, N, 64, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, H, N, 64, generator=g) * 0.5).to(torch.bfloat16)
    v = torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16)
    return q, k, v


@pytest.mark.gpu
@pytest.mark.parametrize("B", [1, 3, 8, 11, 17])
@pytest.mark.parametrize("pinned", [True, False])
def test_host_prefill_matches_device_entry(B, pinned):
    from ffai_b200 import attention
    q, k, v = _inputs(B, 4, 200, seed=B)
    if pinned:
        q, k, v = q.pin_memory(), k.pin_memory(), v.pin_memory()
    lse = torch.empty(B, 4, 200, dtype=torch.float32, pin_memory=pinned)
    got = attention.prefill_host(q, k, v, device=0, scale=0.125, out_dtype=torch.bfloat16, lse=lse)
    want, want_lse = attention.prefill(q.cuda(), k.cuda(), v.cuda(), scale=0.125,
                                       out_dtype=torch.bfloat16, with_lse=True)
    assert torch.equal(got, want.cpu())
    assert torch.equal(lse, want_lse.cpu())


@pytest.mark.gpu
def test_host_prefill_repeated_calls_reuse_the_pipeline():
    # a second call with a different batch reuses the context's slots and streams
    from ffai_b200 import attention
    for B, seed in ((13, 1), (5, 2), (13, 3)):
        q, k, v = (t.pin_memory() for t in _inputs(B, 2, 130, seed))
        got = attention.prefill_host(q, k, v, device=0, scale=0.125, out_dtype=torch.float32)
        want = attention.prefill(q.cuda(), k.cuda(), v.cuda(), scale=0.125, out_dtype=torch.float32)
        assert torch.equal(got, want.cpu())
