"""ffai_attn_decode_static: the decode entry point that allocates nothing.

Collected last (file name).  Each case runs the static-scratch entry twice in
a row (the second call relies on the first leaving every ticket at zero) and
compares both against ffai_attn_decode with the same split count, which runs
the same split kernel on the context's allocated workspace.
"""

import pytest
import torch

from ffai_b200 import attention, workloads

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

CASES = [
    # beams, heads, keys, cache dtype, k layout, num_splits
    (5, 12, 1500, torch.bfloat16, "heads", 12),
    (5, 12, 1500, torch.bfloat16, "kt", 0),
    (5, 12, 448, torch.float32, "kt", 0),
    (1, 20, 3000, torch.float16, "heads", 24),
    (5, 12, 37, torch.bfloat16, "heads", 3),
    (2, 6, 1, torch.bfloat16, "heads", 1),
]


@pytest.mark.parametrize("beams,heads,keys,dtype,layout,splits", CASES)
def test_static_matches_allocating_entry(beams, heads, keys, dtype, layout, splits):
    q, k, v = workloads.decode_inputs(keys, seed=40 + keys, dtype=dtype, beams=beams, heads=heads)
    qd, vd = q.to(DEV), v.to(DEV)
    kd = (k.transpose(-1, -2).contiguous() if layout == "kt" else k).to(DEV)
    ref, ref_lse = attention.decode(qd, kd, vd, k_layout=layout, num_splits=splits,
                                    with_lse=True, scale=0.125)
    for call in range(2):
        out, lse = attention.decode_static(qd, kd, vd, k_layout=layout, num_splits=splits,
                                           with_lse=True, scale=0.125)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"call {call}: output differs"
        assert torch.equal(lse, ref_lse), f"call {call}: lse differs"


def test_static_allocates_no_device_memory():
    q, k, v = workloads.decode_inputs(1500, seed=50)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out = torch.empty(5, 12, 1, 64, device=DEV)
    attention.decode_static(qd, kd, vd, num_splits=12, out=out)  # first call: module, symbol
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(5):
        attention.decode_static(qd, kd, vd, num_splits=12, out=out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_static_rejects_oversize_shapes():
    # 80 x 64 rows split 64 ways: 327680 (row, split) slots > 4096
    q, k, v = workloads.decode_inputs(128, seed=51, beams=80, heads=64)
    with pytest.raises(attention.AttnError) as e:
        attention.decode_static(q.to(DEV), k.to(DEV), v.to(DEV), num_splits=64)
    assert "static scratch" in str(e.value)
    # one split needs no scratch: any row count up to the grid limit is served
    out = attention.decode_static(q.to(DEV), k.to(DEV), v.to(DEV), num_splits=1)
    ref = attention.decode(q.to(DEV), k.to(DEV), v.to(DEV), num_splits=1)
    assert torch.equal(out, ref)
