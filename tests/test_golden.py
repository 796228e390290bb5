"""Golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py).

CPU: the oracle still produces the stored bits, and stays within 1e-5 of the
f64 textbook formula.  GPU: each CUDA path meets its tolerance against the
stored outputs through the C ABI.
"""

import os
import sys

import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, assert_f32_close

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_golden as G  # noqa: E402

DEV = "cuda:0"


def _golden(name):
    with np.load(G.path(name)) as z:
        return z["out"]


@pytest.mark.parametrize("name", list(G.CASES))
def test_oracle_reproduces_golden(oracle, name):
    kind, p = G.CASES[name]
    got = G.expected(kind, p)
    assert np.array_equal(got, _golden(name)), f"{name}: oracle output drifted"


@pytest.mark.parametrize("name", [n for n, (k, _) in G.CASES.items() if k != "ragged"])
def test_golden_vs_f64(oracle, name):
    kind, p = G.CASES[name]
    gold = _golden(name)
    if kind == "encoder":
        q, k, v = G.encoder_inputs(**p)
        ref, _ = oracle.naive_attention_f64(q, k, v, scale=p["scale"])
    else:
        q, k, v = G.decode_inputs(**p)
        ref, _ = oracle.naive_attention_f64(q[:, None, :], k, v)
        ref = ref[:, 0]
    assert_f32_close(gold, ref, name)


def _t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(G.CASES))
def test_cuda_matches_golden(name):
    from ffai_b200 import attention
    kind, p = G.CASES[name]
    gold = _golden(name)
    if kind == "encoder":
        q, k, v = (x[None] for x in G.encoder_inputs(**p))  # (1, H, N, 64)
        if p["bf16"]:
            out = attention.prefill(_t(q, torch.bfloat16), _t(k, torch.bfloat16),
                                    _t(v, torch.bfloat16), scale=p["scale"])
            assert_bf16_close(out[0].cpu().numpy(), gold, name)
        else:
            qd, kd, vd = (_t(x, torch.float32) for x in (q, k, v))
            out = attention.prefill(qd, kd, vd, scale=p["scale"], checked=True)
            assert_f32_close(out[0].cpu().numpy(), gold, name + " checked-f32")
            out = attention.prefill(qd, kd, vd, scale=p["scale"])
            # the tensor-core path rounds f32 operands to bf16 first
            assert_bf16_close(out[0].cpu().numpy(), gold, name + " bf16")
    elif kind == "decode":
        q, k, v = G.decode_inputs(**p)
        dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[p["cache"]]
        rows = p["rows"]
        out = attention.decode(_t(q.reshape(1, rows, 1, 64), torch.float32),
                               _t(k[None], dt), _t(v[None], dt))
        assert_f32_close(out.reshape(rows, 64).cpu().numpy(), gold, name)
    else:
        q, k, v, cu = G.ragged_inputs(**p)
        out = attention.varlen(_t(q, torch.bfloat16), _t(k, torch.bfloat16),
                               _t(v, torch.bfloat16), cu.tolist(), scale=p["scale"])
        assert_bf16_close(out.cpu().numpy(), gold, name)
