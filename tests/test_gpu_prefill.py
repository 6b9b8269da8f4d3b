"""GPU parity for prefill-like shapes (many query tokens per sequence, causal),
the reference's prefill / speculative scenarios run through the same entry
points: q_absorbed with a position per query index, and causal mla_attention
(query i of Sq attends keys 0 .. Sk-Sq+i). Checked against the fp64 oracle:
exact path rel-L2 <= 1e-5, tensor path <= 2e-2.
"""
from __future__ import annotations

import pytest
import torch

from conftest import rel_l2
import mla_configs as mc
from oracle import mla_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def mcc():
    import mla_custom_cuda
    return mla_custom_cuda


@pytest.mark.parametrize("precision,tol", [("exact", 1e-5), ("tensor", 2e-2)])
@pytest.mark.parametrize("B,Sq,Sk", [(1, 64, 512), (2, 128, 128), (1, 200, 1000)])
def test_causal_prefill_attention(mcc, precision, tol, B, Sq, Sk):
    ins = mc.attention_inputs(B, Sq, Sk, seed=7000 + B * 31 + Sq + Sk)
    ref = orc.mla_attention(*(t.double() for t in ins), mc.SCALE, causal=True)
    out = mcc.mla_attention_ex(*(t.to(DEV) for t in ins), mc.SCALE, causal=True, precision=precision)
    torch.cuda.synchronize()
    assert out.shape == ref.shape
    assert rel_l2(out.cpu(), ref) < tol


@pytest.mark.parametrize("precision,tol", [("exact", 1e-5), ("tensor", 2e-2)])
def test_prefill_q_absorbed(mcc, precision, tol):
    w = mc.Workload("prefill", 2, 96, 8)
    t = mc.make_inputs(w, seed=11)
    ra, rr = orc.q_absorbed(*(t[k].double() for k in ("x", "W_q_a", "q_norm_w", "W_q_b", "W_uk")), t["positions"])
    g = {k: v.to(DEV) for k, v in t.items()}
    qa, qr = mcc.q_absorbed_ex(g["x"], g["W_q_a"], g["q_norm_w"], g["W_q_b"], g["W_uk"], g["positions"],
                               mc.NOPE, mc.ROPE, mc.EPS, precision=precision)
    torch.cuda.synchronize()
    assert rel_l2(qa.cpu(), ra) < tol
    assert rel_l2(qr.cpu(), rr) < tol
