"""The reference's PRODUCTION_SCENARIOS shapes (exhaustive_benchmark_suite.py:
78-173: decode, speculative decode and prefill chunks, all without a mask)
through the whole layer forward, in both precisions, checked on sampled rows
against the oracle: the first and last query of the first and last sequence.

Exact precision: rel-L2 <= 1e-5 against the reference's path run in fp32 on
those rows, and within 5x of that path's own error against fp64 (check_3d.py
criterion). Tensor precision: rel-L2 <= 2e-2 against fp64.
"""
from __future__ import annotations

import pytest
import torch

from conftest import rel_l2
import mla_configs as mc
from oracle import mla_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _oracle_rows(t, w, b, qs, dtype):
    """Oracle output of sequence b at query indices qs (each query needs only its
    own Q-prep row and all of the sequence's keys)."""
    s = {k: (v[b:b + 1].cpu() if k in ("x", "c_kv", "pe_cache") else v.cpu()) for k, v in t.items()}
    s = {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in s.items()}
    x = s["x"][:, qs]
    qa, qr = orc.q_absorbed(x, s["W_q_a"], s["q_norm_w"], s["W_q_b"], s["W_uk"], s["positions"][qs])
    return orc.mla_attention(qa, qr, s["c_kv"], s["pe_cache"], s["W_uv"], w.scale, False)


@pytest.mark.parametrize("precision", ["exact", "tensor"])
@pytest.mark.parametrize("name", sorted(mc.SCENARIOS))
def test_scenario_layer_forward(name, precision):
    import mla_custom_cuda as mcc
    w = mc.SCENARIOS[name]
    t = mc.make_inputs(w, device=DEV, gen="device", seed=3)
    qa, qr = mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                               w.nope, w.rope, mc.EPS, precision=precision)
    out = mcc.mla_attention_ex(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale, precision=precision)
    torch.cuda.synchronize()
    del qa, qr
    assert torch.isfinite(out).all()
    qs = sorted({0, w.sq - 1})
    for b in sorted({0, w.batch - 1}):
        got = out[b:b + 1, qs].cpu()
        ref64 = _oracle_rows(t, w, b, qs, torch.float64)
        if precision == "exact":
            ref32 = _oracle_rows(t, w, b, qs, torch.float32)
            assert rel_l2(got, ref32) < 1e-5
            assert rel_l2(got, ref64) < 5 * max(rel_l2(ref32, ref64), 1e-7)
        else:
            assert rel_l2(got, ref64) < 2e-2
    del out, t
    torch.cuda.empty_cache()
