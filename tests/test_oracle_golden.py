"""The CPU oracle against the reference's own outputs (tests/golden/), CPU only.

Pins oracle/mla_oracle.py: fixtures were produced by the reference's
PyTorch functions (exhaustive_benchmark_suite.py:268-304) on the same seeded
inputs, by tests/golden/make_golden.py.
"""
from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, checksum, load_golden, rel_l2, sampled
import mla_configs as mc
from oracle import mla_oracle as orc

ATTN_FILES = sorted(os.path.basename(p) for p in glob.glob(str(GOLDEN / "attn_*.npz")))


@pytest.mark.parametrize("fname", ATTN_FILES)
def test_oracle_attention_matches_reference(fname):
    d = load_golden(fname)
    B, Sq, Sk, seed = int(d["B"]), int(d["Sq"]), int(d["Sk"]), int(d["seed"])
    ins = mc.attention_inputs(B, Sq, Sk, seed=seed)
    np.testing.assert_allclose(checksum(*ins), d["in_checksum"], rtol=1e-12)
    out64 = orc.mla_attention(*(t.double() for t in ins), scale=mc.SCALE)
    out32 = orc.mla_attention(*ins, scale=mc.SCALE)
    # fp64 oracle equals the fp64 reference to rounding; fp32 to fp32 noise
    np.testing.assert_allclose(sampled(out64, d["out64_idx"]), d["out64_val"], rtol=1e-10, atol=1e-11)
    np.testing.assert_allclose(out64.reshape(-1, out64.shape[-1]).sum(-1).numpy(), d["out64_rowsum"],
                               rtol=1e-9, atol=1e-9)
    assert rel_l2(sampled(out32, d["out32_idx"]), d["out32_val"]) < 2e-6


@pytest.mark.parametrize("fname", ["causal_2x4x37.npz", "causal_1x8x300.npz"])
def test_oracle_causal_matches_reference_prefixes(fname):
    d = load_golden(fname)
    B, Sq, Sk, seed = int(d["B"]), int(d["Sq"]), int(d["Sk"]), int(d["seed"])
    ins = mc.attention_inputs(B, Sq, Sk, seed=seed)
    np.testing.assert_allclose(checksum(*ins), d["in_checksum"], rtol=1e-12)
    out = orc.mla_attention(*(t.double() for t in ins), scale=mc.SCALE, causal=True)
    assert rel_l2(out, d["out64_full"]) < 1e-7


def test_oracle_causal_single_query_is_unmasked():
    ins = mc.attention_inputs(2, 1, 50, seed=11)
    a = orc.mla_attention(*(t.double() for t in ins), scale=mc.SCALE, causal=True)
    b = orc.mla_attention(*(t.double() for t in ins), scale=mc.SCALE, causal=False)
    assert torch.equal(a, b)


def test_oracle_forward_c0_matches_reference():
    d = load_golden("forward_c0.npz")
    t = mc.make_inputs(mc.CONFIGS["c0"], seed=0)
    np.testing.assert_allclose(
        checksum(*(t[k] for k in ("x", "W_q_a", "W_q_b", "W_uk", "W_uv", "c_kv", "pe_cache"))),
        d["in_checksum"], rtol=1e-12)
    t64 = {k: (v.double() if v.is_floating_point() else v) for k, v in t.items()}
    qa, qr = orc.q_absorbed(t64["x"], t64["W_q_a"], t64["q_norm_w"], t64["W_q_b"], t64["W_uk"],
                            t64["positions"])
    assert rel_l2(qa, d["qa64_full"]) < 1e-7
    assert rel_l2(qr, d["qr64_full"]) < 1e-7
    out = orc.mla_attention(qa, qr, t64["c_kv"], t64["pe_cache"], t64["W_uv"], mc.SCALE)
    assert rel_l2(out, d["out64_full"]) < 1e-7
    # fp32 oracle vs fp32 reference: same ATen ops, same rounding regime
    qa32, qr32 = orc.q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"])
    assert rel_l2(qa32, d["qa32_full"]) < 2e-6
    assert rel_l2(qr32, d["qr32_full"]) < 2e-6


def test_oracle_small_dims_match_reference():
    d = load_golden("forward_small.npz")
    w = mc.Workload("small", 3, 2, 19, hidden=96, heads=4, q_lora=48, kv_rank=32, nope=16, rope=8, v_dim=24)
    t = mc.make_inputs(w, seed=3)
    t64 = {k: (v.double() if v.is_floating_point() else v) for k, v in t.items()}
    qa, qr = orc.q_absorbed(t64["x"], t64["W_q_a"], t64["q_norm_w"], t64["W_q_b"], t64["W_uk"],
                            t64["positions"], nope_dim=16, rope_dim=8)
    assert rel_l2(qa, d["qa64_full"]) < 1e-12
    assert rel_l2(qr, d["qr64_full"]) < 1e-12
    out = orc.mla_attention(qa, qr, t64["c_kv"], t64["pe_cache"], t64["W_uv"], w.scale)
    assert rel_l2(out, d["out64_full"]) < 1e-12


def test_rope_inverse_frequencies_are_correctly_rounded():
    # The kernels build the RoPE table as float(10000 ** (2j/rope)) then 1/x; the
    # reference's torch expression must give the same bits (see qprep_exact.cu).
    for rope in (8, 16, 64, 128):
        t = torch.arange(0, rope, 2, dtype=torch.float32) / rope
        torch_inv = (1.0 / (10000 ** t)).numpy()
        mine = np.array([np.float32(1.0) / np.float32(10000.0 ** (2 * j / rope)) for j in range(rope // 2)],
                        dtype=np.float32)
        assert np.array_equal(torch_inv, mine)


def test_kv_cache_rows_compose_the_pinned_functions():
    """oracle.kv_cache_rows is the reference's rmsnorm and apply_rope (both pinned
    by the goldens above) applied to x @ W_kv_a."""
    from oracle import mla_oracle as orc
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 3, 64, generator=g, dtype=torch.float64)
    W = torch.randn(64, 40, generator=g, dtype=torch.float64)
    gain = torch.rand(32, generator=g, dtype=torch.float64)
    pos = torch.tensor([5, 6, 7])
    c, pe = orc.kv_cache_rows(x, W, gain, pos, kv_rank=32)
    kv = x @ W
    assert torch.equal(c, orc.rmsnorm(kv[..., :32], gain))
    assert torch.equal(pe, orc.apply_rope(kv[..., 32:].unsqueeze(2), pos, 8).squeeze(2))
