"""GPU parity of the exact-arithmetic path (MLA_PREC_EXACT) through the
drop-in module and its C ABI, against the reference's outputs (tests/golden/)
and the CPU oracle. These re-host the reference's own checks:
check_3d.py (11 tile-straddling shapes, error < 5x the fp32-vs-fp64 noise),
check_dtypes.py (fp32 1e-5, fp64 1e-13, fp16 3e-2 max-rel; output dtype kept)
and run_scenario's full-forward comparison (exhaustive_benchmark_suite.py:467-484).
"""
from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden, rel_l2, sampled
import mla_configs as mc
from oracle import mla_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATTN_FILES = sorted(os.path.basename(p) for p in glob.glob(str(GOLDEN / "attn_*.npz")))


@pytest.fixture(scope="module")
def mcc():
    import mla_custom_cuda
    mla_custom_cuda.set_precision("exact")
    return mla_custom_cuda


def _attn_inputs(d, dtype=torch.float32):
    B, Sq, Sk, seed = int(d["B"]), int(d["Sq"]), int(d["Sk"]), int(d["seed"])
    return [t.to(DEV, dtype) for t in mc.attention_inputs(B, Sq, Sk, seed=seed)]


@pytest.mark.parametrize("fname", ATTN_FILES)
def test_attention_fp32_shapes(mcc, fname):
    d = load_golden(fname)
    out = mcc.mla_attention(*_attn_inputs(d), mc.SCALE)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and tuple(out.shape) == tuple(d["out64_shape"])
    got = sampled(out, d["out64_idx"])
    ref = d["out64_val"]
    noise = np.abs(d["out32_val"] - ref).max()
    err = np.abs(got - ref).max()
    assert err < 5 * max(noise, 1e-6), (err, noise)          # check_3d.py:40-44
    assert rel_l2(got, ref) < 1e-5
    # the fp32 path (3xTF32 tensor-core contractions) keeps the accuracy of the
    # reference's own fp32 run: rel-L2 against fp64 within 2x of it
    assert rel_l2(got, ref) < 2 * max(rel_l2(d["out32_val"], ref), 1e-7)
    rows = out.double().reshape(-1, out.shape[-1]).sum(-1).cpu().numpy()
    np.testing.assert_allclose(rows, d["out64_rowsum"], rtol=1e-4, atol=1e-4 * np.abs(ref).max())


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.float64, 1e-13),
                                       (torch.float16, 3e-2), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("fname", ["attn_1x1x64.npz", "attn_1x1x16384.npz"])
def test_attention_dtypes(mcc, dtype, tol, fname):
    """check_dtypes.py:23-38: plain (Sk=64) and long (Sk=16384) paths per dtype."""
    d = load_golden(fname)
    ins = _attn_inputs(d, dtype)
    out = mcc.mla_attention(*ins, mc.SCALE)
    assert out.dtype == dtype
    if dtype in (torch.float32, torch.float64):
        ref = d["out64_val"]
    else:  # reference on the same rounded operands
        ref = sampled(orc.mla_attention(*(t.double().cpu() for t in ins), scale=mc.SCALE), d["out64_idx"])
    got = sampled(out, d["out64_idx"])
    assert np.abs(got - ref).max() / np.abs(ref).max() < tol


@pytest.mark.parametrize("fname", ["causal_2x4x37.npz", "causal_1x8x300.npz"])
def test_attention_causal(mcc, fname):
    d = load_golden(fname)
    out = mcc.mla_attention_ex(*_attn_inputs(d), mc.SCALE, causal=True)
    assert rel_l2(out.cpu(), d["out64_full"]) < 1e-5


def test_forward_c0_fp32(mcc):
    """Full layer forward at config 0 (B=1, Sk=256) against the reference."""
    d = load_golden("forward_c0.npz")
    t = {k: v.to(DEV) for k, v in mc.make_inputs(mc.CONFIGS["c0"], seed=0).items()}
    qa, qr = mcc.q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                            mc.NOPE, mc.ROPE, mc.EPS)
    out = mcc.mla_attention(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], mc.SCALE)
    assert rel_l2(qa.cpu(), d["qa64_full"]) < 1e-5
    assert rel_l2(qr.cpu(), d["qr64_full"]) < 1e-5
    assert rel_l2(out.cpu(), d["out64_full"]) < 1e-5


def test_forward_small_dims_fp64(mcc):
    d = load_golden("forward_small.npz")
    w = mc.Workload("small", 3, 2, 19, hidden=96, heads=4, q_lora=48, kv_rank=32, nope=16, rope=8, v_dim=24)
    t = {k: (v.to(DEV, torch.float64) if v.is_floating_point() else v.to(DEV))
         for k, v in mc.make_inputs(w, seed=3).items()}
    qa, qr = mcc.q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"], 16, 8,
                            mc.EPS)
    assert qa.dtype == torch.float64
    assert rel_l2(qa.cpu(), d["qa64_full"]) < 1e-12
    assert rel_l2(qr.cpu(), d["qr64_full"]) < 1e-11
    out = mcc.mla_attention(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale)
    assert rel_l2(out.cpu(), d["out64_full"]) < 1e-11


@pytest.mark.parametrize("B,Sq", [(1, 1), (5, 3), (20, 1)])
def test_q_absorbed_tile_shapes_vs_oracle(mcc, B, Sq):
    """Row counts on both sides of the 16-row and 128-row tiles, against the fp64 oracle."""
    w = mc.Workload("q", B, Sq, 8)
    t = mc.make_inputs(w, seed=B * 10 + Sq)
    g = {k: v.to(DEV) for k, v in t.items()}
    qa, qr = mcc.q_absorbed(g["x"], g["W_q_a"], g["q_norm_w"], g["W_q_b"], g["W_uk"], g["positions"],
                            mc.NOPE, mc.ROPE, mc.EPS)
    t64 = {k: (v.double() if v.is_floating_point() else v) for k, v in t.items()}
    ra, rr = orc.q_absorbed(t64["x"], t64["W_q_a"], t64["q_norm_w"], t64["W_q_b"], t64["W_uk"], t64["positions"])
    assert rel_l2(qa.cpu(), ra) < 1e-5
    assert rel_l2(qr.cpu(), rr) < 1e-5


def test_empty_and_zero_key_inputs(mcc):
    qa, qr, ck, pe, wuv = (t.to(DEV) for t in mc.attention_inputs(2, 1, 0, seed=1))
    out = mcc.mla_attention(qa, qr, ck, pe, wuv, mc.SCALE)
    assert out.shape == (2, 1, 128, 128) and bool((out == 0).all())
    qa, qr, ck, pe, wuv = (t.to(DEV) for t in mc.attention_inputs(0, 1, 8, seed=1))
    assert mcc.mla_attention(qa, qr, ck, pe, wuv, mc.SCALE).shape == (0, 1, 128, 128)


def test_shape_errors_raise_runtime_error(mcc):
    qa, qr, ck, pe, wuv = (t.to(DEV) for t in mc.attention_inputs(1, 1, 8, seed=1))
    with pytest.raises(RuntimeError):
        mcc.mla_attention(qa, qr, ck[:, :, :256], pe, wuv, mc.SCALE)
    t = {k: v.to(DEV) for k, v in mc.make_inputs(mc.Workload("e", 1, 2, 8), seed=0).items()}
    with pytest.raises(RuntimeError, match="positions"):
        mcc.q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"][:1],
                       mc.NOPE, mc.ROPE, mc.EPS)


def test_runs_on_the_current_stream(mcc):
    d = load_golden("attn_2x3x1000.npz")
    ins = _attn_inputs(d)
    ref = mcc.mla_attention(*ins, mc.SCALE)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = mcc.mla_attention(*ins, mc.SCALE)
    s.synchronize()
    assert torch.equal(out, ref)   # deterministic: no atomics on this path


def test_exact_fp32_past_the_score_limit_causal(mcc):
    """B*Sq*H*Sk above 2^31 (long causal prefill): the exact fp32 attention runs
    per block of queries, each on the keys its last query sees. Rows on both
    sides of the block boundary match the oracle (each row against its own
    visible keys)."""
    B, Sq, Sk = 1, 4096, 4200
    assert B * Sq * 128 * Sk >= 2 ** 31
    qa, qr, ck, pe, wuv = (t.to(DEV) for t in mc.attention_inputs(B, Sq, Sk, seed=17))
    out = mcc.mla_attention_ex(qa, qr, ck, pe, wuv, mc.SCALE, causal=True, precision="exact")
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    for q in (0, 2047, 2048, Sq - 1):
        keys = Sk - Sq + q + 1
        args = [qa[:, q:q + 1].cpu(), qr[:, q:q + 1].cpu(), ck[:, :keys].cpu(), pe[:, :keys].cpu(), wuv.cpu()]
        ref32 = orc.mla_attention(*args, mc.SCALE, False)
        ref64 = orc.mla_attention(*(a.double() for a in args), mc.SCALE, False)
        got = out[:, q:q + 1].cpu()
        assert rel_l2(got, ref32) < 1e-5
        assert rel_l2(got.double(), ref64) < 5 * max(rel_l2(ref32.double(), ref64), 1e-7)
