"""GPU parity of the tensor-core path (MLA_PREC_TENSOR): tcgen05 attention with
bf16 operands (fp16 for fp16 storage) and fp32 accumulation. Tolerance
rel-L2 <= 2e-2 against the fp64 reference (the bound stated for the
tensor-core paths); typical error is ~3e-3 for bf16 operands.
"""
from __future__ import annotations

import glob
import os

import pytest
import torch

from conftest import GOLDEN, load_golden, rel_l2, sampled
import mla_configs as mc
from oracle import mla_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = 2e-2
ATTN_FILES = sorted(os.path.basename(p) for p in glob.glob(str(GOLDEN / "attn_*.npz")))


@pytest.fixture(scope="module")
def mcc():
    import mla_custom_cuda
    return mla_custom_cuda


def _ins(d, dtype=torch.float32):
    B, Sq, Sk, seed = int(d["B"]), int(d["Sq"]), int(d["Sk"]), int(d["seed"])
    return [t.to(DEV, dtype) for t in mc.attention_inputs(B, Sq, Sk, seed=seed)]


@pytest.mark.parametrize("fname", ATTN_FILES)
def test_tc_attention_fp32_storage(mcc, fname):
    d = load_golden(fname)
    out = mcc.mla_attention_ex(*_ins(d), mc.SCALE, precision="tensor")
    assert out.dtype == torch.float32 and not torch.isnan(out).any()
    err = rel_l2(sampled(out, d["out64_idx"]), d["out64_val"])
    assert err < TOL, err
    assert err < 8e-3, f"bf16-operand error {err} is far above the expected ~3e-3"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("fname", ["attn_1x1x4999.npz", "attn_2x3x1000.npz", "attn_5x13x71.npz"])
def test_tc_attention_16bit_storage(mcc, dtype, fname):
    d = load_golden(fname)
    ins = _ins(d, dtype)
    out = mcc.mla_attention_ex(*ins, mc.SCALE, precision="tensor")
    assert out.dtype == dtype
    ref = orc.mla_attention(*(t.double().cpu() for t in ins), scale=mc.SCALE)
    assert rel_l2(out.cpu(), ref) < TOL


@pytest.mark.parametrize("fname", ["causal_2x4x37.npz", "causal_1x8x300.npz"])
def test_tc_attention_causal(mcc, fname):
    d = load_golden(fname)
    out = mcc.mla_attention_ex(*_ins(d), mc.SCALE, causal=True, precision="tensor")
    assert rel_l2(out.cpu(), d["out64_full"]) < TOL


def test_tc_lazy_rescale_path(mcc):
    """Later keys with much larger scores force the running-max rescale of O."""
    qa, qr, ck, pe, wuv = (t.to(DEV) for t in mc.attention_inputs(2, 1, 3000, seed=77))
    ramp = torch.linspace(0.2, 3.0, 3000, device=DEV)[None, :, None]
    ck = ck * ramp
    pe = pe * ramp
    out = mcc.mla_attention_ex(qa, qr, ck, pe, wuv, mc.SCALE, precision="tensor")
    ref = orc.mla_attention(*(t.double().cpu() for t in (qa, qr, ck, pe, wuv)), scale=mc.SCALE)
    assert rel_l2(out.cpu(), ref) < TOL


def test_tc_is_deterministic(mcc):
    ins = [t.to(DEV) for t in mc.attention_inputs(3, 2, 2500, seed=5)]
    a = mcc.mla_attention_ex(*ins, mc.SCALE, precision="tensor")
    b = mcc.mla_attention_ex(*ins, mc.SCALE, precision="tensor")
    assert torch.equal(a, b)


@pytest.mark.parametrize("cfg", ["c1", "c2", "c3"])
def test_tc_full_size_configs_match_exact_path(mcc, cfg):
    """Full configuration sizes: the tensor-core path against the exact path on
    the same seeded inputs (size-independent check), and two sequences against
    the fp64 CPU oracle."""
    w = mc.CONFIGS[cfg]
    g = torch.Generator(device=DEV).manual_seed(11)
    B, Sq, Sk = w.batch, w.sq, w.sk
    qa = torch.randn(B, Sq, 128, 512, device=DEV, generator=g) * 0.2
    qr = torch.randn(B, Sq, 128, 64, device=DEV, generator=g) * 0.8
    ck = torch.randn(B, Sk, 512, device=DEV, generator=g)
    pe = torch.randn(B, Sk, 64, device=DEV, generator=g)
    wuv = torch.randn(128, 128, 512, device=DEV, generator=g) * 0.02
    tc = mcc.mla_attention_ex(qa, qr, ck, pe, wuv, w.scale, causal=w.causal, precision="tensor")
    ex = mcc.mla_attention_ex(qa, qr, ck, pe, wuv, w.scale, causal=w.causal, precision="exact")
    assert rel_l2(tc, ex) < TOL
    for b in (0, B - 1):
        ref = orc.mla_attention(*(t[b:b + 1].double().cpu() for t in (qa, qr, ck, pe)), wuv.double().cpu(),
                                scale=w.scale, causal=w.causal)
        assert rel_l2(tc[b:b + 1].cpu(), ref) < TOL


def test_tc_box_scale_bf16_config(mcc):
    """Config c4 shape per GPU (128 of the 1024-sequence box job), bf16 storage,
    against the fp32 exact path on the fp32 draws."""
    w = mc.CONFIGS["c4"]
    g = torch.Generator(device=DEV).manual_seed(4)
    B = 128
    f32 = [torch.randn(*s, device=DEV, generator=g) * sc for s, sc in
           (((B, 1, 128, 512), 0.2), ((B, 1, 128, 64), 0.8), ((B, w.sk, 512), 1.0), ((B, w.sk, 64), 1.0),
            ((128, 128, 512), 0.02))]
    out = mcc.mla_attention_ex(*(t.bfloat16() for t in f32), w.scale, precision="tensor")
    ref = mcc.mla_attention_ex(*f32, w.scale, precision="exact")
    assert out.dtype == torch.bfloat16
    assert rel_l2(out.float(), ref) < TOL


@pytest.mark.parametrize("B,Sq", [(1, 1), (5, 3), (20, 1), (128, 1), (200, 1)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_tc_q_absorbed_vs_oracle(mcc, B, Sq, dtype):
    """Tensor-core Q-prep (tcgen05 projections, tf32 or bf16/fp16 operands)
    against the fp64 oracle on the same (storage-rounded) inputs."""
    w = mc.Workload("q", B, Sq, 8, dtype=dtype)
    t = mc.make_inputs(w, seed=B * 10 + Sq)
    g = {k: v.to(DEV) for k, v in t.items()}
    qa, qr = mcc.q_absorbed_ex(g["x"], g["W_q_a"], g["q_norm_w"], g["W_q_b"], g["W_uk"], g["positions"],
                               mc.NOPE, mc.ROPE, mc.EPS, precision="tensor")
    assert qa.dtype == dtype and qr.dtype == dtype
    t64 = {k: (v.double() if v.is_floating_point() else v) for k, v in t.items()}
    ra, rr = orc.q_absorbed(t64["x"], t64["W_q_a"], t64["q_norm_w"], t64["W_q_b"], t64["W_uk"], t64["positions"])
    assert rel_l2(qa.cpu(), ra) < TOL
    assert rel_l2(qr.cpu(), rr) < TOL


def test_tc_forward_c0_vs_reference(mcc):
    """Whole layer forward at config 0, tensor precision, against the reference's fp64 output."""
    d = load_golden("forward_c0.npz")
    t = {k: v.to(DEV) for k, v in mc.make_inputs(mc.CONFIGS["c0"], seed=0).items()}
    qa, qr = mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                               mc.NOPE, mc.ROPE, mc.EPS, precision="tensor")
    out = mcc.mla_attention_ex(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], mc.SCALE, precision="tensor")
    assert rel_l2(qa.cpu(), d["qa64_full"]) < TOL
    assert rel_l2(out.cpu(), d["out64_full"]) < TOL


@pytest.mark.parametrize("precision", ["exact", "tensor"])
@pytest.mark.parametrize("parts", [2, 4])
def test_key_shards_partial_and_combine(mcc, precision, parts):
    """Key sharding emulated on one GPU: partial attention per key shard plus the
    log-sum-exp merge equals attention over all keys; lse matches the oracle."""
    from mla_custom_cuda import sharding
    qa, qr, ck, pe, wuv = (t.to(DEV) for t in mc.attention_inputs(3, 2, 2000, seed=8))
    outs, lses = [], []
    for r in range(parts):
        k0, k1 = sharding.key_shard(2000, r, parts)
        o, l = mcc.mla_attention_partial(qa, qr, ck[:, k0:k1], pe[:, k0:k1], wuv, mc.SCALE, precision=precision)
        outs.append(o)
        lses.append(l)
    merged, L = mcc.lse_combine(torch.stack(outs), torch.stack(lses))
    full = mcc.mla_attention_ex(qa, qr, ck, pe, wuv, mc.SCALE, precision=precision)
    tol = 1e-5 if precision == "exact" else TOL
    assert rel_l2(merged, full) < tol
    _, ref_lse = orc.mla_attention_partial(*(t.double().cpu() for t in (qa, qr, ck, pe, wuv)), mc.SCALE)
    assert rel_l2(L.cpu(), ref_lse) < (1e-6 if precision == "exact" else 1e-3)


@pytest.mark.parametrize("B,Sq", [(1, 1), (5, 3), (128, 1), (200, 1)])
def test_packed_q_absorbed_vs_oracle(mcc, B, Sq):
    """Q-prep from bf16-packed weights (fp32 storage, tensor precision) against the
    fp64 oracle, and against the unpacked tensor-precision path."""
    w = mc.Workload("q", B, Sq, 8)
    t = mc.make_inputs(w, seed=B * 7 + Sq)
    g = {k: v.to(DEV) for k, v in t.items()}
    packed = mcc.pack_q_weights(g["W_q_a"], g["W_q_b"], g["W_uk"], mc.NOPE, mc.ROPE)
    qa, qr = mcc.q_absorbed_packed(g["x"], packed, g["q_norm_w"], g["positions"], mc.EPS)
    assert qa.dtype == torch.float32 and qa.shape == (B, Sq, 128, 512) and qr.shape == (B, Sq, 128, 64)
    t64 = {k: (v.double() if v.is_floating_point() else v) for k, v in t.items()}
    ra, rr = orc.q_absorbed(t64["x"], t64["W_q_a"], t64["q_norm_w"], t64["W_q_b"], t64["W_uk"], t64["positions"])
    assert rel_l2(qa.cpu(), ra) < TOL
    assert rel_l2(qr.cpu(), rr) < TOL
    qa2, qr2 = mcc.q_absorbed_ex(g["x"], g["W_q_a"], g["q_norm_w"], g["W_q_b"], g["W_uk"], g["positions"],
                                 mc.NOPE, mc.ROPE, mc.EPS, precision="tensor")
    assert rel_l2(qa, qa2) < TOL


@pytest.mark.parametrize("fname", ATTN_FILES)
def test_packed_uv_attention_vs_golden(mcc, fname):
    """Attention with W_uv packed to bf16 (bf16 context, kind::f16 projection,
    fp32 output) against the reference goldens, and against the unpacked
    tensor-precision path (same decode kernel; only the 3d operands differ)."""
    d = load_golden(fname)
    qa, qr, ck, pe, wuv = _ins(d)
    packed = mcc.pack_uv_weights(wuv)
    assert packed.buf.dtype == torch.bfloat16 and packed.buf.numel() == wuv.numel()
    out = mcc.mla_attention_packed(qa, qr, ck, pe, packed, mc.SCALE)
    assert out.dtype == torch.float32 and not torch.isnan(out).any()
    assert rel_l2(sampled(out, d["out64_idx"]), d["out64_val"]) < TOL
    ref = mcc.mla_attention_ex(qa, qr, ck, pe, wuv, mc.SCALE, precision="tensor")
    assert rel_l2(out, ref) < 1e-2


def test_packed_uv_attention_causal_and_rejects(mcc):
    """Causal multi-query decode through the packed path against the oracle;
    16-bit operands are rejected (the packing is for fp32 storage)."""
    qa, qr, ck, pe, wuv = (t.to(DEV) for t in mc.attention_inputs(2, 3, 700, seed=41))
    packed = mcc.pack_uv_weights(wuv)
    out = mcc.mla_attention_packed(qa, qr, ck, pe, packed, mc.SCALE, causal=True)
    ref = orc.mla_attention(*(t.double().cpu() for t in (qa, qr, ck, pe, wuv)), mc.SCALE, True)
    assert rel_l2(out.cpu(), ref) < TOL
    with pytest.raises((RuntimeError, ValueError)):
        mcc.pack_uv_weights(wuv.to(torch.bfloat16))
    with pytest.raises((RuntimeError, ValueError)):
        mcc.mla_attention_packed(qa.half(), qr.half(), ck.half(), pe.half(), packed, mc.SCALE)
