"""The drop-in module driven exactly as the reference's own wrappers drive its
extension (exhaustive_benchmark_suite.py:261-265 split_wkv_b, :311-336
prepare_q_mla_absorbed_cuda / mla_attention_official_cuda, :393-397
cuda_fully_fused_mla_attention): W_uk and W_uv are non-contiguous slices of one
wkv_b [H, nope+v, kv_rank], every operand goes through .contiguous(), the
scale is sqrt(nope+rope), and q_absorbed / mla_attention are called
positionally with the default (exact) precision. The result is compared with
the reference's own outputs at config 0 (tests/golden/forward_c0.npz) with the
check_3d.py criterion (error < 5x the fp32-vs-fp64 noise) and rel-L2 <= 1e-5.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_l2
import mla_configs as mc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_reference_wrapper_call_pattern_config0():
    import mla_custom_cuda
    mla_custom_cuda.set_precision("exact")
    assert mla_custom_cuda.binding() == "extension", "the built C++ extension should carry the drop-in calls"
    d = load_golden("forward_c0.npz")
    t = {k: v.to(DEV) for k, v in mc.make_inputs(mc.CONFIGS["c0"], seed=0).items()}
    nope, rope = mc.NOPE, mc.ROPE
    wkv_b = torch.cat([t["W_uk"], t["W_uv"]], dim=1)              # [H, nope + v, kv_rank]
    W_uk, W_uv = wkv_b[:, :nope, :], wkv_b[:, nope:, :]           # split_wkv_b: views, not contiguous
    qa, qr = mla_custom_cuda.q_absorbed(t["x"], t["W_q_a"].contiguous(), t["q_norm_w"].contiguous(),
                                        t["W_q_b"].contiguous(), W_uk.contiguous(), t["positions"],
                                        nope, rope, mc.EPS)
    scale = float(nope + rope) ** 0.5
    out = mla_custom_cuda.mla_attention(qa.contiguous(), qr.contiguous(), t["c_kv"].contiguous(),
                                        t["pe_cache"].contiguous(), W_uv.contiguous(), scale)
    torch.cuda.synchronize()
    assert isinstance(qa, torch.Tensor) and qa.shape == (1, 1, 128, 512) and out.shape == (1, 1, 128, 128)
    ref64, ref32 = d["out64_full"], d["out32_full"]
    got = out.double().cpu().numpy()
    noise = np.abs(ref32 - ref64).max()
    assert np.abs(got - ref64).max() < 5 * max(noise, 1e-7)
    assert rel_l2(got, ref64) < 1e-5


def test_non_contiguous_views_are_accepted_directly():
    """The extension makes operands contiguous itself (mla_kernels.cu:610-615), so
    passing the split_wkv_b views without .contiguous() gives the same result."""
    import mla_custom_cuda
    qa, qr, ck, pe, wuv = (x.to(DEV) for x in mc.attention_inputs(2, 1, 300, seed=9))
    wkv_b = torch.cat([torch.zeros_like(wuv), wuv], dim=1)
    view = wkv_b[:, 128:, :]
    a = mla_custom_cuda.mla_attention(qa, qr, ck, pe, view, 192 ** 0.5)
    b = mla_custom_cuda.mla_attention(qa, qr, ck, pe, wuv.contiguous(), 192 ** 0.5)
    assert torch.equal(a, b)
