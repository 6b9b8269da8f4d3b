"""Host-side behaviour of the drop-in module mla_custom_cuda (CPU only)."""
from __future__ import annotations

import pytest
import torch

import mla_custom_cuda as mcc


def test_module_surface_matches_reference():
    # the reference binds exactly these two names (mla_kernels.cu:1688-1692)
    assert callable(mcc.q_absorbed) and callable(mcc.mla_attention)
    assert mcc.library_path().endswith("libmla_b200.so")
    assert mcc.abi_version() >= 1


def test_cpu_tensors_are_rejected_no_fallback():
    qa = torch.zeros(1, 1, 128, 512)
    qr = torch.zeros(1, 1, 128, 64)
    ck = torch.zeros(1, 4, 512)
    pe = torch.zeros(1, 4, 64)
    wuv = torch.zeros(128, 128, 512)
    with pytest.raises(RuntimeError, match="CUDA"):
        mcc.mla_attention(qa, qr, ck, pe, wuv, 192 ** 0.5)
    x = torch.zeros(1, 1, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        mcc.q_absorbed(x, torch.zeros(64, 32), torch.ones(32), torch.zeros(32, 4 * 24), torch.zeros(4, 16, 32),
                       torch.zeros(1, dtype=torch.long), 16, 8, 1e-6)


def test_precision_setting():
    assert mcc.get_precision() in ("exact", "tensor")
    old = mcc.get_precision()
    mcc.set_precision("tensor")
    assert mcc.get_precision() == "tensor"
    mcc.set_precision(old)
    with pytest.raises(ValueError):
        mcc.set_precision("fp8")


def test_packing_rejects_cpu_and_16bit_weights():
    with pytest.raises(RuntimeError, match="CUDA"):
        mcc.pack_q_weights(torch.zeros(64, 32), torch.zeros(32, 96), torch.zeros(4, 16, 32), 16, 8)
