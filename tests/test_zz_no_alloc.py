"""The allocation-free attention entry point, mla_attention_noalloc, through the C ABI.

It exists for callers that cannot allocate device memory when they call (a
server whose memory pool already owns the GPU, or code where cudaMalloc may not
be called): its workspace is a fixed device array inside the library. Checked
here against the ordinary tensor-core entry point on two calls in a row, which
also shows that the shared array carries nothing stale from one call to the
next. This file is named so that pytest collects it last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import rel_l2
import mla_configs as mc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = 2e-2   # tolerance of the tensor-core tests


@pytest.fixture(scope="module")
def lib():
    import mla_custom_cuda
    lib = mla_custom_cuda._lib
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    lib.mla_attention_noalloc.restype = ctypes.c_int
    lib.mla_attention_noalloc.argtypes = ([ctypes.c_int] + [vp] * 5 + [i64] * 7
                                          + [ctypes.c_double, ctypes.c_int, vp, vp])
    lib.mla_attention_noalloc_max_scratch.restype = ctypes.c_size_t
    lib.mla_last_error_message.restype = ctypes.c_char_p
    return lib


def _call(lib, ins, dtype_code, causal=False):
    qa, qr, ck, pe, wuv = ins
    B, Sq, H, R = qa.shape
    out = torch.empty((B, Sq, H, wuv.shape[1]), dtype=qa.dtype, device=DEV)
    st = lib.mla_attention_noalloc(dtype_code, qa.data_ptr(), qr.data_ptr(), ck.data_ptr(), pe.data_ptr(),
                                   wuv.data_ptr(), B, Sq, ck.shape[1], H, R, qr.shape[3], wuv.shape[1],
                                   mc.SCALE, int(causal), out.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.mla_last_error_message().decode()
    return out


def test_noalloc_matches_tensor_core_entry_point_twice(lib):
    import mla_custom_cuda as mcc
    cases = [((1, 1, 256), False), ((16, 2, 4999), True)]
    for (B, Sq, Sk), causal in cases:
        ins = [t.to(DEV) for t in mc.attention_inputs(B, Sq, Sk, seed=B + Sk)]
        got = _call(lib, ins, 0, causal)
        ref = mcc.mla_attention_ex(*ins, mc.SCALE, causal=causal, precision="tensor")
        torch.cuda.synchronize()
        assert not torch.isnan(got).any()
        assert rel_l2(got, ref) < TOL


def test_noalloc_rejects_shapes_beyond_the_fixed_scratch(lib):
    assert lib.mla_attention_noalloc_max_scratch() == 96 << 20
    st = lib.mla_attention_noalloc(0, None, None, None, None, None, 1024, 1, 4989, 128, 512, 64, 128,
                                   mc.SCALE, 0, None, None)
    assert st == 3   # MLA_ERR_WORKSPACE
    assert b"maximum" in lib.mla_last_error_message()
