"""The C-ABI library loads and exports every entry point include/mla_b200.h
declares; host-side validation returns the documented status codes. CPU only:
no call here reaches a kernel."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import PKG, ROOT

HEADER = ROOT / "include" / "mla_b200.h"
LIB = PKG / "lib" / "libmla_b200.so"


def declared_symbols():
    text = HEADER.read_text()
    return re.findall(r"MLA_API\s+[\w\s\*]+?\b(mla_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    assert LIB.exists(), "build the library first: python mla-cuda_b200/build.py"
    return ctypes.CDLL(str(LIB))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("mla_q_absorbed", "mla_attention", "mla_q_absorbed_workspace_size",
              "mla_attention_workspace_size", "mla_abi_version", "mla_status_string",
              "mla_last_error_message"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in {HEADER.name} but not exported"


def test_abi_version(lib):
    text = HEADER.read_text()
    ver = int(re.search(r"#define MLA_B200_ABI_VERSION (\d+)", text).group(1))
    assert lib.mla_abi_version() == ver


def test_status_strings(lib):
    lib.mla_status_string.restype = ctypes.c_char_p
    assert lib.mla_status_string(0) == b"ok"
    assert lib.mla_status_string(3) == b"workspace too small"


def _q_ws(lib, *args):
    lib.mla_q_absorbed_workspace_size.restype = ctypes.c_int
    out = ctypes.c_size_t(0)
    st = lib.mla_q_absorbed_workspace_size(*[ctypes.c_int(a) for a in args[:2]],
                                           *[ctypes.c_int64(a) for a in args[2:]], ctypes.byref(out))
    return st, out.value


def test_q_validation_codes(lib):
    lib.mla_last_error_message.restype = ctypes.c_char_p
    st, _ = _q_ws(lib, 0, 0, 1, 1, 7168, 1536, 128, 128, 63, 512)   # odd rope
    assert st == 1 and b"rope" in lib.mla_last_error_message()
    st, _ = _q_ws(lib, 9, 0, 1, 1, 7168, 1536, 128, 128, 64, 512)   # bad dtype
    assert st == 2
    st, _ = _q_ws(lib, 0, 7, 1, 1, 7168, 1536, 128, 128, 64, 512)   # bad precision
    assert st == 2
    st, n = _q_ws(lib, 0, 0, 128, 1, 7168, 1536, 128, 128, 64, 512)
    assert st == 0 and n > 128 * 1536 * 4


def test_attention_validation_codes(lib):
    lib.mla_attention_workspace_size.restype = ctypes.c_int
    out = ctypes.c_size_t(0)
    i64 = ctypes.c_int64
    # causal with sk < sq is rejected
    st = lib.mla_attention_workspace_size(0, 0, i64(1), i64(8), i64(4), i64(128), i64(512), i64(64),
                                          i64(128), 1, ctypes.byref(out))
    assert st == 1
    st = lib.mla_attention_workspace_size(0, 0, i64(128), i64(1), i64(4989), i64(128), i64(512), i64(64),
                                          i64(128), 0, ctypes.byref(out))
    assert st == 0
    # the exact path stages one fp32 score per (row, key)
    assert out.value >= 128 * 128 * 4989 * 4


def test_attention_rejects_missing_workspace(lib):
    lib.mla_attention.restype = ctypes.c_int
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    fake = vp(0x1000)
    st = lib.mla_attention(0, 0, fake, fake, fake, fake, fake, i64(1), i64(1), i64(16), i64(128), i64(512),
                           i64(64), i64(128), ctypes.c_double(13.8), 0, fake, vp(0), ctypes.c_size_t(0),
                           vp(0))
    assert st == 3   # MLA_ERR_WORKSPACE, detected before any device work


def _size_t():
    return ctypes.c_size_t(0)


def test_pack_q_weights_size_and_validation(lib):
    f = lib.mla_pack_q_weights_size
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int] + [ctypes.c_int64] * 6 + [ctypes.POINTER(ctypes.c_size_t)]
    n = _size_t()
    assert f(0, 7168, 1536, 128, 128, 64, 512, ctypes.byref(n)) == 0
    # bf16 copies of W_q_a, W_q_b, W_uk, each part 256-byte aligned
    expect = 7168 * 1536 * 2 + 1536 * 128 * 192 * 2 + 128 * 128 * 512 * 2
    assert expect <= n.value < expect + 3 * 256
    assert f(3, 7168, 1536, 128, 128, 64, 512, ctypes.byref(n)) == 2      # bf16 storage: MLA_ERR_UNSUPPORTED
    assert f(0, 7168, 1536, 128, 128, 63, 512, ctypes.byref(n)) == 1      # odd rope: invalid argument
    g = lib.mla_pack_q_weights
    g.restype = ctypes.c_int
    g.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 6 + [ctypes.c_void_p, ctypes.c_size_t,
                                                                                     ctypes.c_void_p]
    assert g(0, None, None, None, 7168, 1536, 128, 128, 64, 512, None, 0, None) == 1   # null pointers


def test_q_absorbed_packed_validation(lib):
    f = lib.mla_q_absorbed_packed_workspace_size
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int] + [ctypes.c_int64] * 8 + [ctypes.POINTER(ctypes.c_size_t)]
    n = _size_t()
    assert f(0, 0, 1, 7168, 1536, 128, 128, 64, 512, ctypes.byref(n)) == 0 and n.value == 0   # empty batch
    assert f(2, 4, 1, 7168, 1536, 128, 128, 64, 512, ctypes.byref(n)) == 2                   # fp16: unsupported


def test_kv_cache_write_validation(lib):
    f = lib.mla_kv_cache_write_workspace_size
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_int] + [ctypes.c_int64] * 5 + [ctypes.POINTER(ctypes.c_size_t)]
    n = _size_t()
    assert f(0, 0, 0, 1, 7168, 512, 64, ctypes.byref(n)) == 0 and n.value == 0
    assert f(1, 0, 4, 1, 7168, 512, 64, ctypes.byref(n)) == 2      # fp64: unsupported
    assert f(0, 0, 4, 1, 7168, 2048, 64, ctypes.byref(n)) == 2     # kv_rank above 1024
    assert f(0, 7, 4, 1, 7168, 512, 64, ctypes.byref(n)) == 2      # unknown precision
    w = lib.mla_kv_cache_write
    w.restype = ctypes.c_int
    w.argtypes = ([ctypes.c_int, ctypes.c_int] + [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 6
                  + [ctypes.c_double] + [ctypes.c_void_p] * 3 + [ctypes.c_size_t, ctypes.c_void_p])
    assert w(0, 0, None, None, None, None, None, 1, 1, 7168, 512, 64, 16, 1e-6, None, None, None, 0, None) == 1


def test_status_strings_cover_every_code(lib):
    lib.mla_status_string.restype = ctypes.c_char_p
    names = [lib.mla_status_string(c).decode() for c in range(6)]
    assert names[5] == "device-side failure" and len(set(names)) == 6


def test_pack_uv_weights_and_packed_attention_validation(lib):
    f = lib.mla_pack_uv_weights_size
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int] + [ctypes.c_int64] * 3 + [ctypes.POINTER(ctypes.c_size_t)]
    n = _size_t()
    assert f(0, 128, 128, 512, ctypes.byref(n)) == 0 and n.value == 128 * 128 * 512 * 2   # one bf16 copy
    assert f(3, 128, 128, 512, ctypes.byref(n)) == 2      # bf16 storage: MLA_ERR_UNSUPPORTED
    assert f(0, 0, 128, 512, ctypes.byref(n)) == 1        # empty: invalid argument
    g = lib.mla_pack_uv_weights
    g.restype = ctypes.c_int
    g.argtypes = [ctypes.c_int, ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_void_p, ctypes.c_size_t,
                                                                           ctypes.c_void_p]
    assert g(0, None, 128, 128, 512, None, 0, None) == 1  # null pointers
    a = lib.mla_attention_packed_uv
    a.restype = ctypes.c_int
    a.argtypes = ([ctypes.c_int] + [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 7
                  + [ctypes.c_double, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p])
    args = [None] * 5 + [4, 1, 4989, 128, 512, 64, 128, 13.856, 0, None, None, 0, None]
    assert a(2, *args) == 2                                # fp16 storage: unsupported
    bad = list(args)
    bad[8] = 256                                           # kv_rank 256: not a tensor-core shape
    assert a(0, *bad) == 2
    assert a(0, *args) == 1                                # covered shape, null W_uv_packed: invalid argument
