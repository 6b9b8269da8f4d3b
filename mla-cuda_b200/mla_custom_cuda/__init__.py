"""Drop-in replacement of the reference's ``mla_custom_cuda`` extension module.

The reference builds ``mla_custom_cuda`` from ``mla_kernels.cu`` with pybind11
and exposes two functions (mla_kernels.cu:1688-1692):

    q_absorbed(x, W_q_a, q_norm_w, W_q_b, W_uk, positions, nope_dim, rope_dim, eps)
        -> [q_absorbed, q_rope]
    mla_attention(q_absorbed, q_rope, c_kv, pe_cache, W_uv, scale) -> out

This module keeps those names, positional signatures, return types and error
behaviour (shape errors raise ``RuntimeError``, like TORCH_CHECK) and runs the
B200 kernels of ``libmla_b200.so`` through its C ABI (include/mla_b200.h).
The four entry points q_absorbed / mla_attention (and their ``_ex`` forms) go
through the C++ torch extension ``mla_custom_cuda._C``, built by
``mla-cuda_b200/setup.py`` as the reference builds its own (setup.py:20-26);
when that extension has not been built they use ``ctypes`` on the same C ABI.
The other functions (key-shard partials and merge, weight packing, device
status, kernel timing) always use ``ctypes``.
Outputs and workspaces are allocated with torch's caching allocator on the
inputs' device, and all work is enqueued on torch's current stream, as in the
reference (mla_kernels.cu:664-667, :1528-1549).

There is no CPU or PyTorch fallback: importing this module fails if the
library is missing, and every call requires CUDA tensors.

Precision: the default, ``"exact"``, computes to the accuracy of the accumulate
dtype like the reference (fp64 for fp64 tensors, fp32 otherwise; fp32 runs its
contractions on the tensor cores in 3xTF32). ``"tensor"`` runs the
tcgen05 tensor-core kernels (bf16 operands, fp32 accumulation) where they cover
the shape. Select it with ``set_precision("tensor")``, the ``MLA_PRECISION``
environment variable, or the ``precision=`` argument of the ``*_ex`` calls.
"""
from __future__ import annotations

import ctypes
import math
import os
from pathlib import Path
from typing import List, Optional

import torch

__all__ = [
    "q_absorbed", "mla_attention", "q_absorbed_ex", "mla_attention_ex",
    "mla_attention_partial", "lse_combine",
    "set_precision", "get_precision", "library_path", "abi_version",
    "device_status", "clear_device_status", "check_device", "set_wait_limit_ns", "wait_selftest",
    "kernel_timing", "kv_cache_write", "pack_q_weights", "q_absorbed_packed", "PackedQWeights",
    "pack_uv_weights", "mla_attention_packed", "PackedUVWeights",
]

_LIB_PATH = Path(__file__).resolve().parent.parent / "lib" / "libmla_b200.so"

_DTYPE_CODES = {torch.float32: 0, torch.float64: 1, torch.float16: 2, torch.bfloat16: 3}
_PRECISIONS = {"exact": 0, "tensor": 1}

_c_i64 = ctypes.c_int64
_c_vp = ctypes.c_void_p
_c_size = ctypes.c_size_t


def _load() -> ctypes.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(
            f"mla_custom_cuda: {_LIB_PATH} is missing; build it with "
            f"`python mla-cuda_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(str(_LIB_PATH))
    lib.mla_abi_version.restype = ctypes.c_int
    lib.mla_status_string.restype = ctypes.c_char_p
    lib.mla_status_string.argtypes = [ctypes.c_int]
    lib.mla_last_error_message.restype = ctypes.c_char_p
    lib.mla_q_absorbed_workspace_size.restype = ctypes.c_int
    lib.mla_q_absorbed_workspace_size.argtypes = [ctypes.c_int, ctypes.c_int] + [_c_i64] * 8 + [
        ctypes.POINTER(_c_size)]
    lib.mla_q_absorbed.restype = ctypes.c_int
    lib.mla_q_absorbed.argtypes = ([ctypes.c_int, ctypes.c_int] + [_c_vp] * 6 + [_c_i64] * 8
                                   + [ctypes.c_double, _c_vp, _c_vp, _c_vp, _c_size, _c_vp])
    lib.mla_attention_workspace_size.restype = ctypes.c_int
    lib.mla_attention_workspace_size.argtypes = ([ctypes.c_int, ctypes.c_int] + [_c_i64] * 7
                                                 + [ctypes.c_int, ctypes.POINTER(_c_size)])
    lib.mla_attention.restype = ctypes.c_int
    lib.mla_attention.argtypes = ([ctypes.c_int, ctypes.c_int] + [_c_vp] * 5 + [_c_i64] * 7
                                  + [ctypes.c_double, ctypes.c_int, _c_vp, _c_vp, _c_size, _c_vp])
    lib.mla_attention_partial.restype = ctypes.c_int
    lib.mla_attention_partial.argtypes = ([ctypes.c_int, ctypes.c_int] + [_c_vp] * 5 + [_c_i64] * 7
                                          + [ctypes.c_double, _c_vp, _c_vp, _c_vp, _c_size, _c_vp])
    lib.mla_lse_combine.restype = ctypes.c_int
    lib.mla_lse_combine.argtypes = [ctypes.c_int] + [_c_i64] * 3 + [_c_vp] * 5
    lib.mla_device_status.restype = ctypes.c_int
    lib.mla_device_status.argtypes = [_c_vp, ctypes.POINTER(ctypes.c_int)]
    lib.mla_device_status_clear.restype = ctypes.c_int
    lib.mla_device_status_clear.argtypes = [_c_vp]
    lib.mla_set_wait_limit_ns.restype = ctypes.c_int
    lib.mla_set_wait_limit_ns.argtypes = [ctypes.c_uint64, _c_vp]
    lib.mla_wait_selftest.restype = ctypes.c_int
    lib.mla_wait_selftest.argtypes = [_c_vp]
    lib.mla_pack_q_weights_size.restype = ctypes.c_int
    lib.mla_pack_q_weights_size.argtypes = [ctypes.c_int] + [_c_i64] * 6 + [ctypes.POINTER(_c_size)]
    lib.mla_pack_q_weights.restype = ctypes.c_int
    lib.mla_pack_q_weights.argtypes = [ctypes.c_int] + [_c_vp] * 3 + [_c_i64] * 6 + [_c_vp, _c_size, _c_vp]
    lib.mla_q_absorbed_packed_workspace_size.restype = ctypes.c_int
    lib.mla_q_absorbed_packed_workspace_size.argtypes = [ctypes.c_int] + [_c_i64] * 8 + [ctypes.POINTER(_c_size)]
    lib.mla_q_absorbed_packed.restype = ctypes.c_int
    lib.mla_q_absorbed_packed.argtypes = ([ctypes.c_int] + [_c_vp] * 4 + [_c_i64] * 8
                                          + [ctypes.c_double, _c_vp, _c_vp, _c_vp, _c_size, _c_vp])
    lib.mla_kv_cache_write_workspace_size.restype = ctypes.c_int
    lib.mla_kv_cache_write_workspace_size.argtypes = [ctypes.c_int, ctypes.c_int] + [_c_i64] * 5 + [
        ctypes.POINTER(_c_size)]
    lib.mla_kv_cache_write.restype = ctypes.c_int
    lib.mla_kv_cache_write.argtypes = ([ctypes.c_int, ctypes.c_int] + [_c_vp] * 5 + [_c_i64] * 6
                                       + [ctypes.c_double, _c_vp, _c_vp, _c_vp, _c_size, _c_vp])
    lib.mla_pack_uv_weights_size.restype = ctypes.c_int
    lib.mla_pack_uv_weights_size.argtypes = [ctypes.c_int] + [_c_i64] * 3 + [ctypes.POINTER(_c_size)]
    lib.mla_pack_uv_weights.restype = ctypes.c_int
    lib.mla_pack_uv_weights.argtypes = [ctypes.c_int, _c_vp] + [_c_i64] * 3 + [_c_vp, _c_size, _c_vp]
    lib.mla_attention_packed_uv.restype = ctypes.c_int
    lib.mla_attention_packed_uv.argtypes = ([ctypes.c_int] + [_c_vp] * 5 + [_c_i64] * 7
                                            + [ctypes.c_double, ctypes.c_int, _c_vp, _c_vp, _c_size, _c_vp])
    lib.mla_timing_enable.restype = ctypes.c_int
    lib.mla_timing_enable.argtypes = [ctypes.c_int]
    lib.mla_timing_read.restype = ctypes.c_int
    lib.mla_timing_read.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]
    return lib


_lib = _load()
try:   # the C++ extension over the same library (optional; ctypes otherwise)
    from . import _C  # noqa: E402
except ImportError:
    _C = None
# MLA_CHECK=1: after every call, wait for the stream and raise RuntimeError if a
# kernel recorded a device-side failure (costs a synchronisation per call).
_checked = os.environ.get("MLA_CHECK", "0").strip() not in ("", "0")
_precision = os.environ.get("MLA_PRECISION", "exact").strip().lower()
if _precision not in _PRECISIONS:
    raise ImportError(f"mla_custom_cuda: MLA_PRECISION must be one of {sorted(_PRECISIONS)}")


def library_path() -> str:
    """Path of the loaded C-ABI library."""
    return str(_LIB_PATH)


def binding() -> str:
    """How q_absorbed / mla_attention reach the library: "extension" or "ctypes"."""
    return "extension" if _C is not None else "ctypes"


def abi_version() -> int:
    return int(_lib.mla_abi_version())


def set_precision(precision: str) -> None:
    """Default arithmetic of later calls: "exact" or "tensor"."""
    global _precision
    p = precision.strip().lower()
    if p not in _PRECISIONS:
        raise ValueError(f"precision must be one of {sorted(_PRECISIONS)}, got {precision!r}")
    _precision = p


def get_precision() -> str:
    return _precision


def _stream_of(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(device=None) -> int:
    """Waits for the current stream of `device` and returns the device-side
    failure code of the library's kernels there (0 = none). A non-zero code
    means a kernel gave up on a bounded wait; the outputs of that call are
    invalid. The code stays set until clear_device_status()."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    code = ctypes.c_int(0)
    with torch.cuda.device(device):
        st = _lib.mla_device_status(_stream_of(device), ctypes.byref(code))
    if st not in (0, 5):   # 5 = MLA_ERR_DEVICE: reported through the code
        _raise_status(st, "device_status")
    return int(code.value)


def check_device(device=None) -> None:
    """Raises RuntimeError if a kernel recorded a device-side failure on `device`."""
    code = device_status(device)
    if code:
        raise RuntimeError(f"mla_custom_cuda: device-side failure code {code}: "
                           f"{_lib.mla_last_error_message().decode(errors='replace')}")


def clear_device_status(device=None) -> None:
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(device):
        _raise_status(_lib.mla_device_status_clear(_stream_of(device)), "clear_device_status")


def set_wait_limit_ns(ns: int, device=None) -> None:
    """Bound on every mbarrier wait of later kernel launches on `device` (0 restores
    the default of 2 s)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(device):
        _raise_status(_lib.mla_set_wait_limit_ns(int(ns), _stream_of(device)), "set_wait_limit_ns")


def wait_selftest(device=None) -> None:
    """Launches a kernel whose single bounded wait is on a barrier nothing
    completes; after the wait limit it records code 900 in the device status."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(device):
        _raise_status(_lib.mla_wait_selftest(_stream_of(device)), "wait_selftest")


def kernel_timing(enable: Optional[bool] = None):
    """Device time of the tensor-core decode-attention kernel alone.

    kernel_timing(True) starts recording an event pair around each of its
    launches; kernel_timing() returns (total_ms, launches) since the last read;
    kernel_timing(False) stops. Not for use inside CUDA graph capture."""
    if enable is not None:
        _raise_status(_lib.mla_timing_enable(int(bool(enable))), "kernel_timing")
        return None
    ms, n = ctypes.c_double(0.0), ctypes.c_int64(0)
    _raise_status(_lib.mla_timing_read(ctypes.byref(ms), ctypes.byref(n)), "kernel_timing")
    return float(ms.value), int(n.value)


def _after_call(device) -> None:
    if _checked:
        check_device(device)


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _raise_status(st: int, what: str) -> None:
    if st != 0:
        detail = _lib.mla_last_error_message().decode(errors="replace")
        name = _lib.mla_status_string(st).decode(errors="replace")
        raise RuntimeError(f"{what}: {name}: {detail}")


def _prec_code(precision: Optional[str]) -> int:
    p = _precision if precision is None else precision.strip().lower()
    if p not in _PRECISIONS:
        raise ValueError(f"precision must be one of {sorted(_PRECISIONS)}, got {precision!r}")
    return _PRECISIONS[p]


def _prec_name(precision: Optional[str]) -> str:
    p = _precision if precision is None else precision.strip().lower()
    if p not in _PRECISIONS:
        raise ValueError(f"precision must be one of {sorted(_PRECISIONS)}, got {precision!r}")
    return p


def _float_operands(name_tensors, device=None):
    dtype = None
    for name, t in name_tensors:
        _check(isinstance(t, torch.Tensor), f"{name} must be a tensor")
        _check(t.is_cuda, f"{name} must be a CUDA tensor (there is no CPU path)")
        _check(t.dtype in _DTYPE_CODES, f"{name}: unsupported dtype {t.dtype}")
        if dtype is None:
            dtype, device = t.dtype, t.device
        _check(t.dtype == dtype, f"{name} has dtype {t.dtype}, expected {dtype}")
        _check(t.device == device, f"{name} is on {t.device}, expected {device}")
    return dtype, device


def q_absorbed_ex(x, W_q_a, q_norm_w, W_q_b, W_uk, positions, nope_dim: int, rope_dim: int,
                  eps: float, precision: Optional[str] = None) -> List[torch.Tensor]:
    """q_absorbed with an explicit precision; see q_absorbed."""
    dtype, device = _float_operands(
        [("x", x), ("W_q_a", W_q_a), ("q_norm_w", q_norm_w), ("W_q_b", W_q_b), ("W_uk", W_uk)])
    _check(x.dim() == 3, f"x must be [B, Sq, hidden] (got {tuple(x.shape)})")
    _check(W_q_a.dim() == 2, f"W_q_a must be [hidden, q_lora] (got {tuple(W_q_a.shape)})")
    _check(W_uk.dim() == 3, f"W_uk must be [H, nope, kv_rank] (got {tuple(W_uk.shape)})")
    B, Sq, hidden = x.shape
    q_lora = W_q_a.shape[1]
    H, nope_w, R = W_uk.shape
    nope_dim, rope_dim = int(nope_dim), int(rope_dim)
    qk = nope_dim + rope_dim
    _check(W_q_a.shape[0] == hidden, "W_q_a must be [hidden, q_lora]")
    _check(W_q_b.dim() == 2 and W_q_b.shape[0] == q_lora and W_q_b.shape[1] == H * qk,
           "W_q_b must be [q_lora, H*(nope+rope)]")
    _check(q_norm_w.dim() == 1 and q_norm_w.shape[0] == q_lora,
           f"q_norm_w must be a 1-D tensor of length q_lora (got {list(q_norm_w.shape)})")
    _check(nope_w == nope_dim, f"W_uk must be [H, nope_dim={nope_dim}, kv_rank] (got {tuple(W_uk.shape)})")
    _check(isinstance(positions, torch.Tensor) and positions.dim() == 1 and positions.shape[0] == Sq,
           f"positions must be a 1-D tensor of length Sq (got "
           f"{list(positions.shape) if isinstance(positions, torch.Tensor) else type(positions)})")
    _check(not positions.is_floating_point() and not positions.is_complex(),
           "positions must be an integer tensor")
    if _C is not None:
        with torch.cuda.device(device):
            res = _C.q_absorbed_ex(x, W_q_a, q_norm_w, W_q_b, W_uk, positions, nope_dim, rope_dim, float(eps),
                                   _prec_name(precision))
        _after_call(device)
        return list(res)
    xc, Wa, g, Wb, Wk = (t.contiguous() for t in (x, W_q_a, q_norm_w, W_q_b, W_uk))
    pos = positions.to(device=device, dtype=torch.int64).contiguous()
    qa = torch.empty((B, Sq, H, R), dtype=dtype, device=device)
    qr = torch.empty((B, Sq, H, rope_dim), dtype=dtype, device=device)
    dt, pc = _DTYPE_CODES[dtype], _prec_code(precision)
    nbytes = _c_size(0)
    with torch.cuda.device(device):
        _raise_status(_lib.mla_q_absorbed_workspace_size(dt, pc, B, Sq, hidden, q_lora, H, nope_dim,
                                                         rope_dim, R, ctypes.byref(nbytes)),
                      "q_absorbed")
        ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=device)
        stream = torch.cuda.current_stream(device).cuda_stream
        st = _lib.mla_q_absorbed(dt, pc, xc.data_ptr(), Wa.data_ptr(), g.data_ptr(), Wb.data_ptr(),
                                 Wk.data_ptr(), pos.data_ptr(), B, Sq, hidden, q_lora, H, nope_dim,
                                 rope_dim, R, float(eps), qa.data_ptr(), qr.data_ptr(), ws.data_ptr(),
                                 ws.numel(), stream)
    _raise_status(st, "q_absorbed")
    _after_call(device)
    return [qa, qr]


def kv_cache_write(x, W_kv_a, kv_norm_w, positions, slots, c_kv, pe_cache, eps: float = 1e-6,
                   precision: Optional[str] = None) -> None:
    """Writes the new tokens' KV-cache rows in place: for token (b, s),
    c_kv[b, slots[s]] = RMSNorm((x @ W_kv_a)[..., :kv_rank]) * kv_norm_w and
    pe_cache[b, slots[s]] = RoPE((x @ W_kv_a)[..., kv_rank:], positions[s]).

    The reference has no write path (its caches are inputs; the step is only
    mentioned at exhaustive_benchmark_suite.py:189); this composes its rmsnorm
    and apply_rope. x [B,Sq,hidden], W_kv_a [hidden, kv_rank+rope],
    kv_norm_w [kv_rank], positions / slots [Sq] integers, c_kv [B,cap,kv_rank],
    pe_cache [B,cap,rope]; fp32 / fp16 / bf16. A slot outside [0, cap) is not
    written and is reported by device_status() (code 950)."""
    dtype, device = _float_operands([("x", x), ("W_kv_a", W_kv_a), ("kv_norm_w", kv_norm_w), ("c_kv", c_kv),
                                     ("pe_cache", pe_cache)])
    _check(x.dim() == 3 and W_kv_a.dim() == 2 and W_kv_a.shape[0] == x.shape[2], "W_kv_a must be [hidden, kv_rank+rope]")
    B, Sq, hidden = x.shape
    _check(c_kv.dim() == 3 and c_kv.shape[0] == B, "c_kv must be [B, capacity, kv_rank]")
    cap, R = c_kv.shape[1], c_kv.shape[2]
    D = W_kv_a.shape[1] - R
    _check(D >= 0 and tuple(pe_cache.shape) == (B, cap, D), "pe_cache must be [B, capacity, rope]")
    _check(kv_norm_w.dim() == 1 and kv_norm_w.shape[0] == R, "kv_norm_w must be [kv_rank]")
    _check(c_kv.is_contiguous() and pe_cache.is_contiguous(), "the caches must be contiguous (written in place)")
    for name, v in (("positions", positions), ("slots", slots)):
        _check(isinstance(v, torch.Tensor) and v.dim() == 1 and v.shape[0] == Sq and not v.is_floating_point(),
               f"{name} must be a 1-D integer tensor of length Sq")
    xc, W, g = x.contiguous(), W_kv_a.contiguous(), kv_norm_w.contiguous()
    pos = positions.to(device=device, dtype=torch.int64).contiguous()
    sl = slots.to(device=device, dtype=torch.int64).contiguous()
    dt, pc = _DTYPE_CODES[dtype], _prec_code(precision)
    nbytes = _c_size(0)
    with torch.cuda.device(device):
        _raise_status(_lib.mla_kv_cache_write_workspace_size(dt, pc, B, Sq, hidden, R, D, ctypes.byref(nbytes)),
                      "kv_cache_write")
        ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=device)
        st = _lib.mla_kv_cache_write(dt, pc, xc.data_ptr(), W.data_ptr(), g.data_ptr(), pos.data_ptr(), sl.data_ptr(),
                                     B, Sq, hidden, R, D, cap, float(eps), c_kv.data_ptr(), pe_cache.data_ptr(),
                                     ws.data_ptr(), ws.numel(), _stream_of(device))
    _raise_status(st, "kv_cache_write")
    _after_call(device)


class PackedQWeights:
    """W_q_a, W_q_b and W_uk converted once to bf16 (one device buffer), for
    q_absorbed_packed. Holds the dimensions it was packed with."""

    def __init__(self, buf: torch.Tensor, hidden: int, q_lora: int, heads: int, nope: int, rope: int,
                 kv_rank: int):
        self.buf, self.hidden, self.q_lora = buf, hidden, q_lora
        self.heads, self.nope, self.rope, self.kv_rank = heads, nope, rope, kv_rank

    @property
    def device(self):
        return self.buf.device


def pack_q_weights(W_q_a, W_q_b, W_uk, nope_dim: int, rope_dim: int) -> PackedQWeights:
    """One-time bf16 packing of the fp32 Q-prep weights (at weight-load time).
    The reference has no such step: its callers pass the fp32 weights on every
    call (exhaustive_benchmark_suite.py:261-265)."""
    dtype, device = _float_operands([("W_q_a", W_q_a), ("W_q_b", W_q_b), ("W_uk", W_uk)])
    _check(dtype == torch.float32, "pack_q_weights: fp32 weights only (16-bit weights are used as they are)")
    _check(W_q_a.dim() == 2 and W_q_b.dim() == 2 and W_uk.dim() == 3, "pack_q_weights: bad weight ranks")
    hidden, q_lora = W_q_a.shape
    H, nope_w, R = W_uk.shape
    nope_dim, rope_dim = int(nope_dim), int(rope_dim)
    _check(nope_w == nope_dim and tuple(W_q_b.shape) == (q_lora, H * (nope_dim + rope_dim)),
           "pack_q_weights: inconsistent weight shapes")
    nbytes = _c_size(0)
    _raise_status(_lib.mla_pack_q_weights_size(0, hidden, q_lora, H, nope_dim, rope_dim, R, ctypes.byref(nbytes)),
                  "pack_q_weights")
    buf = torch.empty(int(nbytes.value), dtype=torch.uint8, device=device)
    Wa, Wb, Wk = (t.contiguous() for t in (W_q_a, W_q_b, W_uk))
    with torch.cuda.device(device):
        _raise_status(_lib.mla_pack_q_weights(0, Wa.data_ptr(), Wb.data_ptr(), Wk.data_ptr(), hidden, q_lora, H,
                                              nope_dim, rope_dim, R, buf.data_ptr(), buf.numel(),
                                              _stream_of(device)), "pack_q_weights")
    return PackedQWeights(buf, hidden, q_lora, H, nope_dim, rope_dim, R)


def q_absorbed_packed(x, packed: PackedQWeights, q_norm_w, positions, eps: float) -> List[torch.Tensor]:
    """q_absorbed (tensor precision, fp32 storage) from weights packed by
    pack_q_weights: returns [q_absorbed [B,Sq,H,kv_rank], q_rope [B,Sq,H,rope]] in fp32."""
    dtype, device = _float_operands([("x", x), ("q_norm_w", q_norm_w)])
    _check(dtype == torch.float32, "q_absorbed_packed: fp32 x and q_norm_w")
    _check(isinstance(packed, PackedQWeights) and packed.device == device, "packed must be a PackedQWeights on x's device")
    _check(x.dim() == 3 and x.shape[2] == packed.hidden, f"x must be [B, Sq, {packed.hidden}]")
    _check(q_norm_w.dim() == 1 and q_norm_w.shape[0] == packed.q_lora, "q_norm_w must be [q_lora]")
    B, Sq, _ = x.shape
    _check(isinstance(positions, torch.Tensor) and positions.dim() == 1 and positions.shape[0] == Sq,
           "positions must be a 1-D tensor of length Sq")
    xc, g = x.contiguous(), q_norm_w.contiguous()
    pos = positions.to(device=device, dtype=torch.int64).contiguous()
    H, R, D = packed.heads, packed.kv_rank, packed.rope
    qa = torch.empty((B, Sq, H, R), dtype=dtype, device=device)
    qr = torch.empty((B, Sq, H, D), dtype=dtype, device=device)
    nbytes = _c_size(0)
    with torch.cuda.device(device):
        _raise_status(_lib.mla_q_absorbed_packed_workspace_size(0, B, Sq, packed.hidden, packed.q_lora, H, packed.nope,
                                                                D, R, ctypes.byref(nbytes)), "q_absorbed_packed")
        ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=device)
        st = _lib.mla_q_absorbed_packed(0, xc.data_ptr(), packed.buf.data_ptr(), g.data_ptr(), pos.data_ptr(), B, Sq,
                                        packed.hidden, packed.q_lora, H, packed.nope, D, R, float(eps),
                                        qa.data_ptr(), qr.data_ptr(), ws.data_ptr(), ws.numel(), _stream_of(device))
    _raise_status(st, "q_absorbed_packed")
    _after_call(device)
    return [qa, qr]


def q_absorbed(x, W_q_a, q_norm_w, W_q_b, W_uk, positions, nope_dim: int, rope_dim: int,
               eps: float) -> List[torch.Tensor]:
    """Kernel 2 — Q path: wq_b(RMSNorm(x @ W_q_a)) -> absorb @ W_uk, RoPE on q_rope.

    Same contract as the reference (mla_kernels.cu:599-767): returns
    [q_absorbed [B,Sq,H,kv_rank], q_rope [B,Sq,H,rope_dim]] in the input dtype.
    """
    return q_absorbed_ex(x, W_q_a, q_norm_w, W_q_b, W_uk, positions, nope_dim, rope_dim, eps)


def mla_attention_ex(q_absorbed, q_rope, c_kv, pe_cache, W_uv, scale: float, causal: bool = False,
                     precision: Optional[str] = None) -> torch.Tensor:
    """mla_attention with an explicit precision and an optional causal mask.

    causal=True lets query i of Sq attend keys 0 .. Sk-Sq+i (multi-token
    decode); False is the reference's behaviour (all keys).
    """
    dtype, device = _float_operands([("q_absorbed", q_absorbed), ("q_rope", q_rope), ("c_kv", c_kv),
                                     ("pe_cache", pe_cache), ("W_uv", W_uv)])
    _check(q_absorbed.dim() == 4, f"q_absorbed must be [B,Sq,H,kv_rank] (got {tuple(q_absorbed.shape)})")
    B, Sq, H, R = q_absorbed.shape
    _check(q_rope.dim() == 4 and tuple(q_rope.shape[:3]) == (B, Sq, H),
           f"q_rope must be [B,Sq,H,rope] (got {tuple(q_rope.shape)})")
    D = q_rope.shape[3]
    _check(c_kv.dim() == 3 and c_kv.shape[0] == B and c_kv.shape[2] == R,
           f"c_kv must be [B,Sk,kv_rank] (got {tuple(c_kv.shape)})")
    Sk = c_kv.shape[1]
    _check(tuple(pe_cache.shape) == (B, Sk, D), f"pe_cache must be [B,Sk,rope] (got {tuple(pe_cache.shape)})")
    _check(W_uv.dim() == 3 and W_uv.shape[0] == H and W_uv.shape[2] == R,
           f"W_uv must be [H,v_dim,kv_rank] (got {tuple(W_uv.shape)})")
    V = W_uv.shape[1]
    if _C is not None:
        with torch.cuda.device(device):
            out = _C.mla_attention_ex(q_absorbed, q_rope, c_kv, pe_cache, W_uv, float(scale), bool(causal),
                                      _prec_name(precision))
        _after_call(device)
        return out
    qa, qr, ck, pe, wv = (t.contiguous() for t in (q_absorbed, q_rope, c_kv, pe_cache, W_uv))
    out = torch.empty((B, Sq, H, V), dtype=dtype, device=device)
    dt, pc = _DTYPE_CODES[dtype], _prec_code(precision)
    nbytes = _c_size(0)
    with torch.cuda.device(device):
        _raise_status(_lib.mla_attention_workspace_size(dt, pc, B, Sq, Sk, H, R, D, V, int(bool(causal)),
                                                        ctypes.byref(nbytes)), "mla_attention")
        ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=device)
        stream = torch.cuda.current_stream(device).cuda_stream
        st = _lib.mla_attention(dt, pc, qa.data_ptr(), qr.data_ptr(), ck.data_ptr(), pe.data_ptr(),
                                wv.data_ptr(), B, Sq, Sk, H, R, D, V, float(scale), int(bool(causal)),
                                out.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    _raise_status(st, "mla_attention")
    _after_call(device)
    return out


class PackedUVWeights:
    """W_uv [H, v_dim, kv_rank] converted once to bf16, for mla_attention_packed."""

    def __init__(self, buf: torch.Tensor, heads: int, v_dim: int, kv_rank: int):
        self.buf, self.heads, self.v_dim, self.kv_rank = buf, heads, v_dim, kv_rank

    @property
    def device(self):
        return self.buf.device


def pack_uv_weights(W_uv) -> PackedUVWeights:
    """One-time bf16 packing of the fp32 W_uv (at weight-load time). The
    reference passes W_uv on every call and converts nothing
    (exhaustive_benchmark_suite.py:261-265)."""
    dtype, device = _float_operands([("W_uv", W_uv)])
    _check(dtype == torch.float32, "pack_uv_weights: fp32 W_uv only (16-bit weights are used as they are)")
    _check(W_uv.dim() == 3, f"W_uv must be [H,v_dim,kv_rank] (got {tuple(W_uv.shape)})")
    H, V, R = W_uv.shape
    nbytes = _c_size(0)
    _raise_status(_lib.mla_pack_uv_weights_size(0, H, V, R, ctypes.byref(nbytes)), "pack_uv_weights")
    buf = torch.empty(int(nbytes.value) // 2, dtype=torch.bfloat16, device=device)
    wv = W_uv.contiguous()
    with torch.cuda.device(device):
        _raise_status(_lib.mla_pack_uv_weights(0, wv.data_ptr(), H, V, R, buf.data_ptr(), int(nbytes.value),
                                               _stream_of(device)), "pack_uv_weights")
    return PackedUVWeights(buf, H, V, R)


def mla_attention_packed(q_absorbed, q_rope, c_kv, pe_cache, packed: PackedUVWeights, scale: float,
                         causal: bool = False) -> torch.Tensor:
    """mla_attention at tensor precision (fp32 storage) with a W_uv packed by
    pack_uv_weights: the normalised context stays in bf16 and is projected with
    the bf16 W_uv; returns fp32 [B,Sq,H,v_dim]."""
    dtype, device = _float_operands([("q_absorbed", q_absorbed), ("q_rope", q_rope), ("c_kv", c_kv),
                                     ("pe_cache", pe_cache)])
    _check(dtype == torch.float32, "mla_attention_packed: fp32 storage")
    _check(isinstance(packed, PackedUVWeights) and packed.device == device,
           "packed must be a PackedUVWeights on the operands' device")
    _check(q_absorbed.dim() == 4, f"q_absorbed must be [B,Sq,H,kv_rank] (got {tuple(q_absorbed.shape)})")
    B, Sq, H, R = q_absorbed.shape
    _check(H == packed.heads and R == packed.kv_rank, "packed W_uv does not match q_absorbed's heads / kv_rank")
    _check(q_rope.dim() == 4 and tuple(q_rope.shape[:3]) == (B, Sq, H),
           f"q_rope must be [B,Sq,H,rope] (got {tuple(q_rope.shape)})")
    D = q_rope.shape[3]
    _check(c_kv.dim() == 3 and c_kv.shape[0] == B and c_kv.shape[2] == R,
           f"c_kv must be [B,Sk,kv_rank] (got {tuple(c_kv.shape)})")
    Sk = c_kv.shape[1]
    _check(tuple(pe_cache.shape) == (B, Sk, D), f"pe_cache must be [B,Sk,rope] (got {tuple(pe_cache.shape)})")
    V = packed.v_dim
    qa, qr, ck, pe = (t.contiguous() for t in (q_absorbed, q_rope, c_kv, pe_cache))
    out = torch.empty((B, Sq, H, V), dtype=dtype, device=device)
    nbytes = _c_size(0)
    with torch.cuda.device(device):
        _raise_status(_lib.mla_attention_workspace_size(0, 1, B, Sq, Sk, H, R, D, V, int(bool(causal)),
                                                        ctypes.byref(nbytes)), "mla_attention_packed")
        ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=device)
        st = _lib.mla_attention_packed_uv(0, qa.data_ptr(), qr.data_ptr(), ck.data_ptr(), pe.data_ptr(),
                                          packed.buf.data_ptr(), B, Sq, Sk, H, R, D, V, float(scale),
                                          int(bool(causal)), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                          _stream_of(device))
    _raise_status(st, "mla_attention_packed")
    _after_call(device)
    return out


def mla_attention(q_absorbed, q_rope, c_kv, pe_cache, W_uv, scale: float) -> torch.Tensor:
    """Kernel 3 — absorbed MLA: scores -> softmax -> ctx @ c_kv -> @ W_uv.

    Same contract as the reference (mla_kernels.cu:1479-1682): scores are
    divided by ``scale`` (sqrt(192) in the reference's callers); returns a new
    [B,Sq,H,v_dim] tensor in the input dtype.
    """
    return mla_attention_ex(q_absorbed, q_rope, c_kv, pe_cache, W_uv, scale)


def mla_attention_partial(q_absorbed, q_rope, c_kv, pe_cache, W_uv, scale: float,
                          precision: Optional[str] = None):
    """Attention over a shard of the keys: returns (out [B,Sq,H,V], lse [B,Sq,H]
    fp32), lse being the natural-log sum of exp(score) over this shard's keys.
    Shards are merged exactly by lse_combine (no counterpart in the reference)."""
    dtype, device = _float_operands([("q_absorbed", q_absorbed), ("q_rope", q_rope), ("c_kv", c_kv),
                                     ("pe_cache", pe_cache), ("W_uv", W_uv)])
    _check(q_absorbed.dim() == 4, "q_absorbed must be [B,Sq,H,kv_rank]")
    B, Sq, H, R = q_absorbed.shape
    D = q_rope.shape[3]
    _check(tuple(q_rope.shape[:3]) == (B, Sq, H), "q_rope must be [B,Sq,H,rope]")
    _check(c_kv.dim() == 3 and c_kv.shape[0] == B and c_kv.shape[2] == R, "c_kv must be [B,Sk,kv_rank]")
    Sk = c_kv.shape[1]
    _check(tuple(pe_cache.shape) == (B, Sk, D), "pe_cache must be [B,Sk,rope]")
    _check(W_uv.dim() == 3 and W_uv.shape[0] == H and W_uv.shape[2] == R, "W_uv must be [H,v_dim,kv_rank]")
    V = W_uv.shape[1]
    qa, qr, ck, pe, wv = (t.contiguous() for t in (q_absorbed, q_rope, c_kv, pe_cache, W_uv))
    out = torch.empty((B, Sq, H, V), dtype=dtype, device=device)
    lse = torch.empty((B, Sq, H), dtype=torch.float32, device=device)
    dt, pc = _DTYPE_CODES[dtype], _prec_code(precision)
    nbytes = _c_size(0)
    with torch.cuda.device(device):
        _raise_status(_lib.mla_attention_workspace_size(dt, pc, B, Sq, Sk, H, R, D, V, 0, ctypes.byref(nbytes)),
                      "mla_attention_partial")
        ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=device)
        st = _lib.mla_attention_partial(dt, pc, qa.data_ptr(), qr.data_ptr(), ck.data_ptr(), pe.data_ptr(),
                                        wv.data_ptr(), B, Sq, Sk, H, R, D, V, float(scale), out.data_ptr(),
                                        lse.data_ptr(), ws.data_ptr(), ws.numel(),
                                        torch.cuda.current_stream(device).cuda_stream)
    _raise_status(st, "mla_attention_partial")
    _after_call(device)
    return out, lse


def lse_combine(outs: torch.Tensor, lses: torch.Tensor):
    """Merge key-shard partials: outs [P, ..., V], lses [P, ...] fp32 ->
    (out [..., V], lse [...]), out = sum_p exp(lse_p - L) outs_p."""
    dtype, device = _float_operands([("outs", outs)])
    _check(lses.is_cuda and lses.dtype == torch.float32, "lses must be a CUDA float32 tensor")
    _check(tuple(outs.shape[:-1]) == tuple(lses.shape), "outs must be [P, ..., V] with lses [P, ...]")
    P, V = outs.shape[0], outs.shape[-1]
    rows = lses[0].numel()
    o = outs.contiguous()
    l = lses.contiguous()
    out = torch.empty(outs.shape[1:], dtype=dtype, device=device)
    lse = torch.empty(lses.shape[1:], dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        st = _lib.mla_lse_combine(_DTYPE_CODES[dtype], P, rows, V, o.data_ptr(), l.data_ptr(), out.data_ptr(),
                                  lse.data_ptr(), torch.cuda.current_stream(device).cuda_stream)
    _raise_status(st, "lse_combine")
    return out, lse
