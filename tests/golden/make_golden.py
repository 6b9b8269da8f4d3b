"""Generates tests/golden/*.npz from the reference's own PyTorch functions.

Run where the reference project is present, with its checkout directory in the
REFERENCE_DIR environment variable:

    REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py

The reference's exhaustive_benchmark_suite.py imports its CUDA extension at
top level; a stub module is installed under that name first, and only the
device-agnostic PyTorch functions are called (prepare_q_mla_absorbed,
mla_attention_official, split_wkv_b). Inputs come from
mla_configs.make_inputs / attention_inputs with numpy's PCG64 generator, so
the tests regenerate them bit-identically on any machine; each fixture stores
a checksum of its inputs to detect a drift of that generator.

Large outputs are stored as a fixed strided subsample plus per-row sums.
"""
from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "mla-cuda_b200"))
import mla_configs as mc  # noqa: E402

SUBSAMPLE = 4096


def load_reference():
    ref_dir = os.environ.get("REFERENCE_DIR")
    if not ref_dir:
        raise SystemExit("set REFERENCE_DIR to the reference project's checkout directory")
    sys.modules.setdefault("mla_custom_cuda", types.ModuleType("mla_custom_cuda"))
    sys.path.insert(0, ref_dir)
    import exhaustive_benchmark_suite as ebs  # noqa: E402
    return ebs


def checksum(*ts) -> np.ndarray:
    return np.array([float(t.double().sum()) for t in ts] + [float(t.double().abs().sum()) for t in ts])


def sample_idx(n: int) -> np.ndarray:
    if n <= SUBSAMPLE:
        return np.arange(n, dtype=np.int64)
    step = n // SUBSAMPLE
    return (np.arange(SUBSAMPLE, dtype=np.int64) * step + 7) % n


def pack(name: str, t: torch.Tensor, d: dict) -> None:
    flat = t.detach().double().reshape(-1).numpy()
    idx = sample_idx(flat.size)
    d[f"{name}_shape"] = np.array(t.shape, dtype=np.int64)
    d[f"{name}_idx"] = idx
    d[f"{name}_val"] = flat[idx]
    d[f"{name}_rowsum"] = t.detach().double().reshape(-1, t.shape[-1]).sum(-1).numpy()


ATTN_SHAPES = [  # check_3d.py:20-23 plus the plain-path shape of check_dtypes.py:24
    (1, 1, 32), (3, 7, 40), (1, 64, 64), (1, 65, 48), (2, 33, 96), (5, 13, 71),
    (1, 1, 4096), (1, 1, 4999), (2, 3, 1000), (1, 1, 16384), (1, 2, 8191), (1, 1, 64),
]


def main() -> None:
    torch.set_num_threads(os.cpu_count() or 4)
    ebs = load_reference()
    cfg = ebs.DEEPSEEK_V3

    # 1. attention sweeps: raw N(0,1) operands, reference fp64 and fp32 outputs
    for (B, Sq, Sk) in ATTN_SHAPES:
        seed = 1000 + B * 131 + Sq * 17 + Sk
        qa, qr, ck, pe, wuv = mc.attention_inputs(B, Sq, Sk, seed=seed)
        d = {"seed": np.array(seed), "B": np.array(B), "Sq": np.array(Sq), "Sk": np.array(Sk),
             "in_checksum": checksum(qa, qr, ck, pe, wuv)}
        out64 = ebs.mla_attention_official(qa.double(), qr.double(), ck.double(), pe.double(), wuv.double(), cfg)
        out32 = ebs.mla_attention_official(qa, qr, ck, pe, wuv, cfg)
        pack("out64", out64, d)
        pack("out32", out32, d)
        np.savez_compressed(HERE / f"attn_{B}x{Sq}x{Sk}.npz", **d)
        print("attn", B, Sq, Sk, float(out64.abs().max()))

    # 2. causal multi-token decode, pinned through the unmodified reference:
    #    query i of Sq over keys 0 .. Sk-Sq+i equals attention on that key prefix.
    for (B, Sq, Sk) in [(2, 4, 37), (1, 8, 300)]:
        seed = 5000 + B * 131 + Sq * 17 + Sk
        qa, qr, ck, pe, wuv = mc.attention_inputs(B, Sq, Sk, seed=seed)
        rows = []
        for i in range(Sq):
            n = Sk - Sq + i + 1
            rows.append(ebs.mla_attention_official(qa[:, i:i + 1].double(), qr[:, i:i + 1].double(),
                                                   ck[:, :n].double(), pe[:, :n].double(), wuv.double(), cfg))
        out = torch.cat(rows, dim=1)
        d = {"seed": np.array(seed), "B": np.array(B), "Sq": np.array(Sq), "Sk": np.array(Sk),
             "in_checksum": checksum(qa, qr, ck, pe, wuv), "out64_full": out.numpy().astype(np.float32)}
        np.savez_compressed(HERE / f"causal_{B}x{Sq}x{Sk}.npz", **d)
        print("causal", B, Sq, Sk)

    # 3. full layer forward at config 0 (DeepSeek-V3 dims, BASELINE distributions)
    w = mc.CONFIGS["c0"]
    t = mc.make_inputs(w, seed=0)
    Wq = ebs.QProjection(t["W_q_a"], t["q_norm_w"], t["W_q_b"])
    d = {"seed": np.array(0), "in_checksum": checksum(*(t[k] for k in
         ("x", "W_q_a", "W_q_b", "W_uk", "W_uv", "c_kv", "pe_cache")))}
    for acc_name, cast in (("64", torch.float64), ("32", torch.float32)):
        tt = {k: (v.to(cast) if v.is_floating_point() else v) for k, v in t.items()}
        Wq_ = ebs.QProjection(tt["W_q_a"], tt["q_norm_w"], tt["W_q_b"])
        qa, qr = ebs.prepare_q_mla_absorbed(tt["x"], Wq_, tt["W_uk"], tt["positions"], cfg)
        out = ebs.mla_attention_official(qa, qr, tt["c_kv"], tt["pe_cache"], tt["W_uv"], cfg)
        # stored as float32: 6e-8 relative, far below every tolerance used
        d[f"qa{acc_name}_full"] = qa.float().numpy()
        d[f"qr{acc_name}_full"] = qr.float().numpy()
        d[f"out{acc_name}_full"] = out.float().numpy()
    del Wq
    np.savez_compressed(HERE / "forward_c0.npz", **d)
    print("forward c0", float(np.abs(d["out64_full"]).max()))

    # 4. Q-prep with small, non-DeepSeek dimensions (shape generality), fp64 reference
    small = mc.Workload("small", 3, 2, 19, hidden=96, heads=4, q_lora=48, kv_rank=32, nope=16, rope=8, v_dim=24)
    t = mc.make_inputs(small, seed=3)
    scfg = ebs.DeepSeekV3Config(hidden_dim=96, n_heads=4, kv_lora_rank=32, q_lora_rank=48,
                                qk_nope_head_dim=16, qk_rope_head_dim=8, v_head_dim=24)
    tt = {k: (v.double() if v.is_floating_point() else v) for k, v in t.items()}
    qa, qr = ebs.prepare_q_mla_absorbed(tt["x"], ebs.QProjection(tt["W_q_a"], tt["q_norm_w"], tt["W_q_b"]),
                                        tt["W_uk"], tt["positions"], scfg)
    out = ebs.mla_attention_official(qa, qr, tt["c_kv"], tt["pe_cache"], tt["W_uv"], scfg)
    np.savez_compressed(HERE / "forward_small.npz", seed=np.array(3),
                        in_checksum=checksum(*(t[k] for k in ("x", "W_q_a", "W_q_b", "W_uk", "W_uv", "c_kv",
                                                              "pe_cache"))),
                        qa64_full=qa.numpy(), qr64_full=qr.numpy(), out64_full=out.numpy())
    print("forward small")


if __name__ == "__main__":
    main()
