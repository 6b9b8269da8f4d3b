"""Workload configurations and seeded synthetic inputs for the MLA decode path.

The five configurations are the ones the benchmark and parity tests run
(B, Sq, Sk, storage dtype, causal). Model dimensions are DeepSeek-V3's
(exhaustive_benchmark_suite.py:30-52): hidden 7168, 128 heads, q_lora 1536,
kv_lora 512, nope 128, rope 64, v 128.

Distributions: x ~ N(0,1); W_q_a, W_q_b, W_uk, W_uv ~ N(0, 0.02); RMSNorm gain
1; eps 1e-6; c_kv, pe_cache ~ N(0,1); RoPE theta 10000; scores divided by
sqrt(192). Draw order: x, W_q_a, W_q_b, W_uk, W_uv, c_kv, pe_cache. The query
positions are Sk-Sq+1 .. Sk, so a single decode query sits at position Sk.

Two generators:
  * ``gen="numpy"``: numpy PCG64 (np.random.default_rng(seed)), float64 draws
    rounded to float32. Portable across machines; used by parity tests and the
    golden fixtures.
  * ``gen="device"``: torch's generator on the target device. Fast; used by
    the benchmark, where only the distribution matters.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, Optional

import numpy as np
import torch

HIDDEN, HEADS, Q_LORA, KV_RANK, NOPE, ROPE, V_DIM = 7168, 128, 1536, 512, 128, 64, 128
QK_HEAD = NOPE + ROPE
SCALE = float(QK_HEAD) ** 0.5
EPS = 1e-6
W_STD = 0.02


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    sq: int
    sk: int
    dtype: torch.dtype = torch.float32
    causal: bool = False
    hidden: int = HIDDEN
    heads: int = HEADS
    q_lora: int = Q_LORA
    kv_rank: int = KV_RANK
    nope: int = NOPE
    rope: int = ROPE
    v_dim: int = V_DIM

    @property
    def scale(self) -> float:
        return float(self.nope + self.rope) ** 0.5

    def describe(self) -> Dict[str, object]:
        return {"workload": self.name, "batch": self.batch, "sq": self.sq, "sk": self.sk,
                "storage": str(self.dtype).replace("torch.", ""), "causal": self.causal}


CONFIGS = {
    "c0": Workload("c0_tiny_decode", 1, 1, 256),
    "c1": Workload("c1_decode_b128_sk4989", 128, 1, 4989),
    "c2": Workload("c2_long_ctx_b4_sk65536", 4, 1, 65536),
    "c3": Workload("c3_mtp_b16_sq8_sk4096_causal", 16, 8, 4096, causal=True),
    "c4": Workload("c4_box_b1024_sk4989_bf16", 1024, 1, 4989, dtype=torch.bfloat16),
}


# The reference's PRODUCTION_SCENARIOS (exhaustive_benchmark_suite.py:78-173):
# decode and speculative-decode shapes taken from public serving reports, and
# prefill chunks. The reference runs every one without a mask (each query
# attends all Sk keys), so these do too.
SCENARIOS = {
    "decode_single_user_long_ctx": Workload("decode_single_user_long_ctx", 1, 1, 65536),
    "decode_serving_avg_ctx": Workload("decode_serving_avg_ctx", 128, 1, 4989),
    "decode_serving_long_ctx": Workload("decode_serving_long_ctx", 128, 1, 8192),
    "decode_serving_high_batch": Workload("decode_serving_high_batch", 256, 1, 2048),
    "decode_speculative_2tok": Workload("decode_speculative_2tok", 64, 2, 512),
    "decode_speculative_4tok": Workload("decode_speculative_4tok", 64, 4, 768),
    "decode_speculative_long_ctx": Workload("decode_speculative_long_ctx", 132, 4, 4096),
    "prefill_chat_batch": Workload("prefill_chat_batch", 8, 512, 512),
    "prefill_chunk_2k": Workload("prefill_chunk_2k", 1, 2048, 2048),
    "prefill_chunk_4k": Workload("prefill_chunk_4k", 1, 4096, 4096),
}


def positions_for(sq: int, sk: int) -> torch.Tensor:
    return torch.arange(sk - sq + 1, sk + 1, dtype=torch.int64)


def make_inputs(w: Workload, device="cpu", seed: int = 0, gen: str = "numpy",
                batch: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Seeded inputs of workload ``w`` (optionally with a different batch).

    Returns x, W_q_a, q_norm_w, W_q_b, W_uk, W_uv, c_kv, pe_cache (storage
    dtype ``w.dtype``) and positions (int64).
    """
    B = w.batch if batch is None else batch
    shapes = [
        ("x", (B, w.sq, w.hidden), 1.0),
        ("W_q_a", (w.hidden, w.q_lora), W_STD),
        ("W_q_b", (w.q_lora, w.heads * (w.nope + w.rope)), W_STD),
        ("W_uk", (w.heads, w.nope, w.kv_rank), W_STD),
        ("W_uv", (w.heads, w.v_dim, w.kv_rank), W_STD),
        ("c_kv", (B, w.sk, w.kv_rank), 1.0),
        ("pe_cache", (B, w.sk, w.rope), 1.0),
    ]
    out: Dict[str, torch.Tensor] = {}
    if gen == "numpy":
        rng = np.random.default_rng(seed)
        for name, shape, std in shapes:
            a = rng.standard_normal(shape, dtype=np.float32)
            if std != 1.0:
                a *= np.float32(std)
            out[name] = torch.from_numpy(a).to(device=device, dtype=w.dtype)
    elif gen == "device":
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        for name, shape, std in shapes:
            t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
            if std != 1.0:
                t.mul_(std)
            out[name] = t.to(w.dtype)
    else:
        raise ValueError(f"unknown generator {gen!r}")
    out["q_norm_w"] = torch.ones(w.q_lora, dtype=w.dtype, device=device)
    out["positions"] = positions_for(w.sq, w.sk).to(device)
    return out


def attention_inputs(B: int, Sq: int, Sk: int, seed: int = 0, dtype=torch.float32, device="cpu",
                     heads: int = HEADS, kv_rank: int = KV_RANK, rope: int = ROPE, v_dim: int = V_DIM):
    """Raw N(0,1) attention operands (q_absorbed, q_rope, c_kv, pe_cache, W_uv),
    the distribution of the reference's shape / dtype sweeps (check_3d.py:27-32)."""
    rng = np.random.default_rng(seed)
    shapes = [(B, Sq, heads, kv_rank), (B, Sq, heads, rope), (B, Sk, kv_rank), (B, Sk, rope),
              (heads, v_dim, kv_rank)]
    return tuple(torch.from_numpy(rng.standard_normal(s, dtype=np.float32)).to(device=device, dtype=dtype)
                 for s in shapes)
