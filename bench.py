"""MLA decode layer-forward benchmark (one B200 per rank).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1]
                    [--precision exact|tensor] [--impl ours|reference]

A step is one absorbed-MLA decode layer forward — Q-prep (q_absorbed) plus
attention (mla_attention) — over one batch of the workload, through the
drop-in module ``mla_custom_cuda`` (which calls the C ABI). Default workload:
config c1 (B=128, Sq=1, Sk=4989, fp32 storage, DeepSeek-V3 dims), the
configuration BASELINE.json's metric is quoted on.

Multi-GPU (torchrun, one rank per GPU): batch-sharded weak scaling, each rank
owns its own B sequences and their caches; there is no data-path collective.
Time is the max over ranks (an all-reduce of the device-measured time).

``--impl reference`` times the reference's own PyTorch path for this layer
(restated in oracle/mla_oracle.py) on the host CPU cores with all threads, on
the same workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "mla-cuda_b200"))

import torch  # noqa: E402

import mla_configs as mc  # noqa: E402

METRIC = "MLA decode layer-forward tokens/s at B=128,Sk=4989 (us/layer and cache-read HBM GB/s reported)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1500)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c1", choices=sorted(mc.CONFIGS) + sorted(mc.SCENARIOS))
    ap.add_argument("--reference-gpu", action="store_true",
                    help="also time the reference's own CUDA kernels (mla_kernels.cu built for sm_100a by "
                         "oracle/build_ref.py into oracle/_ref/) on BASELINE configs c0-c3 (extra field)")
    ap.add_argument("--scenarios", action="store_true",
                    help="also time every PRODUCTION_SCENARIOS shape of the reference (extra 'scenarios' field)")
    ap.add_argument("--precision", default="tensor", choices=["exact", "tensor"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--min-warmup-s", type=float, default=1.5,
                    help="minimum warm-up wall time (lets the clock sampler start); 0 under a profiler")
    ap.add_argument("--no-stages", action="store_true", help="skip the per-stage / per-precision timings")
    ap.add_argument("--shard", default=None, choices=["batch", "keys"],
                    help="multi-GPU layout: batch (weak scaling, default) or keys (strong scaling, default for c2)")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch the timed layer forwards one by one instead of replaying a CUDA graph of one")
    ap.add_argument("--no-parity", action="store_true", help="skip the sampled-sequence parity check")
    ap.add_argument("--weights", default="packed", choices=["packed", "plain"],
                    help="tensor precision, fp32 storage: W_q_a / W_q_b / W_uk / W_uv packed once to bf16 "
                         "(default) or the fp32 weights on every call")
    ap.add_argument("--no-key-shard-c2", action="store_true",
                    help="with --gpus N > 1, skip the extra key-sharded c2 measurement")
    ap.add_argument("--qprep", default="redundant", choices=["heads", "redundant"],
                    help="key sharding: Q-prep repeated on every rank (default), or sharded by heads + all-gather of q")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def line_config(w: mc.Workload, world: int, shard: str) -> dict:
    """The workload keys both arms (ours and the reference) print identically."""
    return {**w.describe(), "global_batch": w.batch * (world if shard == "batch" else 1),
            "parallelism": f"batch-shard dp{world}" if shard == "batch" else f"key-shard sp{world}",
            "l2": "no flush: inputs larger than L2 (c_kv + pe_cache %.2f GB per GPU)"
                  % (workload_bytes(w, w.batch)[0] / world ** (shard == "keys") / 1e9)}


def workload_bytes(w: mc.Workload, B: int, sk=None):
    es = torch.tensor([], dtype=w.dtype).element_size()
    cache = B * (w.sk if sk is None else sk) * (w.kv_rank + w.rope) * es
    weights = (w.hidden * w.q_lora + w.q_lora + w.q_lora * w.heads * (w.nope + w.rope)
               + 2 * w.heads * w.kv_rank * w.nope) * es
    acts = B * w.sq * (w.hidden + w.heads * w.v_dim) * es
    return cache, weights, acts


def workload_flops(w: mc.Workload, B: int):
    M = B * w.sq
    q = 2 * M * (w.hidden * w.q_lora + w.q_lora * w.heads * (w.nope + w.rope) + w.heads * w.nope * w.kv_rank)
    attn = 2 * M * w.heads * w.sk * (w.kv_rank + w.rope + w.kv_rank)
    out = 2 * M * w.heads * w.kv_rank * w.v_dim
    return q, attn + out


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


KEY_SHARDED = {"on": False, "heads": False}
PACKED = {"w": None, "uv": None}   # PackedQWeights / PackedUVWeights when the step uses pre-packed weights

# DRAM bytes per launch of the decode kernel, from the ncu capture named below
# (dram__bytes_read.sum + dram__bytes_write.sum), keyed by (config, precision,
# shard, world).
TRAFFIC = {("c1", "tensor", "batch", 1): 1.565e9}
TRAFFIC_SOURCE = ("profiles/mla_decode_tc_kernel_c1.md: ncu capture of mla_decode_tc_kernel at c1, "
                  "dram__bytes_read.sum + dram__bytes_write.sum of one launch")


def run_forward(mcc, t, w, precision):
    if KEY_SHARDED["heads"]:
        # each rank holds its heads' slices of W_q_b / W_uk: local Q-prep, all-gather of q
        from mla_custom_cuda import sharding
        qa, qr = sharding.head_sharded_q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"],
                                                  t["positions"], w.nope, w.rope, mc.EPS, precision=precision)
    elif PACKED["w"] is not None and precision == "tensor":
        qa, qr = mcc.q_absorbed_packed(t["x"], PACKED["w"], t["q_norm_w"], t["positions"], mc.EPS)
    else:
        qa, qr = mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                                   w.nope, w.rope, mc.EPS, precision=precision)
    if KEY_SHARDED["on"]:
        # every rank holds all sequences' queries and its own key slice; partial
        # attention, NCCL all-gather of (out, lse), exact log-sum-exp merge
        from mla_custom_cuda import sharding
        return sharding.sk_sharded_attention(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale,
                                             precision=precision), qa, qr
    if PACKED["uv"] is not None and precision == "tensor":
        return mcc.mla_attention_packed(qa, qr, t["c_kv"], t["pe_cache"], PACKED["uv"], w.scale,
                                        causal=w.causal), qa, qr
    return mcc.mla_attention_ex(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale, causal=w.causal,
                                precision=precision), qa, qr


def cpu_reference_forward(t, w):
    from oracle import mla_oracle as orc
    return orc.forward(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["W_uv"], t["c_kv"],
                       t["pe_cache"], t["positions"], causal=w.causal, scale=w.scale)


def cpu_baseline(w: mc.Workload, reps: int = 3):
    """The reference's PyTorch path on the host cores, all threads, best of `reps`."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    t = mc.make_inputs(w, device="cpu", gen="device", seed=0)
    if w.dtype != torch.float32:
        t = {k: (v.float() if v.is_floating_point() else v) for k, v in t.items()}
    with torch.inference_mode():
        cpu_reference_forward(t, w)
        best = float("inf")
        for _ in range(reps):
            t0 = time.perf_counter()
            cpu_reference_forward(t, w)
            best = min(best, time.perf_counter() - t0)
    tokens = w.batch * w.sq
    return {"value": tokens / best, "unit": "tokens/s", "cores": threads, "kind": "port",
            "cpu_model": cpu_model(), "ms_per_step": best * 1e3,
            "sample": f"full {w.name} forward ({w.batch} sequences), fp32, oracle/mla_oracle.py "
                      f"(the reference's torch ops), best of {reps}"}


def main_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    w = mc.CONFIGS.get(args.config) or mc.SCENARIOS[args.config]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    t = mc.make_inputs(w, device="cpu", gen="device", seed=0)
    if w.dtype != torch.float32:
        t = {k: (v.float() if v.is_floating_point() else v) for k, v in t.items()}
    with torch.inference_mode():
        for _ in range(args.warmup):
            cpu_reference_forward(t, w)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            cpu_reference_forward(t, w)
        el = time.perf_counter() - t0
    tokens = w.batch * w.sq
    v = tokens * args.steps / el
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) cache / activations, N(0,0.02) weights)",
            "config": line_config(w, 1, "batch"),
            "note": "reference PyTorch path (restated in oracle/mla_oracle.py) on host CPU cores",
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "cpu_model": cpu_model(),
                             "sample": f"full {w.name} forward per step, oracle/mla_oracle.py (the reference's "
                                       f"torch ops), {threads} threads"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def device_timed(stream, fn, n, warm=3):
    """Average device time (ms) of fn() over n calls, CUDA events on `stream`."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


def max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    tt = torch.tensor([v], device=dev)
    torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
    return float(tt.item())


def parity_sample(mcc, t, w, precision, seqs):
    """rel-L2 of the GPU layer output against the fp64 oracle, and the
    argmax-of-scores agreement, on a few sequences of the benched inputs."""
    from oracle import mla_oracle as orc
    out, qa, qr = run_forward(mcc, t, w, precision)   # the benched path
    torch.cuda.synchronize()
    W = {k: t[k].double().cpu() for k in ("W_q_a", "q_norm_w", "W_q_b", "W_uk", "W_uv")}
    errs, errs32, noise, agree = [], [], [], []
    for b in seqs:
        x = t["x"][b:b + 1].double().cpu()
        ck, pe = t["c_kv"][b:b + 1].cpu(), t["pe_cache"][b:b + 1].cpu()
        rqa, rqr = orc.q_absorbed(x, W["W_q_a"], W["q_norm_w"], W["W_q_b"], W["W_uk"], t["positions"].cpu())
        ref = orc.mla_attention(rqa, rqr, ck.double(), pe.double(), W["W_uv"], w.scale, w.causal)
        o = out[b:b + 1].double().cpu()
        errs.append(float((o - ref).norm() / ref.norm()))
        exact32 = precision == "exact" and w.dtype == torch.float32
        if exact32:   # the reference's own path runs in fp32
            W32 = {k: v.float() for k, v in W.items()}
            r32a, r32r = orc.q_absorbed(x.float(), W32["W_q_a"], W32["q_norm_w"], W32["W_q_b"], W32["W_uk"],
                                        t["positions"].cpu())
            ref32 = orc.mla_attention(r32a, r32r, ck.float(), pe.float(), W32["W_uv"], w.scale, w.causal)
            errs32.append(float((o - ref32.double()).norm() / ref32.double().norm()))
            noise.append(float((ref32.double() - ref).norm() / ref.norm()))
        gq, gr = qa[b:b + 1].cpu(), qr[b:b + 1].cpu()
        gk, gp = ck, pe
        if precision == "tensor":   # the operands the tensor-core kernel multiplies
            gq, gr, gk, gp = (v.to(torch.bfloat16) for v in (gq, gr, gk, gp))
        s = orc.scores(gq.double(), gr.double(), gk.double(), gp.double(), w.scale, w.causal)
        r = orc.scores(rqa, rqr, ck.double(), pe.double(), w.scale, w.causal)
        agree.append(float((s.argmax(-1) == r.argmax(-1)).double().mean()))
    res = {"sequences": list(seqs), "rel_l2_vs_fp64_oracle": errs, "max_rel_l2": max(errs),
           "argmax_agreement": agree, "min_argmax_agreement": min(agree)}
    if precision == "exact" and w.dtype == torch.float32:
        res.update({"rel_l2_vs_fp32_reference_path": errs32, "fp32_reference_vs_fp64": noise,
                    "tolerance": "1e-5 vs the fp32 reference path; < 5x its own error vs fp64"})
    elif w.dtype in (torch.bfloat16, torch.float16):
        res["tolerance"] = ("2e-2" if w.dtype == torch.bfloat16 else "3e-2") + \
            " vs fp64 (16-bit storage: outputs and intermediates in the storage dtype, as the reference's)"
    else:
        res["tolerance"] = "2e-2 vs fp64"
    return res


def time_scenarios(mcc, dev, stream):
    """Layer forward (q_absorbed + mla_attention, eager, CUDA events) of every
    PRODUCTION_SCENARIOS shape of the reference in both precisions."""
    res = {}
    for name, w in mc.SCENARIOS.items():
        t = mc.make_inputs(w, device=dev, gen="device", seed=7)
        row = {"batch": w.batch, "sq": w.sq, "sk": w.sk}
        for prec in ("tensor", "exact"):
            def step():
                qa, qr = mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"],
                                           t["positions"], w.nope, w.rope, mc.EPS, precision=prec)
                return mcc.mla_attention_ex(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale, precision=prec)
            ms = device_timed(stream, step, 5)
            row[prec] = {"layer_ms": ms, "tokens_per_s": w.batch * w.sq / (ms * 1e-3)}
        res[name] = row
        del t
        torch.cuda.empty_cache()
    return res


def time_reference_gpu(mcc, dev, stream):
    """The reference's two CUDA entry points (mla_kernels.cu, unmodified, built for
    sm_100a) on BASELINE configs c0-c3, fp32, beside this library's exact path on
    the same inputs; CUDA events, 10 calls after 3 warm-ups. The reference has no
    mask, so c3 runs unmasked on both sides here."""
    import importlib.machinery
    import importlib.util
    so = ROOT / "oracle" / "_ref" / "mla_ref_cuda.so"
    if not so.exists():
        return {"unavailable": "oracle/_ref/mla_ref_cuda.so not built (python oracle/build_ref.py)"}
    loader = importlib.machinery.ExtensionFileLoader("mla_ref_cuda", str(so))
    spec = importlib.util.spec_from_file_location("mla_ref_cuda", str(so), loader=loader)
    ref = importlib.util.module_from_spec(spec)
    loader.exec_module(ref)
    res = {}
    for cfg in ("c0", "c1", "c2", "c3"):
        w = mc.CONFIGS[cfg]
        t = mc.make_inputs(w, device=dev, gen="device", seed=11)

        def ref_step():
            qa, qr = ref.q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                                    w.nope, w.rope, mc.EPS)
            return ref.mla_attention(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale)

        def our_step(prec):
            qa, qr = mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                                       w.nope, w.rope, mc.EPS, precision=prec)
            return mcc.mla_attention_ex(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale, precision=prec)

        r_ms = device_timed(stream, ref_step, 10)
        e_ms = device_timed(stream, lambda: our_step("exact"), 10)
        t_ms = device_timed(stream, lambda: our_step("tensor"), 10)
        a, b = ref_step(), our_step("exact")
        torch.cuda.synchronize()
        res[cfg] = {"reference_cuda_ms": r_ms, "ours_exact_ms": e_ms, "ours_tensor_ms": t_ms,
                    "exact_speedup": r_ms / e_ms, "tensor_speedup": r_ms / t_ms,
                    "rel_l2_exact_vs_reference_cuda": float((a.double() - b.double()).norm() / a.double().norm())}
        del t
        torch.cuda.empty_cache()
    return res


def key_shard_c2(mcc, dev, rank, world, steps, precision):
    """Config c2 (B=4, Sk=65536) key-sharded over all ranks inside this run:
    every rank holds 1/world of every sequence's keys, the partials are
    all-gathered over NCCL and merged (strong scaling of one decode step)."""
    from mla_custom_cuda import sharding
    w = mc.CONFIGS["c2"]
    k0, k1 = sharding.key_shard(w.sk, rank, world)
    t = mc.make_inputs(w, device=dev, gen="device", seed=1234)
    t["c_kv"] = t["c_kv"][:, k0:k1].contiguous()
    t["pe_cache"] = t["pe_cache"][:, k0:k1].contiguous()
    stream = torch.cuda.current_stream(dev)
    # tensor precision, fp32 storage: Q-prep from weights packed once to bf16, as
    # in the batch-sharded step (every rank prepares the queries of all sequences)
    packed = (mcc.pack_q_weights(t["W_q_a"], t["W_q_b"], t["W_uk"], w.nope, w.rope)
              if precision == "tensor" and w.dtype == torch.float32 else None)

    def q():
        if packed is not None:
            return mcc.q_absorbed_packed(t["x"], packed, t["q_norm_w"], t["positions"], mc.EPS)
        return mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                                 w.nope, w.rope, mc.EPS, precision=precision)

    def step():
        qa, qr = q()
        return sharding.sk_sharded_attention(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale,
                                             precision=precision)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    torch.distributed.barrier()
    ms = max_over_ranks(device_timed(stream, step, steps, warm=0), world, dev)
    q_ms = max_over_ranks(device_timed(stream, q, steps), world, dev)
    qa, qr = q()
    att_ms = max_over_ranks(device_timed(stream, lambda: mcc.mla_attention_partial(
        qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale, precision=precision), steps), world, dev)
    return {"workload": w.name, "ranks": world, "tokens_per_s": w.batch * w.sq / (ms * 1e-3), "ms_per_step": ms,
            "q_absorbed_ms_per_rank": q_ms, "partial_attention_ms_per_rank": att_ms,
            "all_gather_and_merge_ms": max(ms - q_ms - att_ms, 0.0), "keys_per_rank": k1 - k0,
            "q_prep": "packed bf16 weights" if packed is not None else "storage-dtype weights",
            "timing": "CUDA events on each rank, max over ranks"}


def main_ours(args):
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("NCCL_DEBUG", "WARN")   # keep NCCL's banner off stdout (one JSON line)
        dist.init_process_group("nccl", device_id=dev)
    import mla_custom_cuda as mcc

    w = mc.CONFIGS.get(args.config) or mc.SCENARIOS[args.config]
    precision = args.precision
    B = w.batch
    shard = args.shard or ("keys" if args.config == "c2" else "batch")
    if world == 1:
        shard = "batch"
    sk_local = w.sk
    if shard == "keys":
        if w.causal:
            raise SystemExit("key sharding is for non-causal decode")
        from mla_custom_cuda import sharding
        k0, k1 = sharding.key_shard(w.sk, rank, world)
        sk_local = k1 - k0
        t = mc.make_inputs(w, device=dev, gen="device", seed=1234)   # same queries / weights on every rank
        t["c_kv"] = t["c_kv"][:, k0:k1].contiguous()
        t["pe_cache"] = t["pe_cache"][:, k0:k1].contiguous()
        KEY_SHARDED["on"] = True
        if args.qprep == "heads" and w.heads % world == 0:
            t["W_q_b"], t["W_uk"] = sharding.shard_q_weights(t["W_q_b"], t["W_uk"], w.nope, w.rope, rank, world)
            KEY_SHARDED["heads"] = True
    else:
        t = mc.make_inputs(w, device=dev, gen="device", seed=1234 + rank)
    stream = torch.cuda.current_stream(dev)
    if (args.weights == "packed" and precision == "tensor" and w.dtype == torch.float32
            and not KEY_SHARDED["heads"]):
        # weight-load time, outside every timed region: one bf16 copy of W_q_a, W_q_b, W_uk
        PACKED["w"] = mcc.pack_q_weights(t["W_q_a"], t["W_q_b"], t["W_uk"], w.nope, w.rope)
        PACKED["uv"] = mcc.pack_uv_weights(t["W_uv"])
        torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    # ---- device-resident timed region (whole layer forward, headline precision).
    # The clock sampler starts before the warm-up, which runs for at least W steps
    # and at least --min-warmup-s seconds so nvidia-smi samples a loaded GPU.
    # Batch-sharded steps hold no collective: one layer forward (q_absorbed_ex +
    # mla_attention_ex, 8 kernels) is captured once in a CUDA graph and replayed
    # per step, which removes the host launch gaps; the kernels and their work are
    # the same as an eager call's.
    use_graph = not args.no_graph and not KEY_SHARDED["on"]
    if use_graph:
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                run_forward(mcc, t, w, precision)
        stream.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run_forward(mcc, t, w, precision)
        torch.cuda.synchronize()

        def step():
            graph.replay()
    else:
        def step():
            run_forward(mcc, t, w, precision)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t_w = time.perf_counter()
        n_w = 0
        while True:
            step()
            n_w += 1
            if n_w % 8 == 0:
                torch.cuda.synchronize()
            done = n_w >= max(args.warmup, 3) and time.perf_counter() - t_w >= args.min_warmup_s
            if world > 1:
                # every rank runs the same number of warm-up steps (a key-sharded step
                # holds collectives)
                flag = torch.tensor([0 if done else 1], device=dev, dtype=torch.int32)
                torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MAX)
                done = int(flag.item()) == 0
            if done:
                break
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world, dev)
    tokens_total = B * w.sq * (world if shard == "batch" else 1)
    value = tokens_total / (ms * 1e-3)
    dev_status = mcc.device_status(dev)   # a kernel that gave up on a bounded wait invalidates the run
    if dev_status:
        raise SystemExit(f"device-side failure code {dev_status} during the timed region")

    # ---- per-stage timing (same stream, CUDA events; inputs larger than L2), and
    # the decode-attention kernel alone (event pair around each of its launches)
    n_att = max(5, min(args.steps, 200))
    stages = {}
    kernel_ms = None
    for prec in ((precision,) if args.no_stages else ("tensor", "exact")):
        if KEY_SHARDED["heads"]:
            # local stages of a rank: Q-prep of its heads, attention over its key shard
            from mla_custom_cuda import sharding
            qa, qr = sharding.head_sharded_q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"],
                                                      t["positions"], w.nope, w.rope, mc.EPS, precision=prec)
        else:
            qa, qr = mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                                       w.nope, w.rope, mc.EPS, precision=prec)
        if KEY_SHARDED["on"]:
            att_fn = lambda: mcc.mla_attention_partial(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale,  # noqa
                                                       precision=prec)
        elif prec == "tensor" and PACKED["uv"] is not None:
            att_fn = lambda: mcc.mla_attention_packed(qa, qr, t["c_kv"], t["pe_cache"], PACKED["uv"], w.scale,  # noqa
                                                      causal=w.causal)
        else:
            att_fn = lambda: mcc.mla_attention_ex(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale,  # noqa
                                                  causal=w.causal, precision=prec)
        if prec == "tensor":
            mcc.kernel_timing(True)
        att = device_timed(stream, att_fn, n_att)
        if prec == "tensor":
            tot, cnt = mcc.kernel_timing()
            mcc.kernel_timing(False)
            kernel_ms = max_over_ranks(tot / max(cnt, 1), world, dev) if cnt else None
        att = max_over_ranks(att, world, dev)
        qp = max_over_ranks(device_timed(stream, lambda: mcc.q_absorbed_ex(
            t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"], w.nope, w.rope, mc.EPS,
            precision=prec), n_att), world, dev)
        fwd = att + qp if prec != precision else ms
        stages[prec] = {"q_absorbed_ms": qp, "mla_attention_ms": att, "layer_ms": fwd,
                        "tokens_per_s": tokens_total / (fwd * 1e-3)}
        if prec == "tensor" and PACKED["w"] is not None:
            stages[prec]["q_absorbed_packed_ms"] = max_over_ranks(device_timed(stream, lambda: mcc.q_absorbed_packed(
                t["x"], PACKED["w"], t["q_norm_w"], t["positions"], mc.EPS), n_att), world, dev)
        if prec == "tensor" and kernel_ms:
            stages[prec]["decode_kernel_ms"] = kernel_ms
    att_ms = stages[precision]["mla_attention_ms"]
    q_ms = stages[precision].get("q_absorbed_packed_ms", stages[precision]["q_absorbed_ms"])

    cache_b, weight_b, act_b = workload_bytes(w, B, sk_local)
    qf, af = workload_flops(w, B)
    hbm, bf16_tf, peak_src = peaks()
    # the dominant kernel (decode attention) when it ran, else the attention stage
    dom_ms = kernel_ms if (precision == "tensor" and kernel_ms) else att_ms
    dom_gbs = cache_b / (dom_ms * 1e-3) / 1e9

    # ---- end to end through the public API: the step's hidden states come from
    # pinned host memory and the layer output goes back to pinned host memory;
    # the KV cache and weights stay resident in HBM, as in a decode server.
    # Pipelined (the headline): a decode server overlaps a step's transfers with
    # its neighbours' compute, so each step's inputs go host->device on one copy
    # stream and its output device->host on another, double-buffered, while the
    # layer runs on the compute stream; the timed region ends when the last
    # output is on the host. The layer of each buffer slot is the public-API call
    # sequence captured once in a CUDA graph (as the device-timed value is), so the
    # host launch path stays off the step. Serial: copy in, compute (eager calls),
    # copy out, one step at a time.
    def e2e_run(prec):
        x_host = t["x"].cpu().pin_memory()
        pos_host = t["positions"].cpu().pin_memory()
        outs_host = [torch.empty((B, w.sq, w.heads, w.v_dim), dtype=w.dtype).pin_memory() for _ in range(2)]
        xs_dev = [torch.empty_like(t["x"]) for _ in range(2)]
        pos_dev = [torch.empty_like(t["positions"]) for _ in range(2)]
        t2 = dict(t)
        h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]
        out_ready = [torch.cuda.Event() for _ in range(2)]
        out_done = [torch.cuda.Event() for _ in range(2)]
        used = [False, False]
        graphs, outs_dev = [None, None], [None, None]
        if use_graph:
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            try:
                for sl in range(2):
                    t3 = dict(t)
                    t3["x"], t3["positions"] = xs_dev[sl], pos_dev[sl]
                    xs_dev[sl].copy_(t["x"])
                    pos_dev[sl].copy_(t["positions"])
                    with torch.cuda.stream(side):
                        for _ in range(2):
                            run_forward(mcc, t3, w, prec)
                    side.synchronize()
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        outs_dev[sl], _, _ = run_forward(mcc, t3, w, prec)
                    graphs[sl] = g
            except RuntimeError as e:   # a path that cannot be captured runs eagerly
                print(f"[bench] e2e {prec}: graph capture failed ({e}); eager calls", file=sys.stderr)
                graphs, outs_dev = [None, None], [None, None]
            stream.wait_stream(side)
            torch.cuda.synchronize()

        def serial_step():
            t2["x"] = x_host.to(dev, non_blocking=True)
            t2["positions"] = pos_host.to(dev, non_blocking=True)
            o, _, _ = run_forward(mcc, t2, w, prec)
            outs_host[0].copy_(o, non_blocking=True)

        def pipelined_step(k):
            sl = k % 2
            with torch.cuda.stream(h2d_s):
                if used[sl]:
                    h2d_s.wait_event(in_free[sl])      # step k-2 has consumed this input slot
                xs_dev[sl].copy_(x_host, non_blocking=True)
                pos_dev[sl].copy_(pos_host, non_blocking=True)
                in_ready[sl].record(h2d_s)
            stream.wait_event(in_ready[sl])
            if graphs[sl] is not None:
                # the slot's output buffer is overwritten by the replay: its previous
                # device->host copy (step k-2) must be done
                if used[sl]:
                    stream.wait_event(out_done[sl])
                graphs[sl].replay()
                o = outs_dev[sl]
            else:
                t2["x"], t2["positions"] = xs_dev[sl], pos_dev[sl]
                o, _, _ = run_forward(mcc, t2, w, prec)
            in_free[sl].record(stream)
            out_ready[sl].record(stream)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(out_ready[sl])
                outs_host[sl].copy_(o, non_blocking=True)
                if graphs[sl] is None:
                    o.record_stream(d2h_s)
                out_done[sl].record(d2h_s)
            used[sl] = True

        def pipelined(n):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            h2d_s.wait_event(e0)    # no copy of the timed steps starts before the start event
            d2h_s.wait_event(e0)
            for k in range(n):
                pipelined_step(k)
            for sl in range(2):
                if used[sl]:
                    stream.wait_event(out_done[sl])
            e1.record(stream)
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / n

        n_e = args.steps if prec == precision else n_att
        for _ in range(3):
            serial_step()
        torch.cuda.synchronize()
        barrier()
        s_ms = max_over_ranks(device_timed(stream, serial_step, n_e, warm=0), world, dev)
        pipelined(4)
        barrier()
        e_ms = max_over_ranks(pipelined(n_e), world, dev)
        return {"value": tokens_total / (e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e_ms,
                "h2d_bytes_per_step": x_host.numel() * x_host.element_size() + pos_host.numel() * 8,
                "d2h_bytes_per_step": outs_host[0].numel() * outs_host[0].element_size(),
                "overlap": "pipelined: each step's host->device and device->host copies on their own streams, "
                           "double-buffered, overlapping the neighbouring steps' compute"
                           + ("; the layer of each buffer slot replayed from a CUDA graph of the public-API calls"
                              if graphs[0] is not None else "; eager public-API calls"),
                "serial": {"value": tokens_total / (s_ms * 1e-3), "ms_per_step": s_ms},
                "resident": "KV cache (c_kv, pe_cache) and weights stay in HBM"}

    e2e = None
    if not args.no_e2e:
        e2e = e2e_run(precision)
        if not args.no_stages:
            for prec in stages:
                if prec != precision:
                    stages[prec]["e2e"] = e2e_run(prec)

    scen = time_scenarios(mcc, dev, stream) if (args.scenarios and rank == 0 and world == 1) else None
    ref_gpu = time_reference_gpu(mcc, dev, stream) if (args.reference_gpu and rank == 0 and world == 1) else None

    # ---- c2 key-sharded across all ranks (strong scaling), when several GPUs run
    key_c2 = None
    if world > 1 and shard == "batch" and not args.no_key_shard_c2:
        key_c2 = key_shard_c2(mcc, dev, rank, world, max(20, min(args.steps, 200)), precision)

    # our kernels per layer forward (fp32 storage): tensor = 2a1 GEMM, RMSNorm, 2a2 GEMM,
    # RoPE/gather, 2c GEMM, decode attention, segment combine, W_uv GEMM; exact = the
    # five Q-prep kernels and scores GEMM, softmax rows, P.c_kv GEMM, context reduce, W_uv GEMM
    launches_per_step = 10 if precision == "exact" else 8
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(w)
        parity = None
        if not args.no_parity and not KEY_SHARDED["on"]:
            parity = parity_sample(mcc, t, w, precision, sorted({0, B - 1}))
        dtype_name = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[w.dtype]
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "us_per_layer": ms * 1e3, "higher_is_better": True,
            "scaling": "weak" if shard == "batch" else "strong", "vs_baseline": None,
            "dtype": dtype_name if precision == "exact" else
                     ("bf16" if w.dtype != torch.float16 else "f16") + " tensor-core operands, f32 accumulate, "
                     + dtype_name + " storage",
            "data": "synthetic (seeded N(0,1) cache / activations, N(0,0.02) weights)",
            "config": line_config(w, world, shard),
            "precision": precision,
            "launch": ("CUDA graph of one layer forward (q_absorbed + mla_attention), replayed per step"
                       if use_graph else "eager calls per step")
                      + ("; W_q_a / W_q_b / W_uk / W_uv packed once to bf16 at load (q_absorbed_packed, "
                         "mla_attention_packed)" if PACKED["w"] is not None else "")
                      + (", Q-prep head-sharded + all-gather of q" if KEY_SHARDED["heads"] else ""),
            "stages": stages,
            "roofline": {"bound": "hbm",
                         "kernel": ("mla_decode_tc_kernel (tensor-core decode attention)"
                                    if dom_ms is kernel_ms else "mla_attention stage"),
                         "achieved": dom_gbs, "peak": hbm, "unit": "GB/s", "frac": dom_gbs / hbm,
                         "kernel_ms": dom_ms,
                         "traffic": TRAFFIC.get((args.config, precision, shard, world)),
                         "traffic_source": TRAFFIC_SOURCE,
                         "peak_source": peak_src + " (MEASURED_PEAKS.json hbm_gbs, burst copy)",
                         "algorithmic_bytes_per_launch": cache_b,
                         "algorithmic_bytes": "c_kv + pe_cache of this rank read once: B x Sk_local x 576 x "
                                              "element size",
                         "stage_frac": cache_b / (att_ms * 1e-3) / 1e9 / hbm,
                         "note": "achieved = algorithmic bytes / the decode kernel's average CUDA-event time "
                                 "(event pair around each launch on its stream); stage_frac uses the whole "
                                 "mla_attention stage (decode kernel + segment combine + W_uv projection)"},
            "tflops": {"q_absorbed": qf / (q_ms * 1e-3) / 1e12, "mla_attention": af / (att_ms * 1e-3) / 1e12},
            "clocks": clk.summary(),
            "gpu_launches": launches_per_step * args.steps,
            "device_status": dev_status,
            "parity": parity,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        if key_c2 is not None:
            line["key_shard_c2"] = key_c2
        if scen is not None:
            line["scenarios"] = scen
        if ref_gpu is not None:
            line["reference_gpu"] = ref_gpu
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        main_reference(a)
    else:
        main_ours(a)
