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
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c1", choices=sorted(mc.CONFIGS))
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


def workload_bytes(w: mc.Workload, B: int):
    es = torch.tensor([], dtype=w.dtype).element_size()
    cache = B * w.sk * (w.kv_rank + w.rope) * es
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


def run_forward(mcc, t, w, precision):
    if KEY_SHARDED["heads"]:
        # each rank holds its heads' slices of W_q_b / W_uk: local Q-prep, all-gather of q
        from mla_custom_cuda import sharding
        qa, qr = sharding.head_sharded_q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"],
                                                  t["positions"], w.nope, w.rope, mc.EPS, precision=precision)
    else:
        qa, qr = mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                                   w.nope, w.rope, mc.EPS, precision=precision)
    if KEY_SHARDED["on"]:
        # every rank holds all sequences' queries and its own key slice; partial
        # attention, NCCL all-gather of (out, lse), exact log-sum-exp merge
        from mla_custom_cuda import sharding
        return sharding.sk_sharded_attention(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale,
                                             precision=precision), qa, qr
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
            "ms_per_step": best * 1e3,
            "sample": f"full {w.name} forward ({w.batch} sequences), fp32, oracle/mla_oracle.py "
                      f"(the reference's torch ops), best of {reps}"}


def main_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    w = mc.CONFIGS[args.config]
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
            "config": {**w.describe(), "note": "reference PyTorch path on host CPU cores"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"full {w.name} forward per step, oracle/mla_oracle.py (the reference's "
                                       f"torch ops), {threads} threads"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main_ours(args):
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("NCCL_DEBUG", "WARN")   # keep NCCL's banner off stdout (one JSON line)
        dist.init_process_group("nccl", device_id=dev)
    import mla_custom_cuda as mcc

    w = mc.CONFIGS[args.config]
    precision = args.precision
    B = w.batch
    shard = args.shard or ("keys" if args.config == "c2" else "batch")
    if world == 1:
        shard = "batch"
    if shard == "keys":
        if w.causal:
            raise SystemExit("key sharding is for non-causal decode")
        from mla_custom_cuda import sharding
        k0, k1 = sharding.key_shard(w.sk, rank, world)
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

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def timed(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    # ---- device-resident timed region (whole layer forward, headline precision).
    # The clock sampler starts before the warm-up, which runs for at least W steps
    # and at least --min-warmup-s seconds so nvidia-smi samples a loaded GPU.
    # Batch-sharded steps hold no collective: one layer forward (q_absorbed_ex +
    # mla_attention_ex, 9 kernels) is captured once in a CUDA graph and replayed
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
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        ms = float(tt.item())
    tokens_total = B * w.sq * (world if shard == "batch" else 1)
    value = tokens_total / (ms * 1e-3)

    # ---- per-stage timing (same stream, CUDA events; inputs larger than L2)
    n_att = max(5, args.steps)
    stages = {}
    for prec in ((precision,) if args.no_stages else ("tensor", "exact")):
        if KEY_SHARDED["heads"]:
            # local stages of a rank: Q-prep of its heads, attention over its key shard
            from mla_custom_cuda import sharding
            qa, qr = sharding.head_sharded_q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"],
                                                      t["positions"], w.nope, w.rope, mc.EPS, precision=prec)
            att = timed(lambda: mcc.mla_attention_partial(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale,
                                                          precision=prec), n_att)
        else:
            qa, qr = mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"],
                                       w.nope, w.rope, mc.EPS, precision=prec)
            att = timed(lambda: mcc.mla_attention_ex(qa, qr, t["c_kv"], t["pe_cache"], t["W_uv"], w.scale,
                                                     causal=w.causal, precision=prec), n_att)
        qp = timed(lambda: mcc.q_absorbed_ex(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"],
                                             t["positions"], w.nope, w.rope, mc.EPS, precision=prec), n_att)
        fwd = att + qp if prec != precision else ms
        stages[prec] = {"q_absorbed_ms": qp, "mla_attention_ms": att, "layer_ms": fwd,
                        "tokens_per_s": B * w.sq / (fwd * 1e-3)}
    att_ms = stages[precision]["mla_attention_ms"]
    q_ms = stages[precision]["q_absorbed_ms"]

    cache_b, weight_b, act_b = workload_bytes(w, B)
    qf, af = workload_flops(w, B)
    hbm, bf16_tf, peak_src = peaks()
    att_gbs = cache_b / (att_ms * 1e-3) / 1e9

    # ---- end to end through the public API: the step's hidden states come from
    # pinned host memory and the layer output goes back to pinned host memory;
    # the KV cache and weights stay resident in HBM, as in a decode server.
    e2e = None
    if not args.no_e2e:
        x_host = t["x"].cpu().pin_memory()
        pos_host = t["positions"].cpu().pin_memory()
        out_host = torch.empty((B, w.sq, w.heads, w.v_dim), dtype=w.dtype).pin_memory()
        t2 = dict(t)

        def e2e_step():
            t2["x"] = x_host.to(dev, non_blocking=True)
            t2["positions"] = pos_host.to(dev, non_blocking=True)
            o, _, _ = run_forward(mcc, t2, w, precision)
            out_host.copy_(o, non_blocking=True)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / args.steps
        if world > 1:
            tt = torch.tensor([e_ms], device=dev)
            torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
            e_ms = float(tt.item())
        e2e = {"value": tokens_total / (e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": x_host.numel() * x_host.element_size() + pos_host.numel() * 8,
               "d2h_bytes_per_step": out_host.numel() * out_host.element_size(),
               "resident": "KV cache (c_kv, pe_cache) and weights stay in HBM"}

    # our kernels per layer forward (fp32 storage): tensor = 2a1 GEMM, RMSNorm, 2a2 GEMM,
    # RoPE/gather, 2c GEMM, decode attention, segment combine, W_uv GEMM; exact = the
    # five Q-prep kernels and scores GEMM, softmax rows, P.c_kv GEMM, context reduce, W_uv GEMM
    launches_per_step = 10 if precision == "exact" else 8
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(w)
        dtype_name = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[w.dtype]
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "us_per_layer": ms * 1e3, "higher_is_better": True,
            "scaling": "weak" if shard == "batch" else "strong", "vs_baseline": None,
            "dtype": dtype_name if precision == "exact" else
                     ("bf16" if w.dtype != torch.float16 else "f16") + " tensor-core operands, f32 accumulate, "
                     + dtype_name + " storage",
            "data": "synthetic (seeded N(0,1) cache / activations, N(0,0.02) weights)",
            "config": {**w.describe(), "global_batch": B * (world if shard == "batch" else 1), "precision": precision,
                       "launch": ("CUDA graph of one layer forward (q_absorbed_ex + mla_attention_ex), replayed per step"
                                  if use_graph else "eager calls per step"),
                       "parallelism": f"batch-shard dp{world}" if shard == "batch" else (f"key-shard sp{world} (NCCL all-gather + LSE merge)" + (", Q-prep head-sharded + all-gather of q" if KEY_SHARDED["heads"] else "")),
                       "l2": "inputs larger than L2 (cache %.2f GB per GPU)" % (cache_b / 1e9)},
            "stages": stages,
            "roofline": {"bound": "hbm", "kernel": "mla_attention (cache read)",
                         "achieved": att_gbs, "peak": hbm, "unit": "GB/s", "frac": att_gbs / hbm,
                         "traffic": (1.565e9 if (args.config == "c1" and precision == "tensor" and shard == "batch") else None),
                         "traffic_source": "ncu capture of mla_decode_tc_kernel at c1: dram__bytes_read.sum + "
                                           "dram__bytes_write.sum per launch (1.530 GB + 0.035 GB)",
                         "peak_source": peak_src,
                         "algorithmic_bytes_per_launch": cache_b,
                         "note": "mla_attention stage = fused tcgen05 decode kernel + segment combine + W_uv "
                                 "projection; algorithmic bytes = c_kv + pe_cache read once"},
            "tflops": {"q_absorbed": qf / (q_ms * 1e-3) / 1e12, "mla_attention": af / (att_ms * 1e-3) / 1e12},
            "clocks": clk.summary(),
            "gpu_launches": launches_per_step * args.steps,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        main_reference(a)
    else:
        main_ours(a)
