"""Multi-rank host logic of the sharded layouts, on CPU ranks with gloo:
key-shard ranges, the all-gather of partials in rank order and the exact
log-sum-exp merge (with the oracle's partial attention standing in for the GPU
kernel), and batch-shard ranges."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, ROOT, rel_l2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import sys
    for p in (str(ROOT), str(PKG)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import mla_configs as mc
        from mla_custom_cuda import sharding
        from oracle import mla_oracle as orc
        qa, qr, ck, pe, wuv = (t.double() for t in mc.attention_inputs(2, 2, 97, seed=21))
        k0, k1 = sharding.key_shard(97, rank, world)
        out, lse = orc.mla_attention_partial(qa, qr, ck[:, k0:k1], pe[:, k0:k1], wuv, mc.SCALE)
        outs, lses = sharding.gather_partials(out, lse)
        merged, L = orc.lse_combine(outs, lses)
        full = orc.mla_attention(qa, qr, ck, pe, wuv, mc.SCALE)
        _, full_lse = orc.mla_attention_partial(qa, qr, ck, pe, wuv, mc.SCALE)
        result_q.put((rank, rel_l2(merged, full), rel_l2(L, full_lse)))
    finally:
        dist.destroy_process_group()


def _heads_worker(rank, world, port, result_q):
    import sys
    for p in (str(ROOT), str(PKG)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import mla_configs as mc
        from mla_custom_cuda import sharding
        from oracle import mla_oracle as orc
        small = mc.Workload("small", 3, 2, 19, hidden=96, heads=4, q_lora=48, kv_rank=32, nope=16, rope=8, v_dim=24)
        t = {k: (v.double() if v.is_floating_point() else v) for k, v in mc.make_inputs(small, seed=3).items()}
        Wqb_l, Wuk_l = sharding.shard_q_weights(t["W_q_b"], t["W_uk"], 16, 8, rank, world)
        qa_l, qr_l = orc.q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], Wqb_l, Wuk_l, t["positions"], 16, 8)
        qa, qr = sharding.gather_heads([qa_l, qr_l])
        ra, rr = orc.q_absorbed(t["x"], t["W_q_a"], t["q_norm_w"], t["W_q_b"], t["W_uk"], t["positions"], 16, 8)
        result_q.put((rank, rel_l2(qa, ra), rel_l2(qr, rr)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_q_prep_on_gloo(world):
    """Each rank's head slices of W_q_b / W_uk give its heads' queries, and the
    all-gather reassembles the full q in head order (oracle as the per-rank Q-prep)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_heads_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get() for _ in range(world))
    for rank, e_a, e_r in res:
        assert e_a < 1e-14 and e_r < 1e-14, (rank, e_a, e_r)


@pytest.mark.parametrize("world", [2, 3])
def test_key_sharded_merge_on_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get() for _ in range(world))
    for rank, e_out, e_lse in res:
        assert e_out < 1e-12 and e_lse < 1e-12, (rank, e_out, e_lse)


def test_shard_ranges_cover_exactly():
    from mla_custom_cuda import sharding
    for n, world in [(65536, 8), (4989, 3), (7, 4), (0, 2), (128, 8)]:
        spans = [sharding.key_shard(n, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        sizes = [e - s for s, e in spans]
        assert max(sizes) - min(sizes) <= 1
        assert sharding.batch_shard(n, 0, world) == spans[0]
    with pytest.raises(ValueError):
        sharding.key_shard(10, 4, 4)


def _partials_dtype_worker(rank, world, port, result_q):
    import sys
    for p in (str(ROOT), str(PKG)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mla_custom_cuda import sharding
        g = torch.Generator().manual_seed(100 + rank)
        ok = True
        for out_dtype in (torch.float32, torch.float16):
            out = torch.randn(2, 3, 4, 8, generator=g).to(out_dtype)
            lse = torch.randn(2, 3, 4, generator=g)
            outs, lses = sharding.gather_partials(out, lse)
            # every rank's slice arrives in rank order, dtypes kept
            mine_ok = torch.equal(outs[rank], out) and torch.equal(lses[rank], lse)
            ok = ok and mine_ok and outs.dtype == out_dtype and lses.dtype == torch.float32
            ok = ok and tuple(outs.shape) == (world, 2, 3, 4, 8) and tuple(lses.shape) == (world, 2, 3, 4)
        result_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_gather_partials_keeps_rank_order_and_dtypes():
    """One collective when out and lse share a dtype, two (lse kept in fp32) otherwise."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_partials_dtype_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get() for _ in range(world))
    assert all(ok for _, ok in res), res
