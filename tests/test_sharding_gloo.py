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


def test_key_sharded_attention_rejects_fp64_before_any_work():
    """fp64 would lose its accuracy in the fp32 merge weights: rejected before the
    partial attention or the collective runs (no process group is needed)."""
    from mla_custom_cuda import sharding
    qa = torch.zeros(1, 1, 128, 512, dtype=torch.float64)
    with pytest.raises(RuntimeError, match="fp64"):
        sharding.sk_sharded_attention(qa, qa[..., :64], qa[0], qa[0, ..., :64], qa[0], 1.0)


def _failing_rank_worker(rank, world, port, result_q):
    """Rank 1 leaves between steps (exits after step 0); rank 0 must learn it from
    its next collective, which ends with an error within the process group's
    short timeout instead of hanging."""
    import datetime
    import sys
    for p in (str(ROOT), str(PKG)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from mla_custom_cuda import sharding
    out = torch.randn(1, 1, 2, 8, dtype=torch.float32)
    lse = torch.randn(1, 1, 2)
    sharding.gather_partials(out, lse)            # step 0: both ranks
    if rank == 1:
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()
        os._exit(0)                                # leaves without tearing down the group
    try:
        sharding.gather_partials(out, lse)        # step 1: the peer is gone
        result_q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - any error from the collective is the signal
        result_q.put((rank, f"error: {type(e).__name__}"))
    result_q.close()
    result_q.join_thread()
    os._exit(0)


def test_rank_that_leaves_is_detected_by_the_next_collective():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        assert p.exitcode == 0
    res = dict(q.get() for _ in range(world))
    assert res[1] == "left"
    assert res[0].startswith("error"), res


def _init_failure_worker(port, result_q):
    """A rank whose peer never joins: init_process_group must fail with an error
    after its timeout (the host-side form of a failed communicator set-up)."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        result_q.put("joined")
    except Exception as e:  # noqa: BLE001
        result_q.put(f"error: {type(e).__name__}")
    result_q.close()
    result_q.join_thread()
    os._exit(0)


def test_process_group_init_failure_is_reported():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_init_failure_worker, args=(_free_port(), q))
    p.start()
    p.join(90)
    assert p.exitcode == 0
    assert q.get(timeout=5).startswith("error")
