"""Key-sharded attention over NCCL on two GPUs (one process per GPU): each rank
holds its half of every sequence's keys, runs mla_attention_partial, the
partials are all-gathered and merged (sharding.sk_sharded_attention). Every
rank's output must equal attention over all keys on one GPU (same precision)
and the fp64 oracle. Skipped when fewer than two GPUs are visible."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    for p in (str(ROOT), str(PKG)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        import mla_configs as mc
        import mla_custom_cuda as mcc
        from mla_custom_cuda import sharding
        from oracle import mla_oracle as orc
        res = {}
        qa, qr, ck, pe, wuv = mc.attention_inputs(2, 1, 6000, seed=31)
        k0, k1 = sharding.key_shard(6000, rank, world)
        g = [t.to(dev) for t in (qa, qr, ck[:, k0:k1], pe[:, k0:k1], wuv)]
        ref = orc.mla_attention(*(t.double() for t in (qa, qr, ck, pe, wuv)), scale=mc.SCALE)
        for prec, tol in (("exact", 1e-5), ("tensor", 2e-2)):
            out = sharding.sk_sharded_attention(*g, mc.SCALE, precision=prec)
            full = mcc.mla_attention_ex(qa.to(dev), qr.to(dev), ck.to(dev), pe.to(dev), wuv.to(dev), mc.SCALE,
                                        precision=prec)
            torch.cuda.synchronize()
            e_full = float((out.double() - full.double()).norm() / full.double().norm())
            e_ref = float((out.double().cpu() - ref).norm() / ref.norm())
            res[prec] = (e_full, e_ref, tol)
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_key_sharded_attention_over_nccl_two_gpus():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(world))
    for rank, r in res.items():
        for prec, (e_full, e_ref, tol) in r.items():
            assert e_full < tol and e_ref < tol, (rank, prec, e_full, e_ref)
