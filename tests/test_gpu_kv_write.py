"""KV-cache write (mla_kv_cache_write): new tokens' rows of c_kv and pe_cache
against the oracle's composition of the reference's rmsnorm and apply_rope
(oracle.kv_cache_rows), written at the requested slots and nowhere else.
Tolerances: exact fp32 rel-L2 1e-5 against the fp32 path (the reference's
arithmetic in fp32), tensor / 16-bit 2e-2 against fp64."""
from __future__ import annotations

import pytest
import torch

from conftest import rel_l2
import mla_configs as mc
from oracle import mla_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _case(B, Sq, cap, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, Sq, mc.HIDDEN, generator=g)
    W = torch.randn(mc.HIDDEN, mc.KV_RANK + mc.ROPE, generator=g) * 0.02
    gain = 1.0 + 0.1 * torch.randn(mc.KV_RANK, generator=g)
    pos = torch.arange(cap - Sq + 1, cap + 1, dtype=torch.int64)
    slots = torch.arange(cap - Sq, cap, dtype=torch.int64)
    return x.to(dtype), W.to(dtype), gain.to(dtype), pos, slots


@pytest.mark.parametrize("dtype,precision", [(torch.float32, "exact"), (torch.float32, "tensor"),
                                             (torch.bfloat16, "tensor"), (torch.float16, "exact")])
@pytest.mark.parametrize("B,Sq,cap", [(1, 1, 64), (4, 3, 300), (128, 1, 4989)])
def test_kv_cache_write_vs_oracle(dtype, precision, B, Sq, cap):
    import mla_custom_cuda as mcc
    x, W, gain, pos, slots = _case(B, Sq, cap, dtype, seed=B * 31 + Sq)
    c_kv = torch.full((B, cap, mc.KV_RANK), 7.0, dtype=dtype, device=DEV)
    pe = torch.full((B, cap, mc.ROPE), 7.0, dtype=dtype, device=DEV)
    mcc.kv_cache_write(x.to(DEV), W.to(DEV), gain.to(DEV), pos.to(DEV), slots.to(DEV), c_kv, pe, mc.EPS,
                       precision=precision)
    assert mcc.device_status(DEV) == 0
    got_c, got_p = c_kv[:, slots].cpu(), pe[:, slots].cpu()
    r64 = orc.kv_cache_rows(x.double(), W.double(), gain.double(), pos, mc.KV_RANK, mc.EPS)
    if dtype == torch.float32 and precision == "exact":
        r32 = orc.kv_cache_rows(x, W, gain, pos, mc.KV_RANK, mc.EPS)
        assert rel_l2(got_c, r32[0]) < 1e-5 and rel_l2(got_p, r32[1]) < 1e-5
    assert rel_l2(got_c.double(), r64[0]) < 2e-2 and rel_l2(got_p.double(), r64[1]) < 2e-2
    # every other slot is untouched
    keep = torch.ones(cap, dtype=torch.bool)
    keep[slots] = False
    assert (c_kv[:, keep.to(DEV)] == 7.0).all() and (pe[:, keep.to(DEV)] == 7.0).all()


def test_kv_cache_write_slot_out_of_range_is_reported_not_written():
    import mla_custom_cuda as mcc
    mcc.clear_device_status(DEV)
    x, W, gain, pos, _ = _case(2, 1, 16, torch.float32, seed=5)
    c_kv = torch.zeros(2, 16, mc.KV_RANK, device=DEV)
    pe = torch.zeros(2, 16, mc.ROPE, device=DEV)
    mcc.kv_cache_write(x.to(DEV), W.to(DEV), gain.to(DEV), pos.to(DEV), torch.tensor([16], device=DEV), c_kv, pe)
    assert mcc.device_status(DEV) == 950
    assert (c_kv == 0).all() and (pe == 0).all()
    mcc.clear_device_status(DEV)
    assert mcc.device_status(DEV) == 0


def test_written_cache_feeds_the_decode_path():
    """A token written by kv_cache_write at the last slot and attended by
    mla_attention gives the oracle's layer output over the same cache."""
    import mla_custom_cuda as mcc
    B, Sk = 2, 500
    x, W, gain, pos, slots = _case(B, 1, Sk, torch.float32, seed=9)
    g = torch.Generator().manual_seed(3)
    c_kv = torch.randn(B, Sk, mc.KV_RANK, generator=g)
    pe = torch.randn(B, Sk, mc.ROPE, generator=g)
    cg, pg = c_kv.to(DEV), pe.to(DEV)
    mcc.kv_cache_write(x.to(DEV), W.to(DEV), gain.to(DEV), pos.to(DEV), slots.to(DEV), cg, pg, precision="exact")
    rc, rp = orc.kv_cache_rows(x, W, gain, pos, mc.KV_RANK, mc.EPS)
    c_ref, p_ref = c_kv.clone(), pe.clone()
    c_ref[:, slots], p_ref[:, slots] = rc, rp
    qa, qr, _, _, wuv = mc.attention_inputs(B, 1, Sk, seed=4)
    out = mcc.mla_attention_ex(qa.to(DEV), qr.to(DEV), cg, pg, wuv.to(DEV), mc.SCALE, precision="exact")
    ref = orc.mla_attention(qa.double(), qr.double(), c_ref.double(), p_ref.double(), wuv.double(), mc.SCALE)
    assert rel_l2(out.cpu(), ref) < 1e-5
