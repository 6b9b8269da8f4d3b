"""Device-side failure reporting on the GPU, without faulting it.

Every mbarrier wait in the library's kernels is bounded; a wait that runs out
records a code in the per-device status block and the kernel returns. These
tests make a wait run out on purpose and check that the host sees the code,
and that the context stays usable: the next normal call is correct.
"""
from __future__ import annotations

import pytest
import torch

from conftest import rel_l2
import mla_configs as mc
from oracle import mla_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture()
def mcc():
    import mla_custom_cuda
    torch.cuda.synchronize()
    mla_custom_cuda.clear_device_status(DEV)
    yield mla_custom_cuda
    mla_custom_cuda.set_wait_limit_ns(0, DEV)       # default limit
    mla_custom_cuda.clear_device_status(DEV)


def _attention_ok(mcc):
    ins = [t.to(DEV) for t in mc.attention_inputs(2, 1, 700, seed=3)]
    out = mcc.mla_attention_ex(*ins, mc.SCALE, precision="tensor")
    ref = orc.mla_attention(*(t.double().cpu() for t in ins), scale=mc.SCALE)
    return rel_l2(out.cpu(), ref)


def test_status_starts_clear(mcc):
    assert mcc.device_status(DEV) == 0
    assert _attention_ok(mcc) < 2e-2
    assert mcc.device_status(DEV) == 0


def test_wait_that_runs_out_is_reported(mcc):
    """A bounded wait on a barrier that nothing completes: code 900 after the
    limit (1 ms), reported on the host; clearing it restores status 0 and the
    next tensor-core call is still correct."""
    mcc.set_wait_limit_ns(1_000_000, DEV)
    mcc.wait_selftest(DEV)
    assert mcc.device_status(DEV) == 900
    with pytest.raises(RuntimeError, match="device-side failure"):
        mcc.check_device(DEV)
    mcc.clear_device_status(DEV)
    assert mcc.device_status(DEV) == 0
    mcc.set_wait_limit_ns(0, DEV)
    assert _attention_ok(mcc) < 2e-2
    assert mcc.device_status(DEV) == 0
