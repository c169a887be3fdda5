"""The tensor-core kernels' bounded waits, made to run out on purpose.

Every mbarrier wait in the tcgen05 kernels gives up after a wall-time limit,
sets the context's device status word and unwinds (tensor memory freed,
copies in flight drained), so a stalled pipeline ends as an error status the
host reads instead of a hung GPU.  Here the limit is set to 1 ms and the
next forward withholds the copy of its first key tile (a barrier that
nothing completes, before any MMA is issued): kattn_check_device must report
KATTN_ERR_DEVICE_TIMEOUT, and the next ordinary calls on the same context
must still match the oracle.  Nothing faults: the kernel only waits on a
barrier that no copy will complete, for at most the limit.
"""
import numpy as np
import pytest
import torch

import kerr_attn
from conftest import make_inputs
from test_gpu_parity import assert_parity, gpu_fwd_bwd, oracle_fwd_bwd

pytestmark = pytest.mark.gpu


def test_withheld_load_times_out_then_context_recovers(oracle_lib):
    B, T, H, d = 2, 130, 2, 64
    C = H * d
    qkv, dout = make_inputs(B, T, H, d, seed=77)
    dev = torch.device("cuda", 0)
    with kerr_attn.Context(0) as ctx:
        ctx.set_path(kerr_attn.PATH_TENSOR)
        ctx.check_device()  # no stale flag
        ctx.set_wait_limit(1_000_000)  # 1 ms
        x = torch.from_numpy(qkv).to(dev)
        q, k, v = kerr_attn.split_qkv(x, C)
        o = torch.empty(B, T, C, device=dev)
        lse = torch.empty(B, H, T, device=dev)
        ctx.test_withhold_next_load()
        assert kerr_attn.fwd(ctx, q, k, v, o, lse, H) == 1  # enqueued normally
        with pytest.raises(kerr_attn.KattnError) as e:
            ctx.check_device()
        assert e.value.status == kerr_attn.KATTN_ERR_DEVICE_TIMEOUT
        ctx.check_device()  # the flag was cleared by the report
        # The same context, default limit again: ordinary calls match the oracle.
        ctx.set_wait_limit(0)
        got = gpu_fwd_bwd(ctx, qkv, dout, H, path="tensor")
        assert_parity(got, oracle_fwd_bwd(oracle_lib, qkv, dout, H), case="after a timeout")


def test_wait_limit_argument_checks():
    lib = kerr_attn.lib()
    assert lib.kattn_set_wait_limit(None, 5) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
    assert lib.kattn_test_withhold_next_load(None) == kerr_attn.KATTN_ERR_INVALID_ARGUMENT
