"""Failure detection on the GPU without a GPU fault.

The fused batch-1 kernel waits on data that other CTAs publish (router
logits, finished h units, split down rows).  Every wait is bounded: after
GPEED_OPT_SPIN_LIMIT polls it gives up, sets a timeout bit in the context's
status word and the kernel finishes with invalid results, so the context
stays usable.  The test makes one such wait run out on purpose with a short
limit and a flag that nothing sets (the test-only option that withholds one
router logit), checks that gpeed_ctx_check reports and clears it, and that the
next forward gives the same result as before.  The reference has no device and
only throws (weights.cpp:21,25)."""
import re

import pytest
import torch

from gpeed_b200 import Context, GpeedError, MoeConfig, MoeLayer
from gpeed_b200 import _capi
from tests.helpers import host_layer, rel_l2

pytestmark = pytest.mark.gpu


def test_fused_wait_that_runs_out_is_reported_and_recovered():
    ctx = Context(0)
    cfg = MoeConfig()
    host = host_layer(cfg.hidden, cfg.inter, cfg.n_experts, seed=42, stream0=100, router_seed=1)
    layer = MoeLayer(ctx, cfg).synth(host["router"], host["corr"], 42, 100)
    x = torch.randn(1, cfg.hidden, generator=torch.Generator().manual_seed(11)).to(torch.bfloat16).cuda()
    y_ok = layer.forward(x)
    ctx.check()
    ctx.set_option(_capi.OPT_SPIN_LIMIT, 1 << 12)
    ctx.set_option(_capi.OPT_TEST_WITHHOLD_LOGIT, 5)
    try:
        layer.forward(x)
        with pytest.raises(GpeedError) as e:
            ctx.check()
        assert e.value.code == _capi.ERR_DEVICE
        status = int(re.search(r"device status 0x([0-9a-f]+)", str(e.value)).group(1), 16)
        assert status & 1  # GP_DEV_TIMEOUT_FULL: a consumer gave up waiting
    finally:
        ctx.set_option(_capi.OPT_TEST_WITHHOLD_LOGIT, -1)
        ctx.set_option(_capi.OPT_SPIN_LIMIT, _capi.SPIN_LIMIT_DEFAULT)
    ctx.check()  # the flag was cleared with the counters and tags
    for _ in range(2):
        y = layer.forward(x)
        ctx.check()
        assert rel_l2(y.cpu().numpy(), y_ok.cpu().numpy()) < 1e-6  # sums into y in launch order: to rounding
    with pytest.raises(GpeedError):
        ctx.set_option(_capi.OPT_SPIN_LIMIT, 0)
    ctx.close()
