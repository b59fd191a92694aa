"""The fused batch-1 decode kernel at the reference model's own default MoE
shape: hidden 4096, moe_inter 2048, 288 routed experts, top-8, one shared
expert (glm5::ModelConfig defaults, cpp/core/include/glm5/model_config.h:25,
59-60; Model::moe_forward, cpp/core/src/model.cpp:692-756).

A real GGUF of that model gets these values from its metadata, so the
persistent kernel is instantiated for H = 4096 (16 compute warps, down chunks
of 2048 rows, top-k over up to 512 experts) as well as for the BASELINE
shape.  The oracle needs only the picked experts' bytes: they are generated
from the same counter-based streams as the device layer (expert e's blocks
start at e * rows * in_dim / 256 of its matrix's stream), so the oracle runs a
compact layer of the picks with forced routing, and the picks themselves are
checked against an fp64 top-k of the router logits."""
import numpy as np
import pytest
import torch

from gpeed_b200 import Context, MoeConfig, MoeLayer, _capi
from oracle import oracle
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
LAYER_TOL = 1e-3  # relative L2, layer outputs (north star)
H, I, E, K = 4096, 2048, 288, 8
SEED, S0 = 77, 300


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def glm5_layer(ctx):
    cfg = MoeConfig(hidden=H, inter=I, n_experts=E)
    router = (np.random.default_rng(11).standard_normal((E, H)) * 0.02).astype(np.float32)
    return cfg, router, MoeLayer(ctx, cfg, layer_id=0).synth(router, None, SEED, S0)


def _compact_host(router, picks):
    """Host bytes of the picked experts (in pick order) and the shared expert."""
    gu, dn = I * H // 256, H * I // 256
    host = {
        "gate": np.concatenate([oracle.synth_iq3xxs(SEED, S0 + 0, gu, block0=int(e) * gu) for e in picks]),
        "up": np.concatenate([oracle.synth_iq3xxs(SEED, S0 + 1, gu, block0=int(e) * gu) for e in picks]),
        "down": np.concatenate([oracle.synth_iq3xxs(SEED, S0 + 2, dn, block0=int(e) * dn) for e in picks]),
        "gate_sh": oracle.synth_iq3xxs(SEED, S0 + 3, gu),
        "up_sh": oracle.synth_iq3xxs(SEED, S0 + 4, gu),
        "down_sh": oracle.synth_iq3xxs(SEED, S0 + 5, dn),
    }
    host["router"] = np.ascontiguousarray(router[np.asarray(picks)])
    host["corr"] = np.zeros(len(picks), np.float32)
    return host


def _fp64_topk(router, x):
    s = 1.0 / (1.0 + np.exp(-(router.astype(np.float64) @ x.astype(np.float64))))
    order = np.argsort(-s, kind="stable")
    return set(order[:K].tolist()), s[order[K - 1]] - s[order[K]]


def _fused_ran(ctx, fn):
    """Runs fn with per-stage profiling on; True when the layer ran as the one
    persistent kernel (the separate router / route / down / combine stages
    recorded nothing)."""
    import ctypes
    _capi.call("gpeed_ctx_profile", ctx.handle, 1)
    try:
        fn()
        stage = (ctypes.c_float * 5)()
        calls = ctypes.c_int()
        _capi.call("gpeed_ctx_profile_read", ctx.handle, stage, ctypes.byref(calls))
    finally:
        _capi.call("gpeed_ctx_profile", ctx.handle, 0)
    return stage[0] == 0 and stage[1] == 0 and stage[3] == 0 and stage[4] == 0 and stage[2] > 0


def test_glm5_shape_fused_decode_vs_oracle(ctx, port, glm5_layer):
    cfg, router, dev = glm5_layer
    shape = oracle.Shape(H, I, K, K, cfg.routed_scale, int(cfg.norm_topk), cfg.swiglu_limit)
    rng = np.random.default_rng(5)
    for trial in range(3):
        x = torch.from_numpy(rng.standard_normal((1, H)).astype(np.float32)).to(torch.bfloat16)
        ids = torch.empty(1, K, dtype=torch.int32, device="cuda")
        w = torch.empty(1, K, dtype=torch.float32, device="cuda")
        out = {}
        assert _fused_ran(ctx, lambda: out.setdefault("y", dev.forward(x.cuda(), topk_ids=ids, topk_w=w)))
        ctx.check()
        y = out["y"].cpu().numpy()[0]
        picks = ids.cpu().numpy()[0]
        assert len(set(picks.tolist())) == K and picks.min() >= 0 and picks.max() < E
        xf = x.float().numpy()[0]
        want, margin = _fp64_topk(router, xf)
        if margin > 1e-5:  # (a near-tie may flip with fp32 summation order)
            assert set(picks.tolist()) == want
        host = _compact_host(router, picks)
        y_o, k_o, w_o = port.moe_forward(shape, host, xf, forced=np.arange(K, dtype=np.int32))
        np.testing.assert_allclose(w.cpu().numpy()[0], w_o, rtol=1e-5)
        err = rel_l2(y, y_o)
        assert err < LAYER_TOL, (trial, err)


def test_glm5_shape_fused_matches_multi_kernel_path(ctx, glm5_layer):
    cfg, router, dev = glm5_layer
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16).cuda()
    ids_f = torch.empty(1, K, dtype=torch.int32, device="cuda")
    y_f = dev.forward(x, topk_ids=ids_f)
    ctx.check()
    ctx.set_option(_capi.OPT_FUSED_DECODE, 0)
    try:
        ids_m = torch.empty(1, K, dtype=torch.int32, device="cuda")
        y_m = dev.forward(x, topk_ids=ids_m)
        ctx.check()
    finally:
        ctx.set_option(_capi.OPT_FUSED_DECODE, 1)
    np.testing.assert_array_equal(ids_f.cpu().numpy(), ids_m.cpu().numpy())
    assert rel_l2(y_f.cpu().numpy(), y_m.cpu().numpy()) < 1e-5
    # forced routing that reaches the top of the expert range (ids 256..287 are
    # the top-k warp's candidate column 8, past the BASELINE kernel's 256)
    forced = torch.tensor([[287, 256, 3, 130, 271, 0, 200, 280]], dtype=torch.int32, device="cuda")
    y1 = dev.forward(x, forced_topk=forced)
    ctx.check()
    ctx.set_option(_capi.OPT_FUSED_DECODE, 0)
    try:
        y2 = dev.forward(x, forced_topk=forced)
        ctx.check()
    finally:
        ctx.set_option(_capi.OPT_FUSED_DECODE, 1)
    assert rel_l2(y1.cpu().numpy(), y2.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("world", [2, 8])
def test_glm5_shape_sliced_decode_partial(ctx, glm5_layer, world):
    """Expert-parallel decode at this shape with every rank holding 1/world of
    every expert's 64 units: each emulated rank's part (launches run one after
    another on one GPU; none waits on another) adds up to the one-GPU layer."""
    cfg, router, full = glm5_layer
    ctx2 = Context(0)  # the ranks' layers, freed with it
    try:
        parts = []
        for r in range(world):
            lo, cnt = MoeLayer.unit_slice(cfg, r, world)
            parts.append(MoeLayer(ctx2, cfg, layer_id=r).synth(router, None, SEED, S0).slice_units(lo, cnt))
        X = torch.from_numpy(np.random.default_rng(world).standard_normal((world, H)).astype(np.float32)).to(
            torch.bfloat16).cuda()
        y_ref = torch.empty(world, H, device="cuda")
        ids_ref = torch.empty(world, K, dtype=torch.int32, device="cuda")
        for t in range(world):
            full.forward(X[t:t + 1], y_ref[t:t + 1], topk_ids=ids_ref[t:t + 1])
        y_parts = []
        for r in range(world):
            ids = torch.full((world, K), -1, dtype=torch.int32, device="cuda")
            y_parts.append(parts[r].decode_partial(X, r, topk_ids=ids))
            ctx2.check()
            np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())
        y_ep = torch.stack(y_parts).sum(0).cpu().numpy()
        for t in range(world):
            assert rel_l2(y_ep[t], y_ref.cpu().numpy()[t]) < 1e-5
    finally:
        ctx2.close()
