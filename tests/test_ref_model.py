"""Parity against the reference engine's own glm5::Model.

tests/golden/ref_model.npz holds what the reference's Model::hc_forward (+ the
ffn RMSNorm, model.cpp:205-263, 295-297) and Model::moe_forward
(model.cpp:692-756) compute for the cases in tests.helpers.REF_MODEL_CASES,
each loaded by the reference from a one-block GGUF file
(tests/golden/make_golden.py, oracle/ref_model_harness.cpp).  The CPU tests pin
the oracle to those outputs; the GPU tests load the same GGUF file through the
product's reader and compare the device path with them."""
import os

import numpy as np
import pytest

from tests.helpers import HC_EPS, HC_ITERS, HC_N, HC_RMS_EPS, REF_MODEL_CASES, ref_model_case, rel_l2, \
    write_ref_model_gguf

GOLD = os.path.join(os.path.dirname(__file__), "golden")
LAYER_TOL = 1e-3  # relative L2, layer outputs
CASES = sorted(REF_MODEL_CASES)


@pytest.fixture(scope="module")
def fixture():
    return np.load(os.path.join(GOLD, "ref_model.npz"))


@pytest.fixture(scope="module")
def cases():
    return {name: ref_model_case(name) for name in CASES}


def test_restated_harness_is_the_engine(fixture):
    """The single-token harness behind moe_tiny.npz restates moe_forward around
    the reference's compiled quant.cpp; the engine itself gives the same bits."""
    tiny = np.load(os.path.join(GOLD, "moe_tiny.npz"))
    assert np.array_equal(fixture["tiny_y"].view(np.uint32), tiny["fwd_y"].view(np.uint32))


@pytest.mark.parametrize("name", CASES)
def test_oracle_moe_forward_is_bit_exact_with_the_engine(port, fixture, cases, name):
    from oracle import oracle
    c = cases[name]
    shape = oracle.Shape(c["H"], c["I"], c["E"], c["K"], 2.5, 1, 10.0)
    for i in range(c["n"]):
        y, _, _ = port.moe_forward(shape, c["layer"], c["X"][i])
        assert np.array_equal(y.view(np.uint32), fixture[f"{name}_y"][i].view(np.uint32)), i


@pytest.mark.parametrize("name", CASES)
def test_oracle_mhc_matches_the_engine(port, fixture, cases, name):
    """The oracle sums in plain order, the engine with 8-lane AVX2 partial sums
    (ops.h dot_f32 / rmsnorm): agreement to fp32 rounding."""
    c = cases[name]
    x, post, comb = port.mhc_pre(c["streams"], c["fn"], c["base"], c["scale"], c["norm_w"], HC_N, HC_ITERS, HC_EPS,
                                 HC_RMS_EPS)
    assert rel_l2(x, fixture[f"{name}_x"]) < 1e-6
    np.testing.assert_allclose(post, fixture[f"{name}_post"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(comb, fixture[f"{name}_comb"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("name", CASES)
def test_gguf_reader_sees_the_engines_config(tmp_path, cases, name):
    """The product's GGUF reader derives the MoE fields ModelConfig::from_gguf
    derives (model_config.cpp:80-95) from the same file."""
    from gpeed_b200.gguf import GgufModel
    c = cases[name]
    path = str(tmp_path / f"{name}.gguf")
    write_ref_model_gguf(path, c)
    with GgufModel(path) as m:
        cfg = m.moe_config(0)
    assert (cfg.hidden, cfg.inter, cfg.n_experts, cfg.top_k) == (c["H"], c["I"], c["E"], c["K"])
    assert (cfg.routed_scale, cfg.norm_topk, cfg.swiglu_limit) == (2.5, True, 10.0)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_gpu_layer_from_the_engines_gguf(tmp_path, fixture, cases, name):
    """Same GGUF file, product reader + device path vs the engine: per token
    (the batch-1 path; the fused persistent kernel at hidden 5120) and as one
    batch, fp32 and bf16 inputs; then the mHC -> MoE chain of layer_forward."""
    import torch
    from gpeed_b200 import Context, MoeLayer
    from gpeed_b200.gguf import GgufModel
    from gpeed_b200.moe import MhcParams, mhc_pre
    c = cases[name]
    path = str(tmp_path / f"{name}.gguf")
    write_ref_model_gguf(path, c)
    ctx = Context(0)
    with GgufModel(path) as m:
        layer = MoeLayer.from_gguf(ctx, m, 0)
    want = fixture[f"{name}_y"]
    X = torch.from_numpy(c["X"]).cuda()
    for i in range(c["n"]):
        y = layer.forward(X[i:i + 1])
        ctx.check()
        assert rel_l2(y.cpu().numpy()[0], want[i]) < LAYER_TOL, (i, rel_l2(y.cpu().numpy()[0], want[i]))
    Y = layer.forward(X)
    ctx.check()
    assert rel_l2(Y.cpu().numpy(), want) < LAYER_TOL
    Yb = layer.forward(X.to(torch.bfloat16))
    ctx.check()
    assert rel_l2(Yb.cpu().numpy(), want) < 4e-3  # bf16 inputs: one rounding of x (~2e-3 relative)

    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda()
           for a in (c["streams"], c["fn"], c["base"], c["scale"], c["norm_w"])]
    x, post, comb = mhc_pre(ctx, *dev, params=MhcParams(HC_N, HC_ITERS, HC_EPS, HC_RMS_EPS),
                            x_dtype=torch.float32)
    ctx.check()
    assert rel_l2(x.cpu().numpy(), fixture[f"{name}_x"]) < 1e-5
    np.testing.assert_allclose(post.cpu().numpy(), fixture[f"{name}_post"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(comb.cpu().numpy(), fixture[f"{name}_comb"], rtol=1e-4, atol=1e-6)
    chain = fixture[f"{name}_chain_y"]
    for i in range(c["n"]):
        y = layer.forward(x[i:i + 1])
        ctx.check()
        assert rel_l2(y.cpu().numpy()[0], chain[i]) < LAYER_TOL
    ctx.close()
