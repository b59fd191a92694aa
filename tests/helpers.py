"""Shared builders for parity tests: the same seeded layer on host (for the
oracle) and on the device (for the CUDA path)."""
from __future__ import annotations

import numpy as np

from oracle import oracle

STREAMS = ("gate", "up", "down", "gate_sh", "up_sh", "down_sh")


def host_layer(H, I, E, seed, stream0, router_seed=0, corr=None, shared=True):
    """Raw IQ3_XXS bytes from the host twin of the device generator + fp32 router."""
    nb = lambda rows, inn: rows * inn // 256
    sizes = [nb(E * I, H), nb(E * I, H), nb(E * H, I), nb(I, H), nb(I, H), nb(H, I)]
    layer = {}
    for m, name in enumerate(STREAMS[: 6 if shared else 3]):
        layer[name] = oracle.synth_iq3xxs(seed, stream0 + m, sizes[m])
    rng = np.random.default_rng(router_seed)
    layer["router"] = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    layer["corr"] = np.zeros(E, np.float32) if corr is None else np.asarray(corr, np.float32)
    return layer


def zipf_bias(E, s=1.1, beta=0.25, seed=3):
    """Selection bias (the reference's exp_probs_b) that skews expert loads
    toward a Zipf(s) profile: b_e = beta * (-s * ln(rank_e + 1)) over a seeded
    random ranking of the experts."""
    rank = np.random.default_rng(seed).permutation(E)
    return (beta * (-s * np.log(rank + 1.0))).astype(np.float32)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ggml type id -> (bytes per block, values per block, byte offsets of fp16 scales)
CODECS = {8: (34, 32, (0,)), 10: (84, 256, (80, 82)), 11: (110, 256, (108,)), 14: (210, 256, (208,)),
          18: (98, 256, (0,)), 21: (110, 256, (0,)), 22: (82, 256, (0,)), 23: (136, 256, (0,)),
          1: (2, 1, ()), 30: (2, 1, ())}
CODEC_NAMES = {8: "Q8_0", 10: "Q2_K", 11: "Q3_K", 14: "Q6_K", 18: "IQ3_XXS", 21: "IQ3_S", 22: "IQ2_S",
               23: "IQ4_XS", 1: "F16", 30: "BF16"}


def codec_blocks(dtype: int, nblocks: int, seed: int) -> np.ndarray:
    """Seeded random GGUF blocks of `dtype` (uint8 [nblocks * bytes]): random
    payload bytes, fp16 scales drawn from [1e-4, 2e-3) (element-wise types:
    random finite halves / bf16 values)."""
    bb, vals, dofs = CODECS[dtype]
    rng = np.random.default_rng(seed)
    blk = np.frombuffer(rng.bytes(bb * nblocks), np.uint8).reshape(nblocks, bb).copy()
    for o in dofs:
        d = (1e-4 + 1.9e-3 * rng.random(nblocks)).astype(np.float16)
        blk[:, o:o + 2] = np.frombuffer(d.tobytes(), np.uint8).reshape(nblocks, 2)
    return blk.reshape(-1)


def codec_edge_blocks(dtype: int) -> np.ndarray:
    """Edge cases: zero, negative, subnormal, largest, infinite and NaN fp16
    scales, all-zero and all-one payloads."""
    bb, vals, dofs = CODECS[dtype]
    rng = np.random.default_rng(dtype)
    out = []
    for dbits in (0x0000, 0x8000, 0x0001, 0x03FF, 0x7BFF, 0xFBFF, 0x7C00, 0x7E01):
        for fill in (None, 0x00, 0xFF):
            b = np.frombuffer(rng.bytes(bb), np.uint8).copy() if fill is None else np.full(bb, fill, np.uint8)
            for o in dofs:
                b[o] = dbits & 0xFF
                b[o + 1] = dbits >> 8
            out.append(b)
    return np.concatenate(out)


def hashed_uniform(shape, seed: int, scale: float = 1.0) -> np.ndarray:
    """Deterministic float32 values in [-scale, scale): splitmix64 of
    (seed, element index), top 24 bits as an exact fraction.  Independent of
    numpy's generator streams, so fixtures need store only outputs."""
    n = int(np.prod(shape))
    with np.errstate(over="ignore"):
        z = (np.arange(1, n + 1, dtype=np.uint64) + np.uint64(seed) * np.uint64(0xD1B54A32D192ED03)) \
            * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    u = (z >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -23) - np.float32(1.0)
    return (u * np.float32(scale)).reshape(shape)


# Model-level cases run through the reference engine's own glm5::Model
# (oracle/ref_model_harness.cpp; outputs in tests/golden/ref_model.npz).
# Each is one GGUF holding one block's mHC (hc_ffn_*, ffn_norm) and MoE
# tensors; the MoE layer's expert bytes come from the counter-based generator.
HC_N, HC_ITERS, HC_EPS, HC_RMS_EPS = 4, 20, 1e-6, 1e-5
REF_MODEL_CASES = {
    # hidden, moe_inter, experts, top_k, tokens, input seed, weight seed, first stream
    "h512": dict(H=512, I=512, E=8, K=2, n=3, seed=11, wseed=7, stream0=21),
    "h5120": dict(H=5120, I=1536, E=16, K=4, n=2, seed=12, wseed=7, stream0=31),
}


def ref_model_case(name: str) -> dict:
    """Inputs of one model-level case: mHC parameters and streams, the MoE
    layer (raw IQ3_XXS bytes + fp32 router and bias) and MoE input tokens."""
    c = dict(REF_MODEL_CASES[name])
    H, I, E, N, n, s = c["H"], c["I"], c["E"], HC_N, c["n"], c["seed"]
    W = (2 + N) * N
    c["streams"] = hashed_uniform((n, N, H), s * 16 + 0, 2.0)
    c["fn"] = hashed_uniform((W, N * H), s * 16 + 1, 2.0 ** -6)
    c["base"] = hashed_uniform(W, s * 16 + 2, 1.0)
    c["scale"] = np.array([0.8, 1.1, 1.3], np.float32)
    c["norm_w"] = (1.0 + hashed_uniform(H, s * 16 + 3, 0.125)).astype(np.float32)
    c["router"] = hashed_uniform((E, H), s * 16 + 4, 0.03)
    c["corr"] = hashed_uniform(E, s * 16 + 5, 0.05)
    c["X"] = hashed_uniform((n, H), s * 16 + 6, 2.0)
    nb = lambda rows, inn: rows * inn // 256
    sizes = [nb(E * I, H), nb(E * I, H), nb(E * H, I), nb(I, H), nb(I, H), nb(H, I)]
    c["layer"] = {k: oracle.synth_iq3xxs(c["wseed"], c["stream0"] + m, sizes[m]) for m, k in enumerate(STREAMS)}
    c["layer"]["router"], c["layer"]["corr"] = c["router"], c["corr"]
    return c


def write_ref_model_gguf(path: str, c: dict) -> None:
    """The case as a one-block glm5-next GGUF the reference's Model loads
    (block_count 2: one layer plus the excluded MTP block)."""
    from tests.gguf_writer import F32, U32, moe_block_tensors, moe_metadata, write_gguf
    H, I, E, K, N = c["H"], c["I"], c["E"], c["K"], HC_N
    a = "glm5-next."
    kvs = moe_metadata("glm5-next", H, I, E, K) + [
        (a + "block_count", U32, 2), (a + "vocab_size", U32, 16), (a + "leading_dense_block_count", U32, 0),
        (a + "hyper_connection.count", U32, N), (a + "hyper_connection.sinkhorn_iterations", U32, HC_ITERS),
        (a + "hyper_connection.epsilon", F32, HC_EPS), (a + "attention.layer_norm_rms_epsilon", F32, HC_RMS_EPS)]
    W = (2 + N) * N
    f32 = lambda a_: np.ascontiguousarray(a_, np.float32).tobytes()
    L = c["layer"]
    tensors = [("blk.0.hc_ffn_fn.weight", [N * H, W], 0, f32(c["fn"])),
               ("blk.0.hc_ffn_base.weight", [W], 0, f32(c["base"])),
               ("blk.0.hc_ffn_scale.weight", [3], 0, f32(c["scale"])),
               ("blk.0.ffn_norm.weight", [H], 0, f32(c["norm_w"]))]
    tensors += moe_block_tensors(0, c["router"], c["corr"], L["gate"], L["up"], L["down"], L["gate_sh"],
                                 L["up_sh"], L["down_sh"], H, I, E)
    write_gguf(path, kvs, tensors)
