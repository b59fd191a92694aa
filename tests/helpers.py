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
