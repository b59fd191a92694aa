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
