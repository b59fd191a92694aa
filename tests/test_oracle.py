"""Pins the oracle (CPU restatement) against the reference's own golden data."""
import hashlib
import json
import os
import re
import struct

import numpy as np
import pytest

from oracle import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")
REF_ROOT = oracle.reference_root() or ""
GRID_H = os.path.join(os.path.dirname(__file__), "..", "gpeed_b200", "csrc", "iq3xxs_grid.h")


def _grid_from_header(path, name):
    text = open(path).read()
    if name == "gpeed_iq3xxs_grid":  # values live in a macro shared by host and device copies
        m = re.search(r"#define GPEED_IQ3XXS_GRID_VALUES(.*?)\n\n", text, re.S)
        body = m.group(1).replace("\\", " ")
    else:
        body = re.search(name + r"\s*\[[^\]]*\]\s*=\s*\{(.*?)\};", text, re.S).group(1)
    return [int(t.rstrip("u"), 0) for t in re.split(r"[,\s]+", body) if t]


def test_grid_table_digest():
    grid = _grid_from_header(GRID_H, "gpeed_iq3xxs_grid")
    assert len(grid) == 256
    digest = hashlib.sha256(struct.pack("<256I", *grid)).hexdigest()
    pinned = re.search(r'GPEED_IQ3XXS_GRID_SHA256 "([0-9a-f]+)"', open(GRID_H).read()).group(1)
    assert digest == pinned
    vals = {b for g in grid for b in struct.pack("<I", g)}
    assert vals == {4, 12, 20, 28, 36, 44, 52, 62}


@pytest.mark.skipif(not os.path.exists(os.path.join(REF_ROOT, "cpp")), reason="reference tree not present")
def test_grid_and_signs_match_reference_header():
    hdr = os.path.join(REF_ROOT, "cpp", "core", "include", "glm5", "iq3xxs_tables.h")
    assert _grid_from_header(hdr, "kIq3xxsGrid") == _grid_from_header(GRID_H, "gpeed_iq3xxs_grid")
    signs = _grid_from_header(hdr, "kSignsIq2xs")
    assert signs == [k | ((bin(k).count("1") & 1) << 7) for k in range(128)]
    assert _grid_from_header(hdr, "kMaskIq2xs") == [1 << j for j in range(8)]


def test_selftest_vector(port):
    """tests/gguf_selftest.cpp's IQ3_XXS check (1e-4 relative, :14-18)."""
    d = json.load(open(os.path.join(GOLD, "iq3xxs_selftest.json")))
    blk = np.frombuffer(bytes.fromhex(d["block_hex"]), np.uint8)
    got = port.dequantize(blk)
    want = np.array(d["expected"], np.float64)
    assert np.all(np.abs(got - want) <= 1e-4 * np.maximum(1.0, np.abs(want)))
    # the expected floats were produced in double precision; the fp32 decode
    # is exact here (d = 0.0625 is a power of two)
    assert np.array_equal(got.astype(np.float64), want)


def test_blocks_bit_exact_vs_reference_codec(port):
    z = np.load(os.path.join(GOLD, "iq3xxs_blocks.npz"))
    got = port.dequantize(z["blocks"]).view(np.uint32)
    want = z["decoded_bits"]
    same = (got == want) | (np.isnan(got.view(np.float32)) & np.isnan(want.view(np.float32)))
    assert same.all(), f"{(~same).sum()} mismatching values"


def test_dequantize_rejects_partial_block(port):
    """quant.cpp:523-524 throws when n is not a multiple of 256."""
    blk = np.zeros(98, np.uint8)
    out = np.zeros(256, np.float32)
    rc = port._f("dequantize_iq3xxs")(oracle._p(blk), oracle._p(out), oracle.ctypes.c_uint64(255))
    assert rc != 0


def _tiny_layer():
    z = np.load(os.path.join(GOLD, "moe_tiny.npz"))
    H, I, E, K = int(z["H"]), int(z["I"]), int(z["E"]), int(z["K"])
    seed = int(z["weight_seed"])
    s = [int(v) for v in z["weight_streams"]]
    nb = lambda rows, inn: rows * inn // 256
    layer = dict(
        gate=oracle.synth_iq3xxs(seed, s[0], nb(E * I, H)), up=oracle.synth_iq3xxs(seed, s[1], nb(E * I, H)),
        down=oracle.synth_iq3xxs(seed, s[2], nb(E * H, I)), gate_sh=oracle.synth_iq3xxs(seed, s[3], nb(I, H)),
        up_sh=oracle.synth_iq3xxs(seed, s[4], nb(I, H)), down_sh=oracle.synth_iq3xxs(seed, s[5], nb(H, I)),
        router=z["router"], corr=z["corr"])
    return z, oracle.Shape(H, I, E, K, 2.5, 1, 10.0), layer


def test_moe_tiny_matches_reference_harness(port):
    z, shape, layer = _tiny_layer()
    X = z["X"]
    mv = port.matvec_quant(layer["gate"], int(z["matvec_row0"]), shape.hidden, shape.inter, X[0])
    np.testing.assert_array_equal(mv, z["matvec_y"])
    for t in range(X.shape[0]):
        y, tk, tw = port.moe_forward(shape, layer, X[t])
        np.testing.assert_array_equal(tk, z["fwd_topk"][t])
        np.testing.assert_array_equal(tw, z["fwd_topw"][t])
        np.testing.assert_array_equal(y, z["fwd_y"][t])
    Y, tk, tw = port.moe_batch(shape, layer, X)
    np.testing.assert_array_equal(tk, z["bat_topk"])
    np.testing.assert_array_equal(tw, z["bat_topw"])
    np.testing.assert_array_equal(Y, z["bat_y"])


def test_forced_routing_equals_free_routing(port):
    z, shape, layer = _tiny_layer()
    X = z["X"]
    y0, tk, _ = port.moe_forward(shape, layer, X[1])
    y1, tk1, _ = port.moe_forward(shape, layer, X[1], forced=tk)
    np.testing.assert_array_equal(y0, y1)
    Y0, TK, _ = port.moe_batch(shape, layer, X)
    Y1, _, _ = port.moe_batch(shape, layer, X, forced=TK)
    np.testing.assert_array_equal(Y0, Y1)


def test_synth_generator_distribution():
    b = oracle.synth_iq3xxs(0, 1, 4096).reshape(4096, 98)
    d = b[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    assert d.min() >= 2e-4 * 0.999 and d.max() <= 2e-3 * 1.001
    assert abs(d.mean() - 1.1e-3) < 3e-5
    qs = b[:, 2:66].ravel()
    assert abs(qs.mean() - 127.5) < 1.0
    # block b of a longer run equals the same block generated alone
    np.testing.assert_array_equal(oracle.synth_iq3xxs(0, 1, 1, block0=777), b[777])


@pytest.mark.skipif(not oracle.available("reference"), reason="oracle/_ref not built")
def test_port_equals_compiled_reference_at_full_width():
    """Seeded layer at BASELINE widths (H=5120, I=1536), 4 experts, top-2."""
    port, ref = oracle.Checker("port"), oracle.Checker("reference")
    rng = np.random.default_rng(5)
    H, I, E, K = 5120, 1536, 4, 2
    nb = lambda rows, inn: rows * inn // 256
    layer = dict(gate=oracle.synth_iq3xxs(3, 1, nb(E * I, H)), up=oracle.synth_iq3xxs(3, 2, nb(E * I, H)),
                 down=oracle.synth_iq3xxs(3, 3, nb(E * H, I)), gate_sh=oracle.synth_iq3xxs(3, 4, nb(I, H)),
                 up_sh=oracle.synth_iq3xxs(3, 5, nb(I, H)), down_sh=oracle.synth_iq3xxs(3, 6, nb(H, I)),
                 router=(rng.standard_normal((E, H)) * 0.02).astype(np.float32), corr=np.zeros(E, np.float32))
    shape = oracle.Shape(H, I, E, K, 2.5, 1, 10.0)
    x = rng.standard_normal(H).astype(np.float32)
    a = port.moe_forward(shape, layer, x)
    b = ref.moe_forward(shape, layer, x)
    for u, v in zip(a, b):
        np.testing.assert_array_equal(u, v)
    blocks = oracle.synth_iq3xxs(9, 9, 2000)
    np.testing.assert_array_equal(port.dequantize(blocks).view(np.uint32), ref.dequantize(blocks).view(np.uint32))


@pytest.mark.skipif(not oracle.available("reference"), reason="oracle/_ref not built")
def test_port_equals_compiled_reference_at_the_reference_model_shape():
    """The reference model's default MoE widths (model_config.h:25, 59-60:
    hidden 4096, moe_inter 2048), 8 experts, top-8 (every expert picked, in
    the router's order) and the forced form of the same picks: the port and
    the compiled reference agree bit for bit.  The GPU test at this shape
    compares against the port on the picked experts only."""
    port, ref = oracle.Checker("port"), oracle.Checker("reference")
    rng = np.random.default_rng(6)
    H, I, E, K = 4096, 2048, 8, 8
    nb = lambda rows, inn: rows * inn // 256
    layer = dict(gate=oracle.synth_iq3xxs(4, 1, nb(E * I, H)), up=oracle.synth_iq3xxs(4, 2, nb(E * I, H)),
                 down=oracle.synth_iq3xxs(4, 3, nb(E * H, I)), gate_sh=oracle.synth_iq3xxs(4, 4, nb(I, H)),
                 up_sh=oracle.synth_iq3xxs(4, 5, nb(I, H)), down_sh=oracle.synth_iq3xxs(4, 6, nb(H, I)),
                 router=(rng.standard_normal((E, H)) * 0.02).astype(np.float32), corr=np.zeros(E, np.float32))
    shape = oracle.Shape(H, I, E, K, 2.5, 1, 10.0)
    x = rng.standard_normal(H).astype(np.float32)
    a = port.moe_forward(shape, layer, x)
    b = ref.moe_forward(shape, layer, x)
    for u, v in zip(a, b):
        np.testing.assert_array_equal(u, v)
    forced = np.arange(K, dtype=np.int32)[::-1].copy()
    a = port.moe_forward(shape, layer, x, forced=forced)
    b = ref.moe_forward(shape, layer, x, forced=forced)
    for u, v in zip(a, b):
        np.testing.assert_array_equal(u, v)
