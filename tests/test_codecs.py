"""The other GGUF codecs (gpeed_b200/csrc/codecs.cu, gpeed_dequantize): F16,
BF16, Q8_0, Q2_K, Q3_K, Q6_K, IQ2_S, IQ3_S, IQ4_XS (and IQ3_XXS through the
same entry point), bit-exact with the reference's compiled decoder.

CPU: the codebook header against its pinned digests and the reference's table
header; the C oracle (oracle.c) against the golden blocks decoded by the
reference (tests/golden/codec_blocks.npz) and against the digest of the
reference's decode of a larger seeded set (codec_digests.json); argument
errors.  GPU: the same two checks for the CUDA kernels.  NaN values compare
as NaN: the reference keeps a NaN scale's payload through its products, CUDA
arithmetic returns the canonical NaN.
"""
import ctypes
import hashlib
import json
import os
import re
import struct

import numpy as np
import pytest

from gpeed_b200 import _capi
from oracle import oracle
from tests.helpers import CODEC_NAMES, CODECS, codec_blocks

GOLD = os.path.join(os.path.dirname(__file__), "golden")
GRIDS_H = os.path.join(os.path.dirname(__file__), "..", "gpeed_b200", "csrc", "quant_grids.h")
TYPES = sorted(CODECS)


def _macro(text, name):
    m = re.search(r"#define " + name + r" \\\n(.*?)(?:\n\n|\Z)", text, re.S)
    return [int(v, 0) for v in m.group(1).replace("\\", " ").replace("ull", "").replace("u", "").split(",")
            if v.strip()]


def _same(got_bits, want_bits):
    got, want = np.asarray(got_bits, np.uint32), np.asarray(want_bits, np.uint32)
    gnan = (got & 0x7F800000) == 0x7F800000
    gnan &= (got & 0x7FFFFF) != 0
    wnan = ((want & 0x7F800000) == 0x7F800000) & ((want & 0x7FFFFF) != 0)
    return bool(np.array_equal(gnan, wnan) and np.array_equal(got[~gnan], want[~wnan]))


def test_codebooks_are_pinned():
    text = open(GRIDS_H).read()
    g2, g3, v4 = _macro(text, "GPEED_IQ2S_GRID_VALUES"), _macro(text, "GPEED_IQ3S_GRID_VALUES"), \
        _macro(text, "GPEED_IQ4NL_VALUES")
    assert len(g2) == 1024 and len(g3) == 512 and len(v4) == 16
    pins = dict(re.findall(r'#define (GPEED_\w+_SHA256) "([0-9a-f]+)"', text))
    assert hashlib.sha256(struct.pack("<1024Q", *g2)).hexdigest() == pins["GPEED_IQ2S_GRID_SHA256"]
    assert hashlib.sha256(struct.pack("<512I", *g3)).hexdigest() == pins["GPEED_IQ3S_GRID_SHA256"]
    assert hashlib.sha256(struct.pack("<16b", *v4)).hexdigest() == pins["GPEED_IQ4NL_VALUES_SHA256"]
    ref = oracle.reference_root()
    hdr = os.path.join(ref or "", "cpp", "core", "include", "glm5", "quant_tables.h")
    if os.path.exists(hdr):
        rt = open(hdr).read()
        for name, mine in (("kIq2sGrid", g2), ("kIq3sGrid", g3), ("kValuesIq4nl", v4)):
            body = re.search(name + r"\s*\[[^\]]*\]\s*=\s*\{(.*?)\};", rt, re.S).group(1)
            assert [int(t, 0) for t in body.split(",") if t.strip()] == mine, name


@pytest.mark.parametrize("dtype", TYPES, ids=[CODEC_NAMES[t] for t in TYPES])
def test_oracle_matches_the_reference_decoder(port, dtype):
    z = np.load(os.path.join(GOLD, "codec_blocks.npz"))
    bb, vals, _ = CODECS[dtype]
    blocks = z[f"blocks_{dtype}"]
    got = port.dequantize_type(dtype, blocks, blocks.size // bb * vals)
    np.testing.assert_array_equal(got.view(np.uint32), z[f"bits_{dtype}"])
    big = codec_blocks(dtype, 4096 if vals > 1 else 1 << 20, 900 + dtype)
    out = port.dequantize_type(dtype, big, big.size // bb * vals)
    want = json.load(open(os.path.join(GOLD, "codec_digests.json")))["sha256"][str(dtype)]
    assert hashlib.sha256(out.tobytes()).hexdigest() == want


def test_argument_errors_need_no_device():
    lib = _capi.load()
    assert lib.gpeed_dequantize(2, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_uint64(32), None) \
        == _capi.ERR_UNSUPPORTED  # Q4_0: the reference does not decode it either
    assert b"not implemented" in lib.gpeed_last_error()
    assert lib.gpeed_dequantize(14, ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_uint64(255), None) \
        == _capi.ERR_INVALID
    assert b"multiple of block size" in lib.gpeed_last_error()
    assert lib.gpeed_dequantize(8, ctypes.c_void_p(16), ctypes.c_void_p(8), ctypes.c_uint64(32), None) \
        == _capi.ERR_INVALID


def _gpu_decode(dtype, raw, n):
    import torch
    src = torch.from_numpy(np.ascontiguousarray(raw, np.uint8)).cuda()
    dst = torch.empty(n, dtype=torch.float32, device="cuda")
    _capi.call("gpeed_dequantize", dtype, ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()),
               ctypes.c_uint64(n), None)
    torch.cuda.synchronize()
    return dst.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", TYPES, ids=[CODEC_NAMES[t] for t in TYPES])
def test_gpu_decoder_matches_the_reference_decoder(dtype):
    z = np.load(os.path.join(GOLD, "codec_blocks.npz"))
    bb, vals, _ = CODECS[dtype]
    blocks = z[f"blocks_{dtype}"]
    got = _gpu_decode(dtype, blocks, blocks.size // bb * vals)
    assert _same(got.view(np.uint32), z[f"bits_{dtype}"])
    big = codec_blocks(dtype, 4096 if vals > 1 else 1 << 20, 900 + dtype)
    out = _gpu_decode(dtype, big, big.size // bb * vals)
    want = json.load(open(os.path.join(GOLD, "codec_digests.json")))["sha256"][str(dtype)]
    assert hashlib.sha256(out.tobytes()).hexdigest() == want


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [8, 10, 11, 14, 21, 22, 23])
def test_gpu_decoder_large_and_ragged_vs_oracle(port, dtype):
    """Many blocks (past the grid-stride wrap) and block counts that leave a warp step partly empty."""
    bb, vals, _ = CODECS[dtype]
    for nb in (1, 7, 148 * 8 * 8 * 3 + 5):
        raw = codec_blocks(dtype, nb, nb + dtype)
        n = nb * vals
        np.testing.assert_array_equal(_gpu_decode(dtype, raw, n).view(np.uint32),
                                      port.dequantize_type(dtype, raw, n).view(np.uint32))
