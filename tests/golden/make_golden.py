"""Regenerates the golden fixtures in this folder from the reference itself.

Run where the reference tree and the compiled reference codec exist
(``make -C oracle`` builds oracle/_ref/libgpeed_ref.so from the reference's
cpp/core/src/quant.cpp):

    python tests/golden/make_golden.py --ref <reference root>

Fixtures written (all small, committed):

* iq3xxs_selftest.json   the reference's own IQ3_XXS known-answer vector: the
  block and expected floats that python/tools/make_test_gguf.py (seed 1234,
  d = 0.0625) writes and tests/gguf_selftest.cpp checks at 1e-4 relative.
  Produced by running that script unmodified and reading the block back with
  the reference's python/reference/gguf_reader.py.
* iq3xxs_blocks.npz      seeded random blocks plus hand-picked edge blocks
  (zero, negative, subnormal and largest-normal fp16 scales; all-zero and
  all-one scale/sign words) and their decode by the reference's compiled
  dequantize() - bit patterns, for bit-exact comparison.
* ref_selftest.gguf      the GGUF file that script writes (5 tensors: F32, F16,
  BF16, Q8_0, IQ3_XXS; 7 metadata keys), and
  ref_selftest_gguf.json what the reference's python/reference/gguf_reader.py
  reads from it (version, data offset, metadata, tensor table in file order).
  ``--only gguf`` rewrites just these two.
* codec_blocks.npz       for every codec the reference decodes (F16, BF16,
  Q8_0, Q2_K, Q3_K, Q6_K, IQ3_XXS, IQ3_S, IQ2_S, IQ4_XS): 12 seeded and 24
  edge blocks with the reference's compiled decode (bit patterns), and
  codec_digests.json     the SHA-256 of its decode of 4096 seeded blocks per
  type (2^20 values for F16/BF16); ``--only codecs``.
* moe_tiny.npz           a tiny MoE layer (H=512, I=512, E=8, K=2, 1 shared
  expert; expert bytes from the counter-based generator, seed 7, streams
  gate..down_sh = 1..6) run through the reference harness: matvec_quant outputs, the
  single-token moe_forward path and the batched moe_batch path (top-k ids,
  weights, outputs).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, REPO)
from oracle import oracle  # noqa: E402  (the repo root is not a package path when run as a script)


class Shape(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("inter", ctypes.c_int), ("n_experts", ctypes.c_int),
                ("top_k", ctypes.c_int), ("routed_scale", ctypes.c_float), ("norm_topk", ctypes.c_int),
                ("swiglu_limit", ctypes.c_float)]


def ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def selftest_vector(ref_root: str) -> dict:
    with tempfile.TemporaryDirectory() as tmp:
        subprocess.run([sys.executable, os.path.join(ref_root, "python", "tools", "make_test_gguf.py"),
                        "--out", tmp], check=True, capture_output=True)
        sys.path.insert(0, os.path.join(ref_root, "python", "reference"))
        from gguf_reader import GgufReader  # the reference's reader

        r = GgufReader.open(os.path.join(tmp, "test.gguf"))
        raw = r.read_tensor("test.iq3_xxs", 98) if hasattr(r, "read_tensor") else None
        expected = None
        with open(os.path.join(tmp, "test.expected.txt")) as fh:
            lines = fh.read().splitlines()
        for i, name in enumerate(lines):
            if name == "test.iq3_xxs":
                expected = [float(v) for v in lines[i + 1].split()]
        assert raw is not None and len(raw) == 98 and expected is not None and len(expected) == 256
    return {
        "source": "reference python/tools/make_test_gguf.py (seed 1234, d=0.0625), "
                  "checked by tests/gguf_selftest.cpp at 1e-4 relative",
        "block_hex": bytes(raw).hex(),
        "expected": expected,
    }


def selftest_gguf(ref_root: str) -> None:
    import shutil
    with tempfile.TemporaryDirectory() as tmp:
        subprocess.run([sys.executable, os.path.join(ref_root, "python", "tools", "make_test_gguf.py"),
                        "--out", tmp], check=True, capture_output=True)
        sys.path.insert(0, os.path.join(ref_root, "python", "reference"))
        from gguf_reader import GgufReader  # the reference's reader

        path = os.path.join(tmp, "test.gguf")
        r = GgufReader.open(path)
        table = {
            "source": "reference python/tools/make_test_gguf.py (seed 1234), read by "
                      "python/reference/gguf_reader.py",
            "version": r.version,
            "data_offset": r.data_offset,
            "metadata": r.metadata,
            "tensors": [{"name": n, "dims": list(r.tensors[n].dims), "type": r.tensors[n].ggml_type,
                         "offset": r.tensors[n].offset} for n in r.tensor_order],
        }
        r._fh.close()
        shutil.copyfile(path, os.path.join(HERE, "ref_selftest.gguf"))
    with open(os.path.join(HERE, "ref_selftest_gguf.json"), "w") as fh:
        json.dump(table, fh, indent=1)


def codec_fixture(ref) -> None:
    """Every codec the reference decodes: seeded + edge blocks and the
    reference's compiled decode of them (bit patterns), plus the SHA-256 of its
    decode of a larger seeded set that tests regenerate (tests.helpers)."""
    import hashlib
    sys.path.insert(0, REPO)
    from tests.helpers import CODECS, codec_blocks, codec_edge_blocks
    arrays, digests = {}, {}
    for t, (bb, vals, _) in CODECS.items():
        small = np.concatenate([codec_blocks(t, 12, 500 + t), codec_edge_blocks(t)])
        n = small.size // bb * vals
        out = np.zeros(n, np.float32)
        assert ref.ref_dequantize(t, ptr(small), ptr(out), ctypes.c_uint64(n)) == 0
        arrays[f"blocks_{t}"] = small
        arrays[f"bits_{t}"] = out.view(np.uint32)
        big = codec_blocks(t, 4096 if vals > 1 else 1 << 20, 900 + t)
        n = big.size // bb * vals
        out = np.zeros(n, np.float32)
        assert ref.ref_dequantize(t, ptr(big), ptr(out), ctypes.c_uint64(n)) == 0
        digests[str(t)] = hashlib.sha256(out.tobytes()).hexdigest()
    np.savez_compressed(os.path.join(HERE, "codec_blocks.npz"), **arrays)
    with open(os.path.join(HERE, "codec_digests.json"), "w") as fh:
        json.dump({"source": "reference cpp/core/src/quant.cpp dequantize (compiled), blocks from "
                             "tests.helpers.codec_blocks(type, 4096 blocks or 2^20 halves, seed 900 + type)",
                   "sha256": digests}, fh, indent=1)


def edge_blocks(rng: np.random.Generator) -> np.ndarray:
    blocks = []
    for dbits in (0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0xFBFF, 0x2C00, 0xAC00):
        for aux_fill in (None, 0x00000000, 0xFFFFFFFF, 0x8FFFFFFF, 0x7FFFFFFF):
            b = np.frombuffer(rng.bytes(98), np.uint8).copy()
            b[0] = dbits & 0xFF
            b[1] = dbits >> 8
            if aux_fill is not None:
                b[66:98] = np.frombuffer(np.full(8, aux_fill, np.uint32).tobytes(), np.uint8)
            blocks.append(b)
    b = np.frombuffer(rng.bytes(98), np.uint8).copy()
    b[2:66] = np.arange(64, dtype=np.uint8) * 4 + 3   # spread of grid indices incl. 255
    blocks.append(b)
    return np.stack(blocks)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="reference source tree (default: GPEED_REFERENCE_ROOT, else "
                    "BASELINE.json's reference_path)")
    ap.add_argument("--only", choices=["gguf", "codecs"], default=None)
    args = ap.parse_args()
    args.ref = args.ref or oracle.reference_root()
    if not args.ref:
        ap.error("the reference source tree is required: pass --ref or set GPEED_REFERENCE_ROOT")
    ref = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libgpeed_ref.so"))
    if args.only in (None, "gguf"):
        selftest_gguf(args.ref)
    if args.only in (None, "codecs"):
        codec_fixture(ref)
    if args.only:
        return 0
    rng = np.random.default_rng(20240601)

    with open(os.path.join(HERE, "iq3xxs_selftest.json"), "w") as fh:
        json.dump(selftest_vector(args.ref), fh, indent=1)

    # random + edge blocks decoded by the reference's compiled codec
    rnd = np.frombuffer(rng.bytes(98 * 48), np.uint8).reshape(48, 98).copy()
    rnd[:, 0:2] = np.frombuffer(
        (2e-4 + 1.8e-3 * rng.random(48)).astype(np.float16).tobytes(), np.uint8).reshape(48, 2)
    blocks = np.concatenate([rnd, edge_blocks(rng)])
    out = np.zeros(blocks.shape[0] * 256, np.float32)
    assert ref.ref_dequantize_iq3xxs(ptr(blocks), ptr(out), ctypes.c_uint64(out.size)) == 0
    np.savez_compressed(os.path.join(HERE, "iq3xxs_blocks.npz"), blocks=blocks,
                        decoded_bits=out.view(np.uint32))

    # tiny MoE layer through the reference harness
    H, I, E, K, N = 512, 512, 8, 2, 3

    # expert weights come from the counter-based generator (seed 7, streams
    # 1..6), so the fixture stores only the seed; tests regenerate the bytes.
    orc = ctypes.CDLL(os.path.join(REPO, "oracle", "liboracle.so"))

    def mat(stream, rows, inn):
        nb = rows * inn // 256
        b = np.zeros(nb * 98, np.uint8)
        orc.orc_synth_iq3xxs(ctypes.c_uint64(7), ctypes.c_uint64(stream), ctypes.c_uint64(0),
                             ctypes.c_uint64(nb), ptr(b))
        return b

    gate, up, down = mat(1, E * I, H), mat(2, E * I, H), mat(3, E * H, I)
    gsh, ush, dsh = mat(4, I, H), mat(5, I, H), mat(6, H, I)
    router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    corr = (rng.standard_normal(E) * 0.01).astype(np.float32)
    X = rng.standard_normal((N, H)).astype(np.float32)
    shape = Shape(H, I, E, K, 2.5, 1, 10.0)
    fwd_y = np.zeros((N, H), np.float32)
    fwd_k = np.zeros((N, K), np.int32)
    fwd_w = np.zeros((N, K), np.float32)
    for t in range(N):
        xt = np.ascontiguousarray(X[t])
        yt = np.zeros(H, np.float32)
        kt = np.zeros(K, np.int32)
        wt = np.zeros(K, np.float32)
        assert ref.ref_moe_forward(ctypes.byref(shape), ptr(router), ptr(corr), ptr(gate), ptr(up), ptr(down),
                                   ptr(gsh), ptr(ush), ptr(dsh), ptr(xt), ptr(yt), None, ptr(kt), ptr(wt)) == 0
        fwd_y[t], fwd_k[t], fwd_w[t] = yt, kt, wt
    bat_y = np.zeros((N, H), np.float32)
    bat_k = np.zeros((N, K), np.int32)
    bat_w = np.zeros((N, K), np.float32)
    assert ref.ref_moe_batch(ctypes.byref(shape), ptr(router), ptr(corr), ptr(gate), ptr(up), ptr(down),
                             ptr(gsh), ptr(ush), ptr(dsh), ptr(X), N, ptr(bat_y), None, ptr(bat_k), ptr(bat_w)) == 0
    mv = np.zeros(I, np.float32)
    assert ref.ref_matvec_quant(ptr(gate), ctypes.c_uint64(3 * I), H, I, ptr(X[0].copy()), ptr(mv)) == 0
    np.savez_compressed(os.path.join(HERE, "moe_tiny.npz"), H=H, I=I, E=E, K=K, weight_seed=7,
                        weight_streams=np.array([1, 2, 3, 4, 5, 6]), router=router, corr=corr, X=X,
                        fwd_y=fwd_y, fwd_topk=fwd_k, fwd_topw=fwd_w, bat_y=bat_y, bat_topk=bat_k,
                        bat_topw=bat_w, matvec_row0=3 * I, matvec_y=mv)
    print("wrote fixtures to", HERE)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
