"""ctypes front end for the checkers (TEST INFRASTRUCTURE ONLY).

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg.  ``load("port")`` is the C restatement (oracle/liboracle.so);
``load("reference")`` is the reference's own compiled codec plus harness
(oracle/_ref/libgpeed_ref.so), present when it was built from the reference
sources.  Both expose the same functions, wrapped here for numpy arrays.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libgpeed_ref.so")


class Shape(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("inter", ctypes.c_int), ("n_experts", ctypes.c_int),
                ("top_k", ctypes.c_int), ("routed_scale", ctypes.c_float), ("norm_topk", ctypes.c_int),
                ("swiglu_limit", ctypes.c_float)]


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def reference_root() -> str | None:
    """The reference project's source tree, or None when it is not on this
    machine (it never is on a GPU box).  Taken from GPEED_REFERENCE_ROOT, else
    from the `reference_path` BASELINE.json records for this build."""
    root = os.environ.get("GPEED_REFERENCE_ROOT")
    if not root:
        try:
            with open(os.path.join(HERE, "..", "BASELINE.json")) as fh:
                root = json.load(fh).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root if root and os.path.isdir(os.path.join(root, "cpp")) else None


def build() -> None:
    """Compiles liboracle.so (and oracle/_ref when the reference tree exists)."""
    ref = reference_root()
    subprocess.run(["make", "-s", "-C", HERE] + ([f"REF={ref}"] if ref else []), check=True)


def available(kind: str) -> bool:
    return os.path.exists(PORT_SO if kind == "port" else REF_SO)


class Checker:
    def __init__(self, kind: str = "port"):
        path = PORT_SO if kind == "port" else REF_SO
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run `make -C oracle`)")
        self.kind = kind
        self.lib = ctypes.CDLL(path)
        self.pre = "orc_" if kind == "port" else "ref_"
        f = self._f
        f("dot_f32").restype = ctypes.c_float
        for name in ("dequantize_iq3xxs", "matvec_quant", "matmul_quant", "moe_forward", "moe_batch",
                     "num_threads"):
            f(name).restype = ctypes.c_int

    def _f(self, name):
        return getattr(self.lib, self.pre + name)

    def num_threads(self) -> int:
        return self._f("num_threads")()

    def set_num_threads(self, n: int) -> None:
        """OpenMP threads of the checker's loops from now on."""
        self._f("set_num_threads")(int(n))

    def dequantize(self, blocks: np.ndarray) -> np.ndarray:
        blocks = np.ascontiguousarray(blocks, np.uint8).reshape(-1)
        n = blocks.size // 98 * 256
        out = np.empty(n, np.float32)
        rc = self._f("dequantize_iq3xxs")(_p(blocks), _p(out), ctypes.c_uint64(n))
        if rc:
            raise ValueError("dequantize failed")
        return out

    def dequantize_type(self, dtype: int, raw: np.ndarray, n: int) -> np.ndarray:
        """Any codec the reference decodes (ggml type id), n values."""
        raw = np.ascontiguousarray(raw, np.uint8).reshape(-1)
        out = np.empty(n, np.float32)
        fn = self._f("dequantize")
        fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64]
        rc = fn(dtype, _p(raw), _p(out), ctypes.c_uint64(n))
        if rc:
            raise ValueError(f"dequantize of type {dtype} failed ({rc})")
        return out

    def mhc_pre(self, streams, fn, base, scale, norm_w, N=4, iters=20, hc_eps=1e-6, rms_eps=1e-5):
        """model.cpp:205-263 + the ffn RMSNorm: streams [n][N][H] -> (x [n][H], post [n][N], comb [n][N][N])."""
        streams = np.ascontiguousarray(streams, np.float32)
        n, H = streams.shape[0], streams.shape[-1]
        x = np.empty((n, H), np.float32)
        post = np.empty((n, N), np.float32)
        comb = np.empty((n, N, N), np.float32)
        fn_, base_, scale_, w_ = (np.ascontiguousarray(a, np.float32) for a in (fn, base, scale, norm_w))
        f = self._f("mhc_pre")
        f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                      ctypes.c_float] + [ctypes.c_void_p] * 7
        if f(_p(streams), n, N, H, iters, hc_eps, rms_eps, _p(fn_), _p(base_), _p(scale_), _p(w_), _p(x), _p(post),
             _p(comb)):
            raise ValueError("mhc_pre failed")
        return x, post, comb

    def mhc_post(self, streams_in, mlp, post, comb):
        streams_in = np.ascontiguousarray(streams_in, np.float32)
        n, N, H = streams_in.shape
        out = np.empty_like(streams_in)
        args = [np.ascontiguousarray(a, np.float32) for a in (mlp, post, comb)]
        f = self._f("mhc_post")
        f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
        f(_p(streams_in), _p(args[0]), _p(args[1]), _p(args[2]), n, N, H, _p(out))
        return out

    def matvec_quant(self, w, row0, in_dim, out_dim, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(out_dim, np.float32)
        rc = self._f("matvec_quant")(_p(w), ctypes.c_uint64(row0), in_dim, out_dim, _p(x), _p(y))
        if rc:
            raise ValueError("matvec_quant failed")
        return y

    def matmul_quant(self, w, row0, in_dim, out_dim, X):
        X = np.ascontiguousarray(X, np.float32)
        n = X.shape[0]
        Y = np.empty((n, out_dim), np.float32)
        rc = self._f("matmul_quant")(_p(w), ctypes.c_uint64(row0), in_dim, out_dim, _p(X), n, _p(Y))
        if rc:
            raise ValueError("matmul_quant failed")
        return Y

    def moe_forward(self, shape: Shape, layer: dict, x, forced=None):
        """One token through Model::moe_forward; returns (y, topk ids, weights)."""
        K = shape.top_k
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(shape.hidden, np.float32)
        tk = np.empty(K, np.int32)
        tw = np.empty(K, np.float32)
        fc = None if forced is None else np.ascontiguousarray(forced, np.int32)
        rc = self._f("moe_forward")(ctypes.byref(shape), _p(layer["router"]), _p(layer.get("corr")),
                                    _p(layer["gate"]), _p(layer["up"]), _p(layer["down"]),
                                    _p(layer.get("gate_sh")), _p(layer.get("up_sh")), _p(layer.get("down_sh")),
                                    _p(x), _p(y), _p(fc), _p(tk), _p(tw))
        if rc:
            raise ValueError("moe_forward failed")
        return y, tk, tw

    def moe_batch(self, shape: Shape, layer: dict, X, forced=None):
        """n tokens through Model::moe_batch; returns (Y, topk ids [n,K], weights [n,K])."""
        X = np.ascontiguousarray(X, np.float32)
        n, K = X.shape[0], shape.top_k
        Y = np.empty((n, shape.hidden), np.float32)
        tk = np.empty((n, K), np.int32)
        tw = np.empty((n, K), np.float32)
        fc = None if forced is None else np.ascontiguousarray(forced, np.int32)
        rc = self._f("moe_batch")(ctypes.byref(shape), _p(layer["router"]), _p(layer.get("corr")),
                                  _p(layer["gate"]), _p(layer["up"]), _p(layer["down"]),
                                  _p(layer.get("gate_sh")), _p(layer.get("up_sh")), _p(layer.get("down_sh")),
                                  _p(X), n, _p(Y), _p(fc), _p(tk), _p(tw))
        if rc:
            raise ValueError("moe_batch failed")
        return Y, tk, tw


def synth_iq3xxs(seed: int, stream: int, nblocks: int, block0: int = 0) -> np.ndarray:
    """Host twin of the device generator: nblocks IQ3_XXS blocks as uint8[nblocks*98]."""
    lib = ctypes.CDLL(PORT_SO)
    out = np.empty(nblocks * 98, np.uint8)
    lib.orc_synth_iq3xxs(ctypes.c_uint64(seed), ctypes.c_uint64(stream), ctypes.c_uint64(block0),
                         ctypes.c_uint64(nblocks), _p(out))
    return out
