"""ctypes binding of libgpeed_moe.so (include/gpeed_moe.h).

The library is the product: there is no Python or CPU fallback.  Loading
fails loudly when the shared object is missing.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libgpeed_moe.so")

OK, ERR_INVALID, ERR_CUDA, ERR_DEVICE, ERR_UNSUPPORTED, ERR_NCCL = range(6)
DTYPE_F32, DTYPE_IQ3_XXS, DTYPE_BF16 = 0, 18, 30
OPT_FUSED_DECODE = 1
OPT_FUSED_COOPERATIVE = 2
OPT_TC_MIN_TOKENS = 3
TC_MIN_TOKENS_DEFAULT = 8  # the library's default for OPT_TC_MIN_TOKENS
OPT_FUSED_MAX_TOKENS = 4
FUSED_MAX_TOKENS_DEFAULT = 12
OPT_SPIN_LIMIT = 5
SPIN_LIMIT_DEFAULT = 1 << 22
OPT_TEST_WITHHOLD_LOGIT = 6
IPC_HANDLE_BYTES = 64  # GPEED_IPC_HANDLE_BYTES
TC_SLOT_TOKENS = 224  # rows per expert slot of the tensor-core path (tc_moe.cu, the MMA's N)


class GpeedError(RuntimeError):
    """Raised for a non-zero status; mirrors the reference's std::runtime_error."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"gpeed error {code}: {msg}")
        self.code = code


class MoeShape(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("inter", ctypes.c_int), ("n_experts", ctypes.c_int),
                ("top_k", ctypes.c_int), ("n_shared", ctypes.c_int), ("routed_scale", ctypes.c_float),
                ("norm_topk", ctypes.c_int), ("swiglu_limit", ctypes.c_float)]


class MhcParams(ctypes.Structure):
    _fields_ = [("hc_mult", ctypes.c_int), ("sinkhorn_iters", ctypes.c_int), ("hc_eps", ctypes.c_float),
                ("rms_eps", ctypes.c_float)]


class GgufTensor(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int), ("n_dims", ctypes.c_int), ("dims", ctypes.c_uint64 * 4),
                ("offset", ctypes.c_uint64), ("nbytes", ctypes.c_uint64), ("shard", ctypes.c_int)]


_vp, _i, _u64, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_float
_i64, _cs = ctypes.c_int64, ctypes.c_char_p
# name -> argtypes (every function returns int status unless listed in _RESTYPES)
SIGNATURES = {
    "gpeed_last_error": [],
    "gpeed_version": [],
    "gpeed_ctx_create": [_i, ctypes.POINTER(_vp)],
    "gpeed_ctx_destroy": [_vp],
    "gpeed_ctx_check": [_vp, _vp],
    "gpeed_ctx_set_option": [_vp, _i, _i],
    "gpeed_ctx_profile": [_vp, _i],
    "gpeed_ctx_profile_read": [_vp, _vp, ctypes.POINTER(_i)],
    "gpeed_iq3xxs_dequantize": [_vp, _vp, _u64, _vp],
    "gpeed_dequantize": [_i, _vp, _vp, _u64, _vp],
    "gpeed_tensor_upload": [_vp, _vp, _i, _i, _u64, _i, ctypes.POINTER(_i)],
    "gpeed_tensor_download": [_vp, _i, _vp],
    "gpeed_matvec_quant": [_vp, _i, _u64, _i, _i, _vp, _vp, _vp],
    "gpeed_matmul_quant": [_vp, _i, _u64, _i, _i, _vp, _i, _vp, _vp],
    "gpeed_matmul_quant_noalloc": [_vp, _i, _u64, _i, _i, _vp, _i, _vp, _vp],
    "gpeed_matvec_quant_host": [_vp, _i, _u64, _i, _i, _vp, _vp],
    "gpeed_matmul_quant_host": [_vp, _i, _u64, _i, _i, _vp, _i, _vp],
    "gpeed_moe_load_layer": [_vp, _i, ctypes.POINTER(MoeShape), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i],
    "gpeed_moe_synth_layer": [_vp, _i, ctypes.POINTER(MoeShape), _vp, _vp, _i, _u64, _u64],
    "gpeed_synth_iq3xxs": [_vp, _u64, _u64, _u64, _u64, _vp],
    "gpeed_moe_forward": [_vp, _i, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp],
    "gpeed_moe_forward_host": [_vp, _i, _vp, _i, _i, _vp],
    "gpeed_moe_load_layer_range": [_vp, _i, ctypes.POINTER(MoeShape), _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                   _vp, _i],
    "gpeed_moe_synth_layer_range": [_vp, _i, ctypes.POINTER(MoeShape), _i, _i, _vp, _vp, _i, _u64, _u64],
    "gpeed_moe_route": [_vp, _i, _vp, _i, _i, _vp, _vp, _vp, _vp],
    "gpeed_moe_decode_partial": [_vp, _i, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp],
    "gpeed_ep_setup": [_vp, _i, _i, _i, _vp],
    "gpeed_ep_connect": [_vp, _vp],
    "gpeed_moe_decode_ep": [_vp, _i, _vp, _i, _vp, _vp, _vp, _vp],
    "gpeed_moe_slice_units": [_vp, _i, _i, _i],
    "gpeed_ep_disconnect": [_vp],
    "gpeed_ep_pack": [_vp, _i, _i, _i, _i, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp],
    "gpeed_moe_experts": [_vp, _i, _vp, _i, _i, _vp, _vp, _vp],
    "gpeed_moe_combine": [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp],
    "gpeed_dense_mlp_forward": [_vp, _i, _i, _i, _f, _vp, _i, _i, _vp, _vp],
    "gpeed_mhc_pre": [_vp, _vp, _i, _i, ctypes.POINTER(MhcParams), _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp],
    "gpeed_mhc_post": [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp],
    "gpeed_gguf_open": [_cs, ctypes.POINTER(_vp)],
    "gpeed_gguf_close": [_vp],
    "gpeed_gguf_counts": [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i64), ctypes.POINTER(_i64)],
    "gpeed_gguf_tensor_name": [_vp, _i64, ctypes.POINTER(_cs)],
    "gpeed_gguf_key_name": [_vp, _i64, ctypes.POINTER(_cs)],
    "gpeed_gguf_tensor_info": [_vp, _cs, ctypes.POINTER(GgufTensor)],
    "gpeed_gguf_read": [_vp, _cs, _u64, _u64, _vp],
    "gpeed_gguf_meta_type": [_vp, _cs, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_u64)],
    "gpeed_gguf_meta_f64": [_vp, _cs, _u64, ctypes.POINTER(ctypes.c_double)],
    "gpeed_gguf_meta_u64": [_vp, _cs, ctypes.POINTER(_u64)],
    "gpeed_gguf_meta_str": [_vp, _cs, ctypes.POINTER(_cs)],
    "gpeed_gguf_moe_shape": [_vp, _i, ctypes.POINTER(MoeShape)],
    "gpeed_moe_load_layer_gguf": [_vp, _vp, _i, _i, _i, _i, ctypes.POINTER(MoeShape)],
    "gpeed_tensor_upload_gguf": [_vp, _vp, _cs, ctypes.POINTER(_i)],
}
_RESTYPES = {"gpeed_last_error": ctypes.c_char_p}

_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
                "(or `make -C gpeed_b200/csrc`); there is no CPU fallback")
        lib = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = lib
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        msg = load().gpeed_last_error()
        raise GpeedError(rc, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
