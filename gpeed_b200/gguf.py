"""GGUF model files on the C ABI: the reference's ``glm5::GgufModel`` reader
(cpp/core/include/glm5/gguf.h:70-150, cpp/core/src/gguf.cpp) and the MoE
layer loader that feeds expert tensors from the file mapping to the device.

* ``GgufModel(path)``       - ``GgufModel::load(discover_shards(path))``
  (gguf.cpp:255-326): every "<stem>-NNNNN-of-MMMMM.gguf" shard, mapped
  read-only.
* ``find`` / ``get``        - ``GgufModel::find`` / ``GgufFile::get`` (scalars,
  strings and numeric arrays as Python values).
* ``find_tensor``           - ``GgufModel::find_tensor`` -> ``TensorInfo``.
* ``read``                  - ``GgufFile::read_at`` inside one tensor.
* ``moe_config(blk)``       - the MoE fields of ``ModelConfig::from_gguf``
  (model_config.cpp:80-95) for block ``blk``.
* ``MoeLayer.from_gguf``    - block ``blk``'s router, bias and expert tensors
  (model.cpp:702-754) as a device-resident layer (an expert range for expert
  parallelism).

Errors raise ``GpeedError`` like the reference's ``std::runtime_error``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _capi
from ._capi import GgufTensor, GpeedError, MoeShape, call
from .moe import Context, MoeConfig, MoeLayer

ARRAY, STRING = 9, 8


@dataclass(frozen=True)
class TensorInfo:
    """glm5::TensorInfo (gguf.h:61-70): dims in ggml ne order."""
    name: str
    dims: tuple[int, ...]
    type: int
    offset: int
    nbytes: int
    shard: int

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n


class GgufModel:
    def __init__(self, path: str):
        h = ctypes.c_void_p()
        call("gpeed_gguf_open", path.encode(), ctypes.byref(h))
        self.handle = h
        ns, nt, nk = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
        call("gpeed_gguf_counts", h, ctypes.byref(ns), ctypes.byref(nt), ctypes.byref(nk))
        self.n_shards = ns.value
        name = ctypes.c_char_p()
        self._names = []
        for i in range(nt.value):
            call("gpeed_gguf_tensor_name", h, i, ctypes.byref(name))
            self._names.append(name.value.decode())
        self._name_set = set(self._names)
        self._keys = []
        for i in range(nk.value):
            call("gpeed_gguf_key_name", h, i, ctypes.byref(name))
            self._keys.append(name.value.decode())
        self._key_set = set(self._keys)

    def tensor_names(self) -> list[str]:
        return list(self._names)

    def keys(self) -> list[str]:
        return list(self._keys)

    def find_tensor(self, name: str) -> TensorInfo | None:
        if name not in self._name_set:
            return None
        t = GgufTensor()
        call("gpeed_gguf_tensor_info", self.handle, name.encode(), ctypes.byref(t))
        return TensorInfo(name, tuple(int(d) for d in t.dims[:t.n_dims]), t.dtype, int(t.offset), int(t.nbytes),
                          t.shard)

    def read(self, name: str, offset: int = 0, nbytes: int | None = None) -> np.ndarray:
        """Raw bytes [offset, offset + nbytes) of tensor `name` (default: the whole payload)."""
        if nbytes is None:
            t = self.find_tensor(name)
            if t is None:
                raise GpeedError(_capi.ERR_INVALID, f"weights: missing tensor {name}")
            nbytes = t.nbytes - offset
        out = np.empty(nbytes, np.uint8)
        call("gpeed_gguf_read", self.handle, name.encode(), ctypes.c_uint64(offset), ctypes.c_uint64(nbytes),
             out.ctypes.data_as(ctypes.c_void_p))
        return out

    def find(self, key: str):
        """Metadata value (int / float / bool-as-int / str / list of numbers), None if absent."""
        if key not in self._key_set:
            return None
        t, et, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_uint64()
        call("gpeed_gguf_meta_type", self.handle, key.encode(), ctypes.byref(t), ctypes.byref(et), ctypes.byref(n))
        if t.value == STRING:
            s = ctypes.c_char_p()
            call("gpeed_gguf_meta_str", self.handle, key.encode(), ctypes.byref(s))
            return s.value.decode()
        if t.value == ARRAY:
            if et.value in (STRING, ARRAY):
                raise GpeedError(_capi.ERR_UNSUPPORTED, f"{key}: arrays of strings or arrays are not exposed")
            d = ctypes.c_double()
            vals = []
            for i in range(n.value):
                call("gpeed_gguf_meta_f64", self.handle, key.encode(), ctypes.c_uint64(i), ctypes.byref(d))
                vals.append(int(d.value) if et.value not in (6, 12) else d.value)
            return vals
        if t.value in (6, 12):
            d = ctypes.c_double()
            call("gpeed_gguf_meta_f64", self.handle, key.encode(), ctypes.c_uint64(0), ctypes.byref(d))
            return d.value
        u = ctypes.c_uint64()
        call("gpeed_gguf_meta_u64", self.handle, key.encode(), ctypes.byref(u))
        v = u.value
        if t.value in (1, 3, 5, 11) and v >= 1 << 63:  # signed
            v -= 1 << 64
        return v

    def get(self, key: str):
        v = self.find(key)
        if v is None:
            raise GpeedError(_capi.ERR_INVALID, f"GGUF: missing metadata key {key}")
        return v

    def moe_config(self, blk: int) -> MoeConfig:
        s = MoeShape()
        call("gpeed_gguf_moe_shape", self.handle, blk, ctypes.byref(s))
        return _config(s)

    def close(self) -> None:
        if self.handle:
            call("gpeed_gguf_close", self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _config(s: MoeShape) -> MoeConfig:
    return MoeConfig(hidden=s.hidden, inter=s.inter, n_experts=s.n_experts, top_k=s.top_k, n_shared=s.n_shared,
                     routed_scale=s.routed_scale, norm_topk=bool(s.norm_topk), swiglu_limit=s.swiglu_limit)


def load_moe_layer(ctx: Context, model: GgufModel, blk: int, layer_id: int | None = None, expert_begin: int = 0,
                   expert_count: int | None = None) -> MoeLayer:
    """Block `blk`'s MoE tensors as a device layer; routed experts
    [expert_begin, expert_begin + expert_count) (default: all) plus the shared expert."""
    cfg = model.moe_config(blk)
    layer = MoeLayer(ctx, cfg, layer_id)
    s = MoeShape()
    call("gpeed_moe_load_layer_gguf", ctx.handle, model.handle, blk, layer.layer_id, expert_begin,
         -1 if expert_count is None else expert_count, ctypes.byref(s))
    return layer

