"""Host-side mirror of the reference's expert-op interface, on the C ABI.

* ``WeightStore``  - the reference's ``glm5::WeightStore`` expert entry points
  (cpp/core/include/glm5/weights.h:38-48): tensors are registered by name and
  ``matvec_quant`` / ``matmul_quant`` take the same (name, row0, in_dim,
  out_dim, x, dst) arguments, on CUDA tensors.
* ``MoeLayer``     - ``Model::moe_forward`` / ``Model::moe_batch``
  (cpp/core/src/model.cpp:692-756, model_batch.cpp:165-281) for one layer.
* ``dequantize``   - ``glm5::dequantize`` for IQ3_XXS (quant.cpp:521-573).

Errors surface as ``GpeedError`` (a RuntimeError), as the reference throws
std::runtime_error.  torch is used only for device buffers and streams.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _capi
from ._capi import GpeedError, MoeShape, call

BLOCK_BYTES, QK = 98, 256


def _ptr(t) -> ctypes.c_void_p | None:
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data_as(ctypes.c_void_p)
    return ctypes.c_void_p(t.data_ptr())


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _capi.DTYPE_BF16
    if t.dtype == torch.float32:
        return _capi.DTYPE_F32
    raise GpeedError(_capi.ERR_UNSUPPORTED, f"dtype {t.dtype}")


def _stream(stream) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


class Context:
    """One library context per CUDA device (owns uploaded weights and scratch)."""

    def __init__(self, device: int = 0):
        torch.cuda.init()
        self.device = device
        h = ctypes.c_void_p()
        with torch.cuda.device(device):
            call("gpeed_ctx_create", device, ctypes.byref(h))
        self.handle = h

    def set_option(self, option: int, value: int) -> None:
        call("gpeed_ctx_set_option", self.handle, option, value)

    def check(self, stream=None) -> None:
        call("gpeed_ctx_check", self.handle, _stream(stream))

    def close(self) -> None:
        if self.handle:
            call("gpeed_ctx_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dequantize(blocks: torch.Tensor, stream=None) -> torch.Tensor:
    """IQ3_XXS bytes (uint8 CUDA tensor, n*98) -> float32 (n*256), bit-exact."""
    if blocks.numel() % BLOCK_BYTES:
        raise GpeedError(_capi.ERR_INVALID, "byte count not a multiple of the 98-byte block")
    n = blocks.numel() // BLOCK_BYTES * QK
    out = torch.empty(n, dtype=torch.float32, device=blocks.device)
    call("gpeed_iq3xxs_dequantize", _ptr(blocks), _ptr(out), ctypes.c_uint64(n), _stream(stream))
    return out


class WeightStore:
    """Expert tensors by name, like glm5::WeightStore (weights.h:15-76)."""

    def __init__(self, ctx: Context):
        self.ctx = ctx
        self._handles: dict[str, tuple[int, int, int]] = {}

    def add(self, name: str, raw, rows: int, in_dim: int) -> None:
        """Registers an IQ3_XXS tensor of `rows` rows x `in_dim` weights (numpy/CPU or CUDA bytes)."""
        on_dev = isinstance(raw, torch.Tensor) and raw.is_cuda
        if isinstance(raw, torch.Tensor) and not on_dev:
            raw = raw.numpy()
        raw_c = raw.contiguous() if on_dev else np.ascontiguousarray(raw, np.uint8)
        h = ctypes.c_int()
        call("gpeed_tensor_upload", self.ctx.handle, _ptr(raw_c), int(on_dev), _capi.DTYPE_IQ3_XXS,
             ctypes.c_uint64(rows), in_dim, ctypes.byref(h))
        self._handles[name] = (h.value, rows, in_dim)

    def has(self, name: str) -> bool:
        return name in self._handles

    def _h(self, name: str) -> int:
        if name not in self._handles:
            raise GpeedError(_capi.ERR_INVALID, f"weights: missing tensor {name}")
        return self._handles[name][0]

    def raw_bytes(self, name: str) -> np.ndarray:
        h, rows, in_dim = self._handles[name]
        out = np.empty(rows * (in_dim // QK) * BLOCK_BYTES, np.uint8)
        call("gpeed_tensor_download", self.ctx.handle, h, _ptr(out))
        return out

    def matvec_quant(self, name: str, row0: int, in_dim: int, out_dim: int, x: torch.Tensor,
                     dst: torch.Tensor, stream=None) -> None:
        """dst[j] = sum_i W[row0 + j][i] * x[i] (weights.h:38-41)."""
        call("gpeed_matvec_quant", self.ctx.handle, self._h(name), ctypes.c_uint64(row0), in_dim, out_dim,
             _ptr(x), _ptr(dst), _stream(stream))

    def matmul_quant(self, name: str, row0: int, in_dim: int, out_dim: int, X: torch.Tensor, n_tok: int,
                     Y: torch.Tensor, stream=None) -> None:
        """Y[t][j] = sum_i W[row0 + j][i] * X[t][i] (weights.h:43-48)."""
        call("gpeed_matmul_quant", self.ctx.handle, self._h(name), ctypes.c_uint64(row0), in_dim, out_dim,
             _ptr(X), n_tok, _ptr(Y), _stream(stream))

    def dense_mlp(self, gate: str, up: str, down: str, X: torch.Tensor, Y: torch.Tensor | None = None,
                  swiglu_limit: float = 10.0, stream=None) -> torch.Tensor:
        """Y = down(silu(min(gate X, L)) * clamp(up X, -L, L)) for the dense layers
        (Model::dense_mlp / dense_mlp_batch, model.cpp:677-690, model_batch.cpp:145-163)."""
        if X.dim() == 1:
            X = X.unsqueeze(0)
        dt = _capi.DTYPE_BF16 if X.dtype == torch.bfloat16 else _capi.DTYPE_F32
        if Y is None:
            Y = torch.empty(X.shape[0], X.shape[1], dtype=torch.float32, device=X.device)
        call("gpeed_dense_mlp_forward", self.ctx.handle, self._h(gate), self._h(up), self._h(down),
             ctypes.c_float(swiglu_limit), _ptr(X.contiguous()), dt, X.shape[0], _ptr(Y), _stream(stream))
        return Y


@dataclass
class MoeConfig:
    """MoE fields of glm5::ModelConfig (model_config.h:57-70) at BASELINE sizes."""
    hidden: int = 5120
    inter: int = 1536
    n_experts: int = 160
    top_k: int = 8
    n_shared: int = 1
    routed_scale: float = 2.5
    norm_topk: bool = True
    swiglu_limit: float = 10.0

    def shape(self) -> MoeShape:
        return MoeShape(self.hidden, self.inter, self.n_experts, self.top_k, self.n_shared, self.routed_scale,
                        int(self.norm_topk), self.swiglu_limit)


@dataclass
class MhcParams:
    """mHC constants of glm5::ModelConfig (model_config.h:47-49, 68)."""
    hc_mult: int = 4
    sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    rms_eps: float = 1e-5


def mhc_pre(ctx: Context, streams: torch.Tensor, fn: torch.Tensor, base: torch.Tensor, scale: torch.Tensor,
            norm_w: torch.Tensor, params: MhcParams = MhcParams(), x_dtype=torch.bfloat16, stream=None):
    """Model::hc_forward + the ffn RMSNorm (model.cpp:205-263, 292-296) for n tokens:
    streams [n, N, H] fp32 -> (x [n, H] (the MoE input), post [n, N], comb [n, N, N])."""
    n, N, H = streams.shape
    x = torch.empty(n, H, dtype=x_dtype, device=streams.device)
    post = torch.empty(n, N, dtype=torch.float32, device=streams.device)
    comb = torch.empty(n, N, N, dtype=torch.float32, device=streams.device)
    p = _capi.MhcParams(N, params.sinkhorn_iters, params.hc_eps, params.rms_eps)
    dt = _capi.DTYPE_BF16 if x_dtype == torch.bfloat16 else _capi.DTYPE_F32
    call("gpeed_mhc_pre", ctx.handle, _ptr(streams.contiguous()), n, H, ctypes.byref(p), _ptr(fn.contiguous()),
         _ptr(base.contiguous()), _ptr(scale.contiguous()), _ptr(norm_w.contiguous()), _ptr(x), dt, _ptr(post),
         _ptr(comb), _stream(stream))
    return x, post, comb


def mhc_post(ctx: Context, streams_in: torch.Tensor, mlp_out: torch.Tensor, post: torch.Tensor, comb: torch.Tensor,
             out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Streams after the MLP (model.cpp:309-318): out[t][k] = post[t][k] mlp[t] + sum_m comb[t][m][k] in[t][m]."""
    n, N, H = streams_in.shape
    if out is None:
        out = torch.empty_like(streams_in)
    call("gpeed_mhc_post", ctx.handle, _ptr(streams_in), _ptr(mlp_out.contiguous()), _ptr(post.contiguous()),
         _ptr(comb.contiguous()), n, H, N, _ptr(out), _stream(stream))
    return out


class MoeLayer:
    """One routed-expert MoE layer resident on the device."""

    _next_id = 0

    def __init__(self, ctx: Context, cfg: MoeConfig, layer_id: int | None = None):
        self.ctx, self.cfg = ctx, cfg
        if layer_id is None:
            layer_id = MoeLayer._next_id
            MoeLayer._next_id += 1
        self.layer_id = layer_id
        self._shape = cfg.shape()

    def load(self, router: np.ndarray, corr: np.ndarray | None, gate, up, down, gate_sh=None, up_sh=None,
             down_sh=None) -> "MoeLayer":
        """Raw GGUF IQ3_XXS expert tensors (host numpy or CUDA uint8)."""
        on_dev = isinstance(gate, torch.Tensor) and gate.is_cuda
        conv = (lambda a: a.contiguous()) if on_dev else (lambda a: np.ascontiguousarray(a))
        router = conv(router if on_dev else np.asarray(router, np.float32))
        corr_c = None if corr is None else conv(corr if on_dev else np.asarray(corr, np.float32))
        keep = [conv(t) if t is not None else None for t in (gate, up, down, gate_sh, up_sh, down_sh)]
        call("gpeed_moe_load_layer", self.ctx.handle, self.layer_id, ctypes.byref(self._shape), _ptr(router),
             _ptr(corr_c), *[_ptr(t) for t in keep], int(on_dev))
        return self

    @classmethod
    def from_gguf(cls, ctx: Context, model, blk: int, layer_id: int | None = None, expert_begin: int = 0,
                  expert_count: int | None = None) -> "MoeLayer":
        """Block `blk` of a GGUF model (``gpeed_b200.gguf.GgufModel``), read by tensor name."""
        from .gguf import load_moe_layer
        return load_moe_layer(ctx, model, blk, layer_id, expert_begin, expert_count)

    def synth(self, router: np.ndarray, corr: np.ndarray | None, seed: int, stream0: int) -> "MoeLayer":
        """Expert bytes from the device generator (seed, streams stream0..stream0+5)."""
        router = np.ascontiguousarray(router, np.float32)
        corr_c = None if corr is None else np.ascontiguousarray(corr, np.float32)
        call("gpeed_moe_synth_layer", self.ctx.handle, self.layer_id, ctypes.byref(self._shape), _ptr(router),
             _ptr(corr_c), 0, ctypes.c_uint64(seed), ctypes.c_uint64(stream0))
        return self

    def synth_range(self, router: np.ndarray, corr: np.ndarray | None, seed: int, stream0: int, expert_begin: int,
                    expert_count: int) -> "MoeLayer":
        """Only routed experts [expert_begin, expert_begin + expert_count) plus the
        shared expert, with the bytes of that slice of the whole synthetic layer
        (expert parallelism: one rank's share)."""
        router = np.ascontiguousarray(router, np.float32)
        corr_c = None if corr is None else np.ascontiguousarray(corr, np.float32)
        call("gpeed_moe_synth_layer_range", self.ctx.handle, self.layer_id, ctypes.byref(self._shape), expert_begin,
             expert_count, _ptr(router), _ptr(corr_c), 0, ctypes.c_uint64(seed), ctypes.c_uint64(stream0))
        return self

    def slice_units(self, unit_begin: int, unit_count: int) -> "MoeLayer":
        """Keep units [unit_begin, unit_begin + unit_count) of every routed
        expert, a unit being 32 intermediate rows (gpeed_moe_slice_units): one
        rank's share of the tensor-parallel split of every routed expert; the
        shared expert stays whole.  The layer then serves decode_partial and
        the expert-parallel decode only."""
        call("gpeed_moe_slice_units", self.ctx.handle, self.layer_id, unit_begin, unit_count)
        return self

    @staticmethod
    def unit_slice(cfg: MoeConfig, rank: int, world: int) -> tuple[int, int]:
        """(unit_begin, unit_count) of rank `rank` of `world` equal slices."""
        nu = cfg.inter // 32
        if nu % world:
            raise GpeedError(_capi.ERR_INVALID, f"{nu} units do not split over {world} ranks")
        return rank * (nu // world), nu // world

    def decode_partial(self, x_all: torch.Tensor, own_tok: int, y_part: torch.Tensor | None = None,
                       forced_topk: torch.Tensor | None = None, topk_ids: torch.Tensor | None = None,
                       topk_w: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """One rank's share of an expert-parallel decode step (gpeed_moe_decode_partial):
        x_all [n, H] every rank's token -> y_part [n, H] fp32, the part of each
        token's output that this layer's experts (plus own_tok's shared expert)
        contribute.  The ranks' parts sum to MoeLayer.forward of the whole layer.
        On a sliced layer (slice_units) the part is this slice of every pick
        plus own_tok's whole shared expert."""
        n = x_all.shape[0]
        if y_part is None:
            y_part = torch.empty(n, self.cfg.hidden, dtype=torch.float32, device=x_all.device)
        call("gpeed_moe_decode_partial", self.ctx.handle, self.layer_id, _ptr(x_all), _dtype_code(x_all), n, own_tok,
             _ptr(y_part), _ptr(forced_topk), _ptr(topk_ids), _ptr(topk_w), _stream(stream))
        return y_part

    def forward(self, x: torch.Tensor, y: torch.Tensor | None = None, forced_topk: torch.Tensor | None = None,
                topk_ids: torch.Tensor | None = None, topk_w: torch.Tensor | None = None, stream=None):
        """x [n, H] bf16/fp32 CUDA -> y [n, H] fp32 (Model::moe_forward / moe_batch)."""
        if x.dim() == 1:
            x = x.unsqueeze(0)
        n = x.shape[0]
        if x.dtype == torch.bfloat16:
            dt = _capi.DTYPE_BF16
        elif x.dtype == torch.float32:
            dt = _capi.DTYPE_F32
        else:
            raise GpeedError(_capi.ERR_UNSUPPORTED, f"x dtype {x.dtype}")
        if y is None:
            y = torch.empty(n, self.cfg.hidden, dtype=torch.float32, device=x.device)
        call("gpeed_moe_forward", self.ctx.handle, self.layer_id, _ptr(x.contiguous()), dt, n, _ptr(y),
             _ptr(forced_topk), _ptr(topk_ids), _ptr(topk_w), _stream(stream))
        return y

    def forward_host(self, x: torch.Tensor, y: torch.Tensor | None = None) -> torch.Tensor:
        """x [n, H] bf16/fp32 in host memory -> y [n, H] fp32 in host memory
        (gpeed_moe_forward_host: the reference's callers pass host vectors to
        Model::moe_forward / moe_batch; the call returns with y filled)."""
        if x.dim() == 1:
            x = x.unsqueeze(0)
        if x.is_cuda:
            raise GpeedError(_capi.ERR_INVALID, "forward_host takes host tensors; use forward for device tensors")
        n = x.shape[0]
        if x.dtype == torch.bfloat16:
            dt = _capi.DTYPE_BF16
        elif x.dtype == torch.float32:
            dt = _capi.DTYPE_F32
        else:
            raise GpeedError(_capi.ERR_UNSUPPORTED, f"x dtype {x.dtype}")
        x = x.contiguous()
        if y is None:
            y = torch.empty(n, self.cfg.hidden, dtype=torch.float32)
        if y.is_cuda or y.dtype != torch.float32 or not y.is_contiguous() or y.numel() < n * self.cfg.hidden:
            raise GpeedError(_capi.ERR_INVALID, "y must be a contiguous fp32 host tensor of [n, hidden]")
        call("gpeed_moe_forward_host", self.ctx.handle, self.layer_id, _ptr(x), dt, n, _ptr(y))
        return y
