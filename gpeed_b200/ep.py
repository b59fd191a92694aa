"""Expert-parallel MoE layer: experts split over the ranks of a process group.

The reference runs every expert on one host (model_batch.cpp:165-281); this
layer spreads the E routed experts over `world` ranks in equal contiguous
ranges, keeps tokens data-parallel and replicates the router and the shared
expert.  One forward on each rank:

  1. route its own tokens (router + top-k)                       device
  2. group the (token, k) assignments by destination rank         device
  3. all-to-all: per-rank counts, then token rows and expert ids  collective
  4. gate/up -> SwiGLU -> down for every received row and, in the
     same pass, the shared expert on this rank's own tokens        device
  5. all-to-all: the expert outputs back to their token's rank    collective
  6. y = sum_k w_k D_k + D_shared                                  device

The collectives are torch.distributed all_to_all_single (NCCL between GPUs,
gloo on CPU); the device steps go through an executor.  The product executor
is `CudaExecutor` (libgpeed_moe.so); there is no CPU executor here.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _capi
from ._capi import GpeedError, call
from .moe import Context, MoeConfig, _ptr, _stream


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _capi.DTYPE_BF16
    if t.dtype == torch.float32:
        return _capi.DTYPE_F32
    raise GpeedError(_capi.ERR_UNSUPPORTED, f"dtype {t.dtype}")


class CudaExecutor:
    """Device steps of the expert-parallel forward through the C ABI."""

    def __init__(self, ctx: Context, cfg: MoeConfig, layer_id: int, expert_begin: int, expert_count: int):
        self.ctx, self.cfg, self.layer_id = ctx, cfg, layer_id
        self.expert_begin, self.expert_count = expert_begin, expert_count
        self._shape = cfg.shape()
        self.device = torch.device("cuda", ctx.device)

    def synth(self, router, corr, seed: int, stream0: int) -> None:
        import numpy as np
        router = np.ascontiguousarray(router, np.float32)
        corr_c = None if corr is None else np.ascontiguousarray(corr, np.float32)
        call("gpeed_moe_synth_layer_range", self.ctx.handle, self.layer_id, ctypes.byref(self._shape),
             self.expert_begin, self.expert_count, _ptr(router), _ptr(corr_c), 0, ctypes.c_uint64(seed),
             ctypes.c_uint64(stream0))

    def load(self, router, corr, gate, up, down, gate_sh, up_sh, down_sh) -> None:
        """gate/up/down: this rank's experts only (GGUF IQ3_XXS bytes, host numpy)."""
        import numpy as np
        conv = lambda a: None if a is None else np.ascontiguousarray(a)
        router = np.ascontiguousarray(router, np.float32)
        corr_c = None if corr is None else np.ascontiguousarray(corr, np.float32)
        keep = [conv(t) for t in (gate, up, down, gate_sh, up_sh, down_sh)]
        call("gpeed_moe_load_layer_range", self.ctx.handle, self.layer_id, ctypes.byref(self._shape),
             self.expert_begin, self.expert_count, _ptr(router), _ptr(corr_c), *[_ptr(t) for t in keep], 0)

    def empty(self, shape, dtype) -> torch.Tensor:
        return torch.empty(shape, dtype=dtype, device=self.device)

    def route(self, x: torch.Tensor):
        n, K = x.shape[0], self.cfg.top_k
        ids = self.empty((n, K), torch.int32)
        w = self.empty((n, K), torch.float32)
        call("gpeed_moe_route", self.ctx.handle, self.layer_id, _ptr(x), _dtype_code(x), n, None, _ptr(ids),
             _ptr(w), _stream(None))
        return ids, w

    def pack(self, ids: torch.Tensor, x: torch.Tensor, world: int):
        n, K = ids.shape
        send_rows = self.empty((n * K, self.cfg.hidden), x.dtype)
        send_ids = self.empty((n * K,), torch.int32)
        counts = self.empty((world,), torch.int32)
        slot_of = self.empty((n, K), torch.int32)
        call("gpeed_ep_pack", self.ctx.handle, self.cfg.n_experts, world, n, K, _ptr(ids), _ptr(x), _dtype_code(x),
             self.cfg.hidden, _ptr(send_rows), _ptr(send_ids), _ptr(counts), _ptr(slot_of), _stream(None))
        return send_rows, send_ids, counts, slot_of

    def experts(self, rows: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        out = self.empty((rows.shape[0], self.cfg.hidden), torch.float32)
        call("gpeed_moe_experts", self.ctx.handle, self.layer_id, _ptr(rows), _dtype_code(rows), rows.shape[0],
             _ptr(ids), _ptr(out), _stream(None))
        return out

    def combine(self, d_rows, slot_of, w, d_shared) -> torch.Tensor:
        n, K = slot_of.shape
        y = self.empty((n, self.cfg.hidden), torch.float32)
        call("gpeed_moe_combine", self.ctx.handle, n, K, self.cfg.hidden, _ptr(d_rows), _ptr(slot_of), _ptr(w),
             _ptr(d_shared), _ptr(y), _stream(None))
        return y


class ExpertParallelLayer:
    """One MoE layer whose routed experts are split over a process group."""

    def __init__(self, cfg: MoeConfig, executor, group=None):
        self.cfg, self.ex, self.group = cfg, executor, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if cfg.n_experts % self.world:
            raise GpeedError(_capi.ERR_INVALID, f"{cfg.n_experts} experts do not split over {self.world} ranks")

    @staticmethod
    def expert_range(cfg: MoeConfig, rank: int, world: int) -> tuple[int, int]:
        epr = cfg.n_experts // world
        return rank * epr, epr

    def _a2a(self, send: torch.Tensor, send_splits, recv_splits) -> torch.Tensor:
        recv = torch.empty((sum(recv_splits),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        dist.all_to_all_single(recv, send.contiguous(), recv_splits, send_splits, group=self.group)
        return recv

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [n, H] (this rank's tokens) -> y [n, H] fp32.

        The received rows and this rank's own rows for the shared expert go
        through one experts pass: the exchange lands in the head of one row
        buffer whose tail holds the own tokens."""
        ex, cfg = self.ex, self.cfg
        n, K = x.shape[0], cfg.top_k
        if n:
            ids, w = ex.route(x)
            send_rows, send_ids, counts, slot_of = ex.pack(ids, x, self.world)
        else:  # a rank without tokens still takes part in every exchange
            w = ex.empty((0, K), torch.float32)
            send_rows = ex.empty((0, cfg.hidden), x.dtype)
            send_ids = ex.empty((0,), torch.int32)
            counts = torch.zeros(self.world, dtype=torch.int32, device=x.device)
            slot_of = ex.empty((0, K), torch.int32)
        send_counts = counts.to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send_splits = send_counts.cpu().tolist()
        recv_splits = recv_counts.cpu().tolist()
        r = sum(recv_splits)
        m = r + (n if cfg.n_shared else 0)
        rows = ex.empty((m, cfg.hidden), x.dtype)
        row_ids = ex.empty((m,), torch.int32)
        dist.all_to_all_single(rows[:r], send_rows.contiguous(), recv_splits, send_splits, group=self.group)
        dist.all_to_all_single(row_ids[:r], send_ids.contiguous(), recv_splits, send_splits, group=self.group)
        if m > r:  # the shared expert on this rank's own tokens
            rows[r:].copy_(x)
            row_ids[r:].fill_(cfg.n_experts)
        d_all = ex.experts(rows, row_ids) if m else ex.empty((0, cfg.hidden), torch.float32)
        d_back = self._a2a(d_all[:r], recv_splits, send_splits)
        if not n:
            return ex.empty((0, cfg.hidden), torch.float32)
        d_shared = d_all[r:] if cfg.n_shared else None
        return ex.combine(d_back, slot_of, w, d_shared)
