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
from .moe import Context, MoeConfig, MoeLayer, _dtype_code, _ptr, _stream




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

    def decode_partial(self, x_all: torch.Tensor, own_tok: int, y_part: torch.Tensor | None = None,
                       stream=None) -> torch.Tensor:
        if y_part is None:
            y_part = self.empty((x_all.shape[0], self.cfg.hidden), torch.float32)
        call("gpeed_moe_decode_partial", self.ctx.handle, self.layer_id, _ptr(x_all), _dtype_code(x_all),
             x_all.shape[0], own_tok, _ptr(y_part), None, None, None, _stream(stream))
        return y_part

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


class StepGuard:
    """Host-side check that every rank reached the same step before any of its
    device work is launched.  Each rank posts "step i" to a shared key-value
    store (torch.distributed's TCPStore) and waits up to `timeout_s` for the
    others' posts; a rank that left between steps (or never joined) turns the
    next step into a GpeedError on the others instead of a collective that
    waits on a missing peer.  Off the device's critical path: use it between
    graph replays in a serving loop, not inside a captured graph."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "gpeed/ep"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix
        self.step = 0

    def __call__(self) -> None:
        import datetime
        key = lambda r: f"{self.prefix}/{self.step}/{r}"
        self.store.set(key(self.rank), "1")
        try:
            self.store.wait([key(r) for r in range(self.world)], datetime.timedelta(seconds=self.timeout_s))
        except Exception as e:  # the store raises on timeout (RuntimeError / DistStoreError)
            missing = [r for r in range(self.world) if not self.store.check([key(r)])]
            raise GpeedError(_capi.ERR_NCCL, f"expert parallelism: rank(s) {missing} did not reach step "
                                             f"{self.step} within {self.timeout_s:.1f} s ({e})") from None
        self.step += 1


class ExpertParallelDecode:
    """Expert-parallel decode of one MoE layer, one token per rank per step.

    The layer's routed experts are split over the ranks (each executor holds
    one contiguous range plus the shared expert).  A step:
      1. all-gather the ranks' tokens                       collective (10 KB each)
      2. every rank runs gpeed_moe_decode_partial: routing of all tokens, its
         experts' share of each token and its own token's shared expert, in
         one persistent kernel                                device
      3. reduce-scatter the partial outputs (sum over ranks)  collective
    No step reads anything back to the host, so steps can be captured in a
    CUDA graph.  With NCCL the collectives are all_gather_into_tensor and
    reduce_scatter_tensor; gloo (CPU tests) has no reduce-scatter and uses
    all_reduce plus the own row.  An optional StepGuard checks on the host,
    before a step's work is launched, that every rank is still there."""

    def __init__(self, cfg: MoeConfig, executor, group=None, guard: StepGuard | None = None):
        self.cfg, self.ex, self.group, self.guard = cfg, executor, group, guard
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if cfg.n_experts % self.world:
            raise GpeedError(_capi.ERR_INVALID, f"{cfg.n_experts} experts do not split over {self.world} ranks")
        if self.world * cfg.top_k > 64 or self.world > 8:
            raise GpeedError(_capi.ERR_UNSUPPORTED, f"{self.world} ranks x top-{cfg.top_k}: at most 8 ranks and 64 "
                                                    f"picks per step")
        self._nccl = dist.get_backend(group) == "nccl"
        self._bufs = {}

    def _buf(self, name, shape, dtype):
        b = self._bufs.get(name)
        if b is None or b.shape != shape or b.dtype != dtype:
            b = self.ex.empty(shape, dtype)
            self._bufs[name] = b
        return b

    def forward(self, x: torch.Tensor, y: torch.Tensor | None = None) -> torch.Tensor:
        """x [1, H] (this rank's token) -> y [1, H] fp32."""
        H, P = self.cfg.hidden, self.world
        if self.guard is not None:
            self.guard()
        x = x.reshape(1, H)
        x_all = self._buf("x_all", (P, H), x.dtype)
        y_part = self._buf("y_part", (P, H), torch.float32)
        if y is None:
            y = self.ex.empty((1, H), torch.float32)
        try:
            if self._nccl:
                dist.all_gather_into_tensor(x_all, x.contiguous(), group=self.group)
            else:
                dist.all_gather(list(x_all.unbind(0)), x.reshape(H).contiguous(), group=self.group)
            self.ex.decode_partial(x_all, self.rank, y_part)
            if self._nccl:
                dist.reduce_scatter_tensor(y, y_part, op=dist.ReduceOp.SUM, group=self.group)
            else:
                dist.all_reduce(y_part, op=dist.ReduceOp.SUM, group=self.group)
                y.copy_(y_part[self.rank:self.rank + 1])
        except RuntimeError as e:  # a collective that failed or timed out (a peer left)
            raise GpeedError(_capi.ERR_NCCL, f"expert-parallel decode step failed: {e}") from e
        return y


class PeerDecode:
    """Expert-parallel decode of one MoE layer with no collective library: one
    token per rank per step, the exchanges inside the persistent kernel over
    NVLink peer memory (gpeed_ep_setup / gpeed_ep_connect / gpeed_moe_decode_ep).

    `layers`: this rank's share of each layer, either its expert range
    (MoeLayer.synth_range / from_gguf with an expert range) or a whole layer
    sliced by units (MoeLayer.slice_units(*MoeLayer.unit_slice(cfg, rank,
    world))), with which every rank runs its slice of every pick: the same
    work on every rank whatever the routing.

    Setup (once per process group, collective): every rank allocates its
    exchange block, the CUDA IPC handles are all-gathered on the host through
    torch.distributed, and every rank maps the others' blocks.  A step is one
    kernel launch per rank: its token reaches every rank as tagged words, all
    tokens are routed, this rank's picks of every token add their down sums
    straight into the owning rank's accumulator, and the launch ends when the
    other ranks have signalled theirs.  Nothing is read back to the host, so
    steps can be captured in CUDA graphs.  Every rank must run the same steps;
    an optional StepGuard checks on the host that every rank is still there
    before a step is launched."""

    def __init__(self, ctx: Context, cfg: MoeConfig, layers, group=None, guard: StepGuard | None = None):
        self.ctx, self.cfg, self.group, self.guard = ctx, cfg, group, guard
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if cfg.n_experts % self.world or self.world > 8 or self.world * cfg.top_k > 64:
            raise GpeedError(_capi.ERR_UNSUPPORTED, f"{self.world} ranks, {cfg.n_experts} experts, top-{cfg.top_k}: "
                                                    "2 .. 8 ranks splitting the experts evenly, at most 64 picks")
        self.layers = {l.layer_id: l for l in (layers if isinstance(layers, (list, tuple)) else [layers])}
        handle = (ctypes.c_uint8 * _capi.IPC_HANDLE_BYTES)()
        call("gpeed_ep_setup", ctx.handle, self.world, self.rank, cfg.hidden, handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        blob = (ctypes.c_uint8 * (_capi.IPC_HANDLE_BYTES * self.world)).from_buffer_copy(b"".join(handles))
        call("gpeed_ep_connect", ctx.handle, blob)
        dist.barrier(group=self.group)  # every block zeroed and mapped before any rank writes into it

    def close(self) -> None:
        """Collective: every rank unmaps the others' blocks, then the group
        meets, so no block is freed (with its context) while still mapped."""
        torch.cuda.synchronize()
        call("gpeed_ep_disconnect", self.ctx.handle)
        dist.barrier(group=self.group)

    def forward(self, layer_id: int, x: torch.Tensor, y: torch.Tensor | None = None, topk_ids=None, topk_w=None,
                stream=None) -> torch.Tensor:
        """x [1, H] (this rank's token, bf16 or fp32) -> y [1, H] fp32, the layer's output for it."""
        if self.guard is not None:
            self.guard()
        H = self.cfg.hidden
        x = x.reshape(1, H).contiguous()
        if y is None:
            y = torch.empty(1, H, dtype=torch.float32, device=x.device)
        call("gpeed_moe_decode_ep", self.ctx.handle, self.layers[layer_id].layer_id, _ptr(x), _dtype_code(x), _ptr(y),
             _ptr(topk_ids), _ptr(topk_w), _stream(stream))
        return y
