"""Expert parallelism on the GPU.  One GPU: two ranks emulated in one process
(two expert-range layers, the exchange done by slicing) against the
single-GPU batched forward.  Two GPUs: the real NCCL exchange."""
import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

from gpeed_b200 import Context, MoeConfig, MoeLayer
from gpeed_b200.ep import CudaExecutor, ExpertParallelLayer
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
SEED, S0 = 42, 100


def _router(cfg):
    return (np.random.default_rng(1).standard_normal((cfg.n_experts, cfg.hidden)) * 0.02).astype(np.float32)


def _tokens(cfg, n):
    return torch.from_numpy(np.random.default_rng(5).standard_normal((n, cfg.hidden)).astype(np.float32)).to(
        torch.bfloat16)


def test_ep_device_steps_emulated_two_ranks():
    """The orchestration, bit for bit: every step on the quantised GEMV path so
    the split layer must reproduce the single-GPU layer exactly (the
    tensor-core experts step has its own test)."""
    from gpeed_b200 import _capi
    ctx = Context(0)
    ctx.set_option(_capi.OPT_TC_MIN_TOKENS, 1 << 30)
    try:
        cfg = MoeConfig()
        router = _router(cfg)
        full = MoeLayer(ctx, cfg, layer_id=300).synth(router, None, SEED, S0)
        splits = [10, 6]
        X = _tokens(cfg, sum(splits)).cuda()
        y_ref = full.forward(X)
        ids_ref = torch.empty(sum(splits), cfg.top_k, dtype=torch.int32, device="cuda")
        full.forward(X, topk_ids=ids_ref)
        ex = []
        for r in range(2):
            lo, cnt = ExpertParallelLayer.expert_range(cfg, r, 2)
            e = CudaExecutor(ctx, cfg, 301 + r, lo, cnt)
            e.synth(router, None, SEED, S0)
            ex.append(e)
        Xr = list(torch.split(X, splits))
        routed = [ex[r].route(Xr[r]) for r in range(2)]
        packed = [ex[r].pack(routed[r][0], Xr[r], 2) for r in range(2)]
        counts = [p[2].cpu().tolist() for p in packed]
        off = [np.concatenate([[0], np.cumsum(c)]).tolist() for c in counts]
        # rank d receives the segments addressed to it, in source order
        recv_rows = [torch.cat([packed[r][0][off[r][d]:off[r][d + 1]] for r in range(2)]) for d in range(2)]
        recv_ids = [torch.cat([packed[r][1][off[r][d]:off[r][d + 1]] for r in range(2)]) for d in range(2)]
        d_recv = [ex[d].experts(recv_rows[d], recv_ids[d]) for d in range(2)]
        recv_off = [np.concatenate([[0], np.cumsum([counts[r][d] for r in range(2)])]).tolist() for d in range(2)]
        ys = []
        for r in range(2):
            d_back = torch.cat([d_recv[d][recv_off[d][r]:recv_off[d][r + 1]] for d in range(2)])
            shared = torch.full((splits[r],), cfg.n_experts, dtype=torch.int32, device="cuda")
            d_sh = ex[r].experts(Xr[r], shared)
            ys.append(ex[r].combine(d_back, packed[r][3], routed[r][1], d_sh))
        ctx.check()
        np.testing.assert_array_equal(torch.cat([routed[0][0], routed[1][0]]).cpu().numpy(), ids_ref.cpu().numpy())
        assert rel_l2(torch.cat(ys).cpu().numpy(), y_ref.cpu().numpy()) < 1e-6
        # a range layer refuses the single-GPU forward
        with pytest.raises(Exception, match="expert-parallel"):
            MoeLayer(ctx, cfg, layer_id=301).forward(X)
    finally:
        ctx.close()


def test_ep_experts_step_tensor_core_path():
    """The experts step of an expert-range layer at prefill sizes (2048 rows for
    its 80 experts, then 1024 rows of the shared expert) runs the tensor-core
    GEMMs; it must agree with the same step on the GEMV path within the layer
    tolerance."""
    from gpeed_b200 import _capi
    ctx = Context(0)
    try:
        cfg = MoeConfig()
        lo, cnt = ExpertParallelLayer.expert_range(cfg, 1, 2)
        ex = CudaExecutor(ctx, cfg, 320, lo, cnt)
        ex.synth(_router(cfg), None, SEED, S0)
        rng = np.random.default_rng(11)
        outs = {}
        for name, m, ids in (("routed", 2048, rng.integers(lo, lo + cnt, 2048)),
                             ("shared", 1024, np.full(1024, cfg.n_experts))):
            rows = _tokens(cfg, m).cuda()
            idt = torch.from_numpy(ids.astype(np.int32)).cuda()
            y_tc = ex.experts(rows, idt)
            ctx.check()
            ctx.set_option(_capi.OPT_TC_MIN_TOKENS, 1 << 30)
            try:
                y_gemv = ex.experts(rows, idt)
                ctx.check()
            finally:
                ctx.set_option(_capi.OPT_TC_MIN_TOKENS, _capi.TC_MIN_TOKENS_DEFAULT)
            outs[name] = rel_l2(y_tc.cpu().numpy(), y_gemv.cpu().numpy())
        assert outs["routed"] < 1e-3 and outs["shared"] < 1e-3, outs
    finally:
        ctx.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, splits, out_dir):
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        from gpeed_b200 import _capi
        ctx = Context(rank)
        ctx.set_option(_capi.OPT_TC_MIN_TOKENS, 1 << 30)  # GEMV path on both sides: exact comparison
        cfg = MoeConfig()
        lo, cnt = ExpertParallelLayer.expert_range(cfg, rank, world)
        ex = CudaExecutor(ctx, cfg, 0, lo, cnt)
        ex.synth(_router(cfg), None, SEED, S0)
        ep = ExpertParallelLayer(cfg, ex)
        X = _tokens(cfg, sum(splits))
        b = sum(splits[:rank])
        y = ep.forward(X[b:b + splits[rank]].cuda())
        ctx.check()
        np.save(os.path.join(out_dir, f"y_{rank}.npy"), y.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_nccl_two_gpus(tmp_path):
    from gpeed_b200 import _capi
    splits = [9, 7]
    cfg = MoeConfig()
    ctx = Context(0)
    ctx.set_option(_capi.OPT_TC_MIN_TOKENS, 1 << 30)
    try:
        y_ref = MoeLayer(ctx, cfg, layer_id=400).synth(_router(cfg), None, SEED, S0).forward(
            _tokens(cfg, sum(splits)).cuda()).cpu().numpy()
    finally:
        ctx.close()
    mpc = mp.get_context("spawn")
    port = _free_port()
    procs = [mpc.Process(target=_nccl_worker, args=(r, 2, port, splits, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    y = np.concatenate([np.load(os.path.join(str(tmp_path), f"y_{r}.npy")) for r in range(2)])
    assert rel_l2(y, y_ref) < 1e-6


# ---- expert-parallel decode: one token per rank, one persistent kernel per rank ----

def _ep_layers(ctx, cfg, world, base_id):
    router = _router(cfg)
    full = MoeLayer(ctx, cfg, layer_id=base_id).synth(router, None, SEED, S0)
    parts = []
    for r in range(world):
        lo, cnt = ExpertParallelLayer.expert_range(cfg, r, world)
        parts.append(MoeLayer(ctx, cfg, layer_id=base_id + 1 + r).synth_range(router, None, SEED, S0, lo, cnt))
    return full, parts


@pytest.mark.parametrize("world", [2, 4, 8])
def test_decode_partial_emulated_ranks(port, world):
    """gpeed_moe_decode_partial for each rank of an emulated `world`-rank step
    (the ranks' launches run one after another on one GPU: nothing waits across
    launches).  Routing is bit-identical to the batch-1 forward of each token;
    the sum of the ranks' parts matches it up to the order of that sum, and the
    oracle at the layer bar; tokens with no pick on a rank get exact zeros."""
    from oracle import oracle
    ctx = Context(0)
    try:
        cfg = MoeConfig()
        full, parts = _ep_layers(ctx, cfg, world, 500 + 20 * world)
        X = torch.from_numpy(np.random.default_rng(world).standard_normal((world, cfg.hidden)).astype(np.float32)).to(
            torch.bfloat16).cuda()
        K = cfg.top_k
        y_ref = torch.empty(world, cfg.hidden, device="cuda")
        ids_ref = torch.empty(world, K, dtype=torch.int32, device="cuda")
        w_ref = torch.empty(world, K, dtype=torch.float32, device="cuda")
        for t in range(world):
            full.forward(X[t:t + 1], y_ref[t:t + 1], topk_ids=ids_ref[t:t + 1], topk_w=w_ref[t:t + 1])
        y_parts = []
        for r in range(world):
            ids = torch.full((world, K), -1, dtype=torch.int32, device="cuda")
            w = torch.zeros(world, K, device="cuda")
            y_parts.append(parts[r].decode_partial(X, r, topk_ids=ids, topk_w=w))
            ctx.check()
            np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())
            np.testing.assert_array_equal(w.cpu().numpy(), w_ref.cpu().numpy())
        y_ep = torch.stack(y_parts).sum(0).cpu().numpy()
        g = ids_ref.cpu().numpy()
        epr = cfg.n_experts // world
        for r in range(world):
            yp = y_parts[r].cpu().numpy()
            for t in range(world):
                if t != r and not ((g[t] >= r * epr) & (g[t] < (r + 1) * epr)).any():
                    assert not yp[t].any()
        for t in range(world):
            assert rel_l2(y_ep[t], y_ref.cpu().numpy()[t]) < 1e-5
        host = {**{n: oracle.synth_iq3xxs(SEED, S0 + m, c) for m, (n, c) in enumerate(
            [("gate", cfg.n_experts * cfg.inter * cfg.hidden // 256), ("up", cfg.n_experts * cfg.inter * cfg.hidden // 256),
             ("down", cfg.n_experts * cfg.hidden * cfg.inter // 256), ("gate_sh", cfg.inter * cfg.hidden // 256),
             ("up_sh", cfg.inter * cfg.hidden // 256), ("down_sh", cfg.hidden * cfg.inter // 256)])},
                "router": _router(cfg), "corr": np.zeros(cfg.n_experts, np.float32)}
        shape = oracle.Shape(cfg.hidden, cfg.inter, cfg.n_experts, K, cfg.routed_scale, int(cfg.norm_topk),
                             cfg.swiglu_limit)
        for t in (0, world - 1):
            y_o, _, _ = port.moe_forward(shape, host, X[t].float().cpu().numpy(), forced=g[t])
            assert rel_l2(y_ep[t], y_o) < 1e-3
    finally:
        ctx.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_decode_partial_sliced_emulated_ranks(world):
    """Each emulated rank holds units [r*NU/world, (r+1)*NU/world) of every
    routed expert and the whole shared expert (gpeed_moe_slice_units): its
    gpeed_moe_decode_partial runs that slice of every pick and its own token's
    shared expert.  Routing is bit-identical to the batch-1 forward; the ranks'
    parts add up to it (SwiGLU is row-wise, so only the order of the down sums
    changes), for `world` tokens and for one token; a sliced layer refuses the
    whole-layer paths."""
    from gpeed_b200 import GpeedError
    ctx = Context(0)
    try:
        cfg = MoeConfig()
        K = cfg.top_k
        router = _router(cfg)
        full = MoeLayer(ctx, cfg, layer_id=900 + 20 * world).synth(router, None, SEED, S0)
        parts = []
        for r in range(world):
            lo, cnt = MoeLayer.unit_slice(cfg, r, world)
            layer = MoeLayer(ctx, cfg, layer_id=901 + 20 * world + r).synth(router, None, SEED, S0)
            parts.append(layer.slice_units(lo, cnt))
        X = torch.from_numpy(np.random.default_rng(10 + world).standard_normal((world, cfg.hidden)).astype(
            np.float32)).to(torch.bfloat16).cuda()
        y_ref = torch.empty(world, cfg.hidden, device="cuda")
        ids_ref = torch.empty(world, K, dtype=torch.int32, device="cuda")
        w_ref = torch.empty(world, K, dtype=torch.float32, device="cuda")
        for t in range(world):
            full.forward(X[t:t + 1], y_ref[t:t + 1], topk_ids=ids_ref[t:t + 1], topk_w=w_ref[t:t + 1])
        y_parts = []
        for r in range(world):
            ids = torch.full((world, K), -1, dtype=torch.int32, device="cuda")
            w = torch.zeros(world, K, device="cuda")
            y_parts.append(parts[r].decode_partial(X, r, topk_ids=ids, topk_w=w))
            ctx.check()
            np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())
            np.testing.assert_array_equal(w.cpu().numpy(), w_ref.cpu().numpy())
            assert y_parts[-1].abs().sum(1).min().item() > 0  # every token has a part on every rank
        y_ep = torch.stack(y_parts).sum(0).cpu().numpy()
        for t in range(world):
            assert rel_l2(y_ep[t], y_ref.cpu().numpy()[t]) < 1e-5, (t, rel_l2(y_ep[t], y_ref.cpu().numpy()[t]))
        # one token alone on the rank that owns it: the same part as its row above
        one = parts[1].decode_partial(X[1:2], 0)
        ctx.check()
        assert rel_l2(one.cpu().numpy()[0], y_parts[1].cpu().numpy()[1]) < 1e-5
        with pytest.raises(GpeedError):
            parts[0].forward(X[:1])
        with pytest.raises(GpeedError):
            parts[0].slice_units(0, 6)  # already sliced
        with pytest.raises(GpeedError):
            full.slice_units(3, 6)  # not on a multiple of the slice
        with pytest.raises(GpeedError):
            full.slice_units(0, 16)  # no kernel for a third of the units
    finally:
        ctx.close()


def test_decode_partial_crowded_rank_and_limits():
    """Every pick of 8 tokens forced onto one rank's experts: that rank runs the
    most slots a launch takes (64 routed + its shared expert), the others only
    their shared expert.  Also the single-token form (every expert held) equals
    gpeed_moe_forward (to rounding: the sums into y land in launch order), and
    out-of-range arguments are refused."""
    from gpeed_b200 import GpeedError
    ctx = Context(0)
    try:
        cfg = MoeConfig()
        world, K = 8, cfg.top_k
        full, parts = _ep_layers(ctx, cfg, world, 700)
        X = torch.from_numpy(np.random.default_rng(3).standard_normal((world, cfg.hidden)).astype(np.float32)).to(
            torch.bfloat16).cuda()
        forced = torch.tensor([[(t + k) % 20 + 40 for k in range(K)] for t in range(world)], dtype=torch.int32,
                              device="cuda")  # experts 40..59: rank 2 of 8
        y_ref = torch.empty(world, cfg.hidden, device="cuda")
        for t in range(world):
            full.forward(X[t:t + 1], y_ref[t:t + 1], forced_topk=forced[t:t + 1])
        y_ep = sum(parts[r].decode_partial(X, r, forced_topk=forced) for r in range(world))
        ctx.check()
        assert rel_l2(y_ep.cpu().numpy(), y_ref.cpu().numpy()) < 1e-5
        one = full.decode_partial(X[:1], 0)
        ctx.check()
        assert rel_l2(one.cpu().numpy(), full.forward(X[:1]).cpu().numpy()) < 1e-6
        with pytest.raises(GpeedError):
            parts[0].decode_partial(torch.zeros(9, cfg.hidden, dtype=torch.bfloat16, device="cuda"), 0)
        with pytest.raises(GpeedError):
            parts[0].decode_partial(X, world)
        with pytest.raises(GpeedError):
            parts[0].decode_partial(X[:1], 0)  # one token needs every expert
    finally:
        ctx.close()


def _nccl_decode_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from gpeed_b200.ep import ExpertParallelDecode
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        ctx = Context(rank)
        cfg = MoeConfig()
        lo, cnt = ExpertParallelLayer.expert_range(cfg, rank, world)
        ex = CudaExecutor(ctx, cfg, 0, lo, cnt)
        ex.synth(_router(cfg), None, SEED, S0)
        ep = ExpertParallelDecode(cfg, ex)
        X = _tokens(cfg, 2 * world).reshape(2, world, cfg.hidden)
        ys = [ep.forward(X[s, rank:rank + 1].cuda()).cpu().numpy() for s in range(2)]
        ctx.check()
        np.save(os.path.join(out_dir, f"yd_{rank}.npy"), np.concatenate(ys))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_decode_nccl_two_gpus(tmp_path):
    cfg = MoeConfig()
    ctx = Context(0)
    try:
        full = MoeLayer(ctx, cfg, layer_id=800).synth(_router(cfg), None, SEED, S0)
        X = _tokens(cfg, 4).reshape(2, 2, cfg.hidden)
        y_ref = np.stack([np.concatenate([full.forward(X[s, r:r + 1].cuda()).cpu().numpy() for s in range(2)])
                          for r in range(2)])
    finally:
        ctx.close()
    mpc = mp.get_context("spawn")
    port = _free_port()
    procs = [mpc.Process(target=_nccl_decode_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(2):
        assert rel_l2(np.load(os.path.join(str(tmp_path), f"yd_{r}.npy")), y_ref[r]) < 1e-5


# ---- expert-parallel decode over peer memory (no collective library on the data path) ----

def _peer_decode_worker(rank, world, port, out_dir, sliced=False):
    import torch.distributed as dist
    from gpeed_b200 import GpeedError, _capi
    from gpeed_b200.ep import PeerDecode
    torch.cuda.set_device(rank)
    # gloo, host only: it carries the IPC handles at setup and the final barrier
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        ctx = Context(rank)
        cfg = MoeConfig()
        if sliced:
            layer = MoeLayer(ctx, cfg, layer_id=0).synth(_router(cfg), None, SEED, S0)
            layer.slice_units(*MoeLayer.unit_slice(cfg, rank, world))
        else:
            lo, cnt = ExpertParallelLayer.expert_range(cfg, rank, world)
            layer = MoeLayer(ctx, cfg, layer_id=0).synth_range(_router(cfg), None, SEED, S0, lo, cnt)
        pd = PeerDecode(ctx, cfg, layer)
        X = _tokens(cfg, 3 * world).reshape(3, world, cfg.hidden)
        ys, ids = [], []
        for s in range(3):
            tk = torch.full((world, cfg.top_k), -1, dtype=torch.int32, device="cuda")
            y = pd.forward(0, X[s, rank:rank + 1].cuda(), topk_ids=tk)
            ctx.check()
            ys.append(y.cpu().numpy())
            ids.append(tk.cpu().numpy())
        np.save(os.path.join(out_dir, f"yp_{rank}.npy"), np.concatenate(ys))
        np.save(os.path.join(out_dir, f"ip_{rank}.npy"), np.stack(ids))
        # rank 1 takes no part in the next step: rank 0's waits for its token run
        # out (a short limit) and the status says so; no fault, no hang
        dist.barrier()
        if rank == 0:
            ctx.set_option(_capi.OPT_SPIN_LIMIT, 1 << 10)
            pd.forward(0, X[0, 0:1].cuda())
            try:
                ctx.check()
                msg = "no error"
            except GpeedError as e:
                msg = str(e)
            with open(os.path.join(out_dir, "timeout.txt"), "w") as fh:
                fh.write(msg)
        dist.barrier()
        pd.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("sliced", [False, True], ids=["expert_ranges", "unit_slices"])
def test_ep_decode_peer_memory_two_gpus(tmp_path, sliced):
    """PeerDecode on two GPUs, each rank holding half the experts or half of
    every expert's units: three steps, each rank's output equals the one-GPU
    layer on its token (the two ranks' sums land in another order: to
    rounding), the picks of both tokens equal the one-GPU routing; then a step
    that one rank skips times out on the other, reported by gpeed_ctx_check."""
    cfg = MoeConfig()
    ctx = Context(0)
    try:
        full = MoeLayer(ctx, cfg, layer_id=810).synth(_router(cfg), None, SEED, S0)
        X = _tokens(cfg, 6).reshape(3, 2, cfg.hidden)
        y_ref = np.zeros((2, 3, cfg.hidden), np.float32)
        id_ref = np.zeros((3, 2, cfg.top_k), np.int32)
        for s in range(3):
            for r in range(2):
                tk = torch.empty(1, cfg.top_k, dtype=torch.int32, device="cuda")
                y_ref[r, s] = full.forward(X[s, r:r + 1].cuda(), topk_ids=tk).cpu().numpy()[0]
                id_ref[s, r] = tk.cpu().numpy()[0]
        ctx.check()
    finally:
        ctx.close()
    mpc = mp.get_context("spawn")
    port = _free_port()
    procs = [mpc.Process(target=_peer_decode_worker, args=(r, 2, port, str(tmp_path), sliced)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(2):
        y = np.load(os.path.join(str(tmp_path), f"yp_{r}.npy"))
        assert rel_l2(y, y_ref[r]) < 1e-5, rel_l2(y, y_ref[r])
        ids = np.load(os.path.join(str(tmp_path), f"ip_{r}.npy"))
        for s in range(3):
            for t in range(2):
                assert sorted(ids[s, t]) == sorted(id_ref[s, t])
    msg = open(os.path.join(str(tmp_path), "timeout.txt")).read()
    assert "device status" in msg and "no error" not in msg, msg
