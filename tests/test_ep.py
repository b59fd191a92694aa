"""Expert parallelism on CPU ranks (gloo): the exchange logic of
ExpertParallelLayer with the oracle doing the device steps.  The world-2 run
must give the same bits as world 1 (same per-row work, only moved between
ranks) and match the reference's batched layer."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from helpers import host_layer, rel_l2

H, I, E, K = 512, 512, 8, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, splits, out_dir):
    import torch
    import torch.distributed as dist

    from ep_oracle_executor import OracleExecutor
    from gpeed_b200.ep import ExpertParallelLayer
    from gpeed_b200.moe import MoeConfig

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg = MoeConfig(hidden=H, inter=I, n_experts=E, top_k=K)
        layer = host_layer(H, I, E, seed=7, stream0=1, router_seed=2)
        X = np.random.default_rng(11).standard_normal((sum(splits), H)).astype(np.float32)
        b = sum(splits[:rank])
        lo, cnt = ExpertParallelLayer.expert_range(cfg, rank, world)
        ep = ExpertParallelLayer(cfg, OracleExecutor(layer, cfg, lo, cnt))
        y = ep.forward(torch.from_numpy(X[b:b + splits[rank]]))
        np.save(os.path.join(out_dir, f"y{world}_{rank}.npy"), y.numpy())
    finally:
        dist.destroy_process_group()


def _run(world, splits, out_dir):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, splits, out_dir)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    return np.concatenate([np.load(os.path.join(out_dir, f"y{world}_{r}.npy")) for r in range(world)])


@pytest.mark.parametrize("splits", [[3, 3], [5, 0]])
def test_expert_parallel_gloo_matches_single_rank(tmp_path, splits):
    from oracle import oracle
    y1 = _run(1, [sum(splits)], str(tmp_path))
    y2 = _run(2, splits, str(tmp_path))
    np.testing.assert_array_equal(y2, y1)
    layer = host_layer(H, I, E, seed=7, stream0=1, router_seed=2)
    X = np.random.default_rng(11).standard_normal((sum(splits), H)).astype(np.float32)
    Y, _, _ = oracle.Checker("port").moe_batch(oracle.Shape(H, I, E, K, 2.5, 1, 10.0), layer, X)
    assert rel_l2(y1, Y) < 1e-5


def _decode_worker(rank, world, port, out_dir, steps, leave_after):
    import datetime

    import torch
    import torch.distributed as dist

    from ep_oracle_executor import OracleExecutor
    from gpeed_b200 import GpeedError
    from gpeed_b200.ep import ExpertParallelDecode, ExpertParallelLayer, StepGuard
    from gpeed_b200.moe import MoeConfig

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    result = "done"
    try:
        cfg = MoeConfig(hidden=H, inter=I, n_experts=E, top_k=K)
        layer = host_layer(H, I, E, seed=7, stream0=1, router_seed=2)
        lo, cnt = ExpertParallelLayer.expert_range(cfg, rank, world)
        guard = StepGuard(store, rank, world, timeout_s=3.0) if leave_after is not None else None
        ep = ExpertParallelDecode(cfg, OracleExecutor(layer, cfg, lo, cnt), guard=guard)
        X = np.random.default_rng(21).standard_normal((steps, world, H)).astype(np.float32)
        ys = []
        dist.barrier()  # both ranks set up: the guard's short wait times steps, not process start-up
        for s in range(steps):
            if leave_after is not None and rank == world - 1 and s == leave_after:
                result = "left"
                break  # this rank leaves between steps, with nothing in flight
            try:
                ys.append(ep.forward(torch.from_numpy(X[s, rank:rank + 1])).numpy()[0])
            except GpeedError as e:
                result = f"raised: {e}"
                break
        np.save(os.path.join(out_dir, f"dec{world}_{rank}.npy"), np.array(ys, np.float32).reshape(-1, H))
        with open(os.path.join(out_dir, f"dec{world}_{rank}.txt"), "w") as fh:
            fh.write(result)
    finally:
        if result != "left":  # a departed peer cannot take part in a final barrier
            dist.destroy_process_group()


def _run_decode(world, out_dir, steps, leave_after=None):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_decode_worker, args=(r, world, port, out_dir, steps, leave_after))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    return [open(os.path.join(out_dir, f"dec{world}_{r}.txt")).read() for r in range(world)]


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_decode_gloo_matches_the_reference(tmp_path, world):
    """One token per rank per step: all-gather, each rank's share of the experts
    (the oracle standing in for gpeed_moe_decode_partial), sum over ranks.  Every
    rank's output matches the reference batch-1 layer for its token."""
    from oracle import oracle
    steps = 2
    status = _run_decode(world, str(tmp_path), steps)
    assert status == ["done"] * world
    layer = host_layer(H, I, E, seed=7, stream0=1, router_seed=2)
    X = np.random.default_rng(21).standard_normal((steps, world, H)).astype(np.float32)
    chk = oracle.Checker("port")
    shape = oracle.Shape(H, I, E, K, 2.5, 1, 10.0)
    for r in range(world):
        y = np.load(os.path.join(str(tmp_path), f"dec{world}_{r}.npy"))
        for s in range(steps):
            want, _, _ = chk.moe_forward(shape, layer, X[s, r])
            assert rel_l2(y[s], want) < 1e-5


def test_rank_that_leaves_between_steps_is_reported(tmp_path):
    """A rank leaves after the first step with nothing in flight.  The other
    ranks learn of it on the host before their next step's device work (the
    StepGuard's store wait runs out) and get a GpeedError instead of a
    collective that waits forever."""
    status = _run_decode(2, str(tmp_path), steps=3, leave_after=1)
    assert status[1] == "left"
    assert status[0].startswith("raised:") and "did not reach step 1" in status[0], status[0]
    y0 = np.load(os.path.join(str(tmp_path), "dec2_0.npy"))
    assert y0.shape == (1, H)  # the first step completed on both ranks
