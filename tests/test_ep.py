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
