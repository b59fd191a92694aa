"""GPU test of gpeed_matmul_quant_noalloc.

That entry point exists for callers that cannot call cudaMalloc once they are
serving: an engine whose own allocator or memory pool owns the GPU's memory,
or a process held to a device-memory budget fixed at start-up.  It keeps its
scratch in one static device array inside the library instead.  It runs the
same plan and kernels as gpeed_matmul_quant, so its output must equal that
entry point's bit for bit, and both must sit within the GEMV bar of the
oracle (the C restatement of WeightStore::matmul_quant, weights.cpp:86-165),
call after call: the shared array keeps the previous call's contents.

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpeed_b200 import Context, GpeedError, WeightStore
from gpeed_b200._capi import call
from oracle import oracle
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
GEMV_TOL = 2e-4  # relative L2 against the oracle, the bar of the other expert-matrix tests


def _run(name, ctx, handle, row0, in_dim, out_dim, X, n_tok, Y):
    call(name, ctx.handle, handle, ctypes.c_uint64(row0), in_dim, out_dim, ctypes.c_void_p(X.data_ptr()), n_tok,
         ctypes.c_void_p(Y.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("in_dim,rows,row0,out_dim,n_tok", [
    (5120, 3072, 1536, 1536, 1),   # aligned rows: the output goes straight to Y
    (1536, 5120, 3, 517, 4),       # unaligned rows: staged in the static scratch, then copied
])
def test_noalloc_matches_allocating_entry_point_twice(port, in_dim, rows, row0, out_dim, n_tok):
    ctx = Context(0)
    ws = WeightStore(ctx)
    raw = oracle.synth_iq3xxs(8, in_dim, rows * in_dim // 256)
    ws.add("w", raw, rows, in_dim)
    handle = ws._handles["w"][0]
    rng = np.random.default_rng(in_dim + n_tok)
    for _ in range(2):  # two calls in a row: the shared scratch holds the previous call's contents
        X = rng.standard_normal((n_tok, in_dim)).astype(np.float32)
        Xd = torch.from_numpy(X).cuda()
        want = torch.full((n_tok, out_dim), float("nan"), device="cuda")
        got = torch.full((n_tok, out_dim), float("nan"), device="cuda")
        _run("gpeed_matmul_quant", ctx, handle, row0, in_dim, out_dim, Xd, n_tok, want)
        _run("gpeed_matmul_quant_noalloc", ctx, handle, row0, in_dim, out_dim, Xd, n_tok, got)
        ctx.check()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all()
        np.testing.assert_array_equal(g.view(np.uint32), w.view(np.uint32))
        ref = port.matmul_quant(raw, row0, in_dim, out_dim, X)
        assert rel_l2(g, ref) < GEMV_TOL, rel_l2(g, ref)
    ctx.close()


def test_noalloc_rejects_calls_beyond_the_static_limit():
    ctx = Context(0)
    ws = WeightStore(ctx)
    rows, in_dim = 20016, 512
    ws.add("w", oracle.synth_iq3xxs(8, 1, rows * in_dim // 256), rows, in_dim)
    X = torch.zeros(64, in_dim, device="cuda")
    Y = torch.zeros(64, 20000, device="cuda")
    with pytest.raises(GpeedError, match="static limit"):
        _run("gpeed_matmul_quant_noalloc", ctx, ws._handles["w"][0], 3, in_dim, 20000, X, 64, Y)
    ctx.close()
