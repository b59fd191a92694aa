"""GPU test of gpeed_matmul_quant_noalloc, the entry point for callers that
cannot allocate device memory while they run (graph capture, a fixed memory
budget, a host engine that owns the allocator).  It must give the same result
as gpeed_matmul_quant, call after call, while using only the library's static
scratch array.  This file is collected last on purpose.
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
GEMV_TOL = 2e-4  # relative L2, same bar as the other expert-matrix tests


def _run(name, ctx, handle, row0, in_dim, out_dim, X, n_tok, Y):
    call(name, ctx.handle, handle, ctypes.c_uint64(row0), in_dim, out_dim, ctypes.c_void_p(X.data_ptr()), n_tok,
         ctypes.c_void_p(Y.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("in_dim,rows,row0,out_dim,n_tok", [
    (5120, 3072, 1536, 1536, 1),   # aligned rows: the output goes straight to Y
    (1536, 5120, 3, 517, 4),       # unaligned rows: staged in the static scratch, then copied
])
def test_noalloc_matches_allocating_entry_point_twice(in_dim, rows, row0, out_dim, n_tok):
    ctx = Context(0)
    ws = WeightStore(ctx)
    ws.add("w", oracle.synth_iq3xxs(8, in_dim, rows * in_dim // 256), rows, in_dim)
    handle = ws._handles["w"][0]
    rng = np.random.default_rng(in_dim + n_tok)
    for _ in range(2):  # two calls in a row: the shared scratch keeps the previous call's contents
        X = torch.from_numpy(rng.standard_normal((n_tok, in_dim)).astype(np.float32)).cuda()
        want = torch.empty(n_tok, out_dim, device="cuda")
        got = torch.full((n_tok, out_dim), float("nan"), device="cuda")
        _run("gpeed_matmul_quant", ctx, handle, row0, in_dim, out_dim, X, n_tok, want)
        _run("gpeed_matmul_quant_noalloc", ctx, handle, row0, in_dim, out_dim, X, n_tok, got)
        ctx.check()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all()
        assert rel_l2(g, w) < GEMV_TOL
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
