"""GGUF reader and layer loader (gpeed_b200/csrc/gguf_loader.cpp).

CPU: the reader against the reference's own selftest file and its Python
reader's view of it (tests/golden/ref_selftest.gguf, ref_selftest_gguf.json),
value types, shards, malformed files, the MoE shape from metadata.
GPU: a tiny layer written as GGUF and loaded by tensor name reproduces the
reference harness's outputs (tests/golden/moe_tiny.npz) and the layer loaded
from raw arrays bit for bit; expert ranges; F16 / BF16 routers.
"""
import json
import os
import struct

import numpy as np
import pytest

from gpeed_b200 import GgufModel, GpeedError, MoeConfig, _capi
from tests.gguf_writer import (ARRAY, BOOL, F32, F64, I8, I16, I32, I64, STRING, U8, U16, U32, U64,
                               moe_block_tensors, moe_metadata, write_gguf)

GOLD = os.path.join(os.path.dirname(__file__), "golden")
LAYER_TOL = 1e-3  # relative L2 against the reference harness, as the other layer tests


@pytest.fixture(scope="module")
def ctx():
    from gpeed_b200 import Context
    c = Context(0)
    yield c
    c.close()


def test_reads_the_reference_selftest_file_like_the_reference_reader():
    want = json.load(open(os.path.join(GOLD, "ref_selftest_gguf.json")))
    with GgufModel(os.path.join(GOLD, "ref_selftest.gguf")) as m:
        assert m.n_shards == 1
        assert m.tensor_names() == [t["name"] for t in want["tensors"]]
        for t in want["tensors"]:
            info = m.find_tensor(t["name"])
            assert list(info.dims) == t["dims"] and info.type == t["type"] and info.offset == t["offset"]
        assert sorted(m.keys()) == sorted(want["metadata"])
        for k, v in want["metadata"].items():
            assert m.get(k) == v, k
        # gguf_selftest.cpp's checks: architecture, alignment, test.array
        assert m.get("general.architecture") == "glm5_next" and m.get("general.alignment") == 32
        # the IQ3_XXS block is the known-answer vector the reference decodes
        block = json.load(open(os.path.join(GOLD, "iq3xxs_selftest.json")))["block_hex"]
        assert m.read("test.iq3_xxs").tobytes().hex() == block
        # payload sizes from the ggml type table (quant.cpp:52-116)
        assert [m.find_tensor(n).nbytes for n in m.tensor_names()] == [32, 8, 8, 34, 98]
        f32 = np.frombuffer(m.read("test.f32").tobytes(), np.float32)
        np.testing.assert_array_equal(f32, [1.5, -2.25, 3.0, 4.5, 0.0, 7.75, -0.5, 100.0])
        assert m.find_tensor("missing") is None
        with pytest.raises(GpeedError, match="missing tensor"):
            m.read("missing", 0, 4)
        with pytest.raises(GpeedError, match="outside"):
            m.read("test.iq3_xxs", 90, 16)


def test_every_value_type_and_custom_alignment(tmp_path):
    p = str(tmp_path / "v.gguf")
    kvs = [("u8", U8, 250), ("i8", I8, -5), ("u16", U16, 65000), ("i16", I16, -300), ("u32", U32, 4000000000),
           ("i32", I32, -7), ("f32", F32, 0.25), ("b", BOOL, 1), ("s", STRING, "héllo"), ("u64", U64, 1 << 60),
           ("i64", I64, -(1 << 40)), ("f64", F64, 1e-300), ("arr_f", ARRAY, (F32, [1.5, -2.0])),
           ("arr_s", ARRAY, (STRING, ["a", "bc"])), ("nested", ARRAY, (ARRAY, [(U8, [1, 2]), (U8, [])])),
           ("empty", ARRAY, (I32, []))]
    write_gguf(p, kvs, [("t0", [7], 0, np.arange(7, dtype=np.float32).tobytes()),
                        ("t1", [3, 2], 26, np.arange(6, dtype=np.int32).tobytes())], alignment=64)
    with GgufModel(p) as m:
        assert m.get("u8") == 250 and m.get("i8") == -5 and m.get("u16") == 65000 and m.get("i16") == -300
        assert m.get("u32") == 4000000000 and m.get("i32") == -7 and m.get("f32") == 0.25 and m.get("b") == 1
        assert m.get("s") == "héllo" and m.get("u64") == 1 << 60 and m.get("i64") == -(1 << 40)
        assert m.get("f64") == 1e-300 and m.get("arr_f") == [1.5, -2.0] and m.get("empty") == []
        assert m.get("general.alignment") == 64
        with pytest.raises(GpeedError):
            m.get("arr_s")
        with pytest.raises(GpeedError):
            m.get("nested")
        assert m.find_tensor("t1").offset == 64 and m.find_tensor("t1").dims == (3, 2)
        np.testing.assert_array_equal(np.frombuffer(m.read("t1").tobytes(), np.int32), np.arange(6))
        np.testing.assert_array_equal(np.frombuffer(m.read("t0", 8, 12).tobytes(), np.float32), [2, 3, 4])


def test_shards_are_found_from_any_one_of_them(tmp_path):
    a = np.arange(4, dtype=np.float32)
    write_gguf(str(tmp_path / "m-00001-of-00002.gguf"), [("general.name", STRING, "first"), ("only1", U32, 1)],
               [("x", [4], 0, a.tobytes()), ("dup", [4], 0, a.tobytes())])
    write_gguf(str(tmp_path / "m-00002-of-00002.gguf"), [("general.name", STRING, "second"), ("only2", U32, 2)],
               [("y", [4], 0, (a + 10).tobytes()), ("dup", [4], 0, (a + 20).tobytes())])
    for path in ("m-00002-of-00002.gguf", "m-00001-of-00002.gguf"):
        with GgufModel(str(tmp_path / path)) as m:
            assert m.n_shards == 2
            assert m.tensor_names() == ["x", "dup", "y"]
            assert m.find_tensor("y").shard == 1 and m.find_tensor("dup").shard == 0
            np.testing.assert_array_equal(np.frombuffer(m.read("y").tobytes(), np.float32), a + 10)
            np.testing.assert_array_equal(np.frombuffer(m.read("dup").tobytes(), np.float32), a)
            assert m.get("general.name") == "first" and m.get("only1") == 1 and m.get("only2") == 2
    # a missing shard is an error, as the reference's open of it throws
    os.remove(tmp_path / "m-00002-of-00002.gguf")
    with pytest.raises(GpeedError, match="cannot open"):
        GgufModel(str(tmp_path / "m-00001-of-00002.gguf"))


def test_malformed_files_fail_cleanly(tmp_path):
    good = tmp_path / "g.gguf"
    write_gguf(str(good), [("k", U32, 1)], [("t", [8], 0, np.zeros(8, np.float32).tobytes())])
    raw = good.read_bytes()
    cases = {
        "magic": b"GGUX" + raw[4:],
        "version": raw[:4] + struct.pack("<I", 1) + raw[8:],
        "truncated_table": raw[:60],
        "tensor_past_end": raw[:-16],
    }
    for name, data in cases.items():
        p = tmp_path / f"{name}.gguf"
        p.write_bytes(data)
        if name == "tensor_past_end":
            with GgufModel(str(p)) as m:  # the table parses; the read is refused
                with pytest.raises(GpeedError, match="outside"):
                    m.read("t")
        else:
            with pytest.raises(GpeedError):
                GgufModel(str(p))
    with pytest.raises(GpeedError, match="cannot open"):
        GgufModel(str(tmp_path / "absent.gguf"))


def test_tensor_dims_that_overflow_or_split_a_block_are_refused(tmp_path):
    """A tensor table whose dims multiply past 64 bits, or whose element count
    is not a whole number of blocks of a known type, is rejected by name
    instead of being accepted with a wrapped byte count."""
    p = tmp_path / "wrap.gguf"
    write_gguf(str(p), [], [("big", [1 << 33, 1 << 33], 0, b"")])
    with pytest.raises(GpeedError, match="big.*overflows"):
        GgufModel(str(p))
    p = tmp_path / "partial.gguf"
    write_gguf(str(p), [], [("half_block", [300], 18, b"\0" * 98)])  # IQ3_XXS blocks hold 256 values
    with pytest.raises(GpeedError, match="half_block.*whole blocks"):
        GgufModel(str(p))
    p = tmp_path / "unknown.gguf"  # a type without a known block size still opens (nbytes 0)
    write_gguf(str(p), [], [("odd", [7], 99, b"\0" * 16)])
    with GgufModel(str(p)) as m:
        assert m.find_tensor("odd").nbytes == 0


def _tiny_bytes(z):
    from oracle import oracle
    H, I, E = (int(z[k]) for k in ("H", "I", "E"))
    seed, s0 = int(z["weight_seed"]), int(z["weight_streams"][0])
    dims = [E * I * H, E * I * H, E * H * I, I * H, I * H, H * I]
    return [oracle.synth_iq3xxs(seed, s0 + m, n // 256) for m, n in enumerate(dims)]


def _write_tiny(path, blk=4, router_type=0, arch="glm5-next", **meta):
    z = np.load(os.path.join(GOLD, "moe_tiny.npz"))
    H, I, E, K = (int(z[k]) for k in ("H", "I", "E", "K"))
    mats = _tiny_bytes(z)
    router = z["router"]
    if router_type == 1:
        router = router.astype(np.float16).astype(np.float32)
    elif router_type == 30:
        router = (router.view(np.uint32) & 0xFFFF0000).view(np.float32)
    write_gguf(str(path), moe_metadata(arch, H, I, E, K, **meta),
               moe_block_tensors(blk, router, z["corr"], *mats, H, I, E, router_type=router_type))
    return z, mats, router


def test_moe_shape_from_metadata(tmp_path):
    z, _, _ = _write_tiny(tmp_path / "t.gguf", scale=1.5, norm=False, limit=7.0)
    with GgufModel(str(tmp_path / "t.gguf")) as m:
        cfg = m.moe_config(4)
        assert cfg == MoeConfig(hidden=int(z["H"]), inter=int(z["I"]), n_experts=int(z["E"]), top_k=int(z["K"]),
                                n_shared=1, routed_scale=1.5, norm_topk=False, swiglu_limit=7.0)
        with pytest.raises(GpeedError, match="missing tensor"):
            m.moe_config(5)
    _write_tiny(tmp_path / "s.gguf", gating=1)
    with GgufModel(str(tmp_path / "s.gguf")) as m:
        with pytest.raises(GpeedError, match="gating"):
            m.moe_config(4)


def test_metadata_that_disagrees_with_the_tensors_is_refused(tmp_path):
    z = np.load(os.path.join(GOLD, "moe_tiny.npz"))
    H, I, E, K = (int(z[k]) for k in ("H", "I", "E", "K"))
    mats = _tiny_bytes(z)
    write_gguf(str(tmp_path / "bad.gguf"), moe_metadata("glm5-next", H, I, E + 1, K),
               moe_block_tensors(0, z["router"], z["corr"], *mats, H, I, E))
    with GgufModel(str(tmp_path / "bad.gguf")) as m:
        with pytest.raises(GpeedError, match="metadata"):
            m.moe_config(0)


def test_layer_load_checks_arguments_before_the_device(tmp_path):
    _write_tiny(tmp_path / "t.gguf")
    lib = _capi.load()
    with GgufModel(str(tmp_path / "t.gguf")) as m:
        assert lib.gpeed_moe_load_layer_gguf(None, m.handle, 4, 0, 0, -1, None) == _capi.ERR_INVALID


# ---- GPU: loading by tensor name reproduces the reference outputs ----

@pytest.mark.gpu
def test_gguf_layer_matches_reference_and_raw_load(tmp_path, ctx):
    import torch
    from gpeed_b200 import MoeLayer
    from tests.helpers import rel_l2
    z, mats, _ = _write_tiny(tmp_path / "t.gguf", blk=4)
    with GgufModel(str(tmp_path / "t.gguf")) as m:
        layer = MoeLayer.from_gguf(ctx, m, 4)
    cfg = layer.cfg
    raw = MoeLayer(ctx, cfg).load(z["router"], z["corr"], *mats)
    X = torch.from_numpy(z["X"]).cuda()
    for t in range(X.shape[0]):
        ids = torch.empty(1, cfg.top_k, dtype=torch.int32, device="cuda")
        y = layer.forward(X[t:t + 1], topk_ids=ids)
        y_raw = raw.forward(X[t:t + 1])
        ctx.check()
        np.testing.assert_array_equal(ids.cpu().numpy()[0], z["fwd_topk"][t])
        assert rel_l2(y.cpu().numpy()[0], z["fwd_y"][t]) < LAYER_TOL
        assert torch.equal(y, y_raw)
    Y = layer.forward(X)
    ctx.check()
    assert rel_l2(Y.cpu().numpy(), z["bat_y"]) < LAYER_TOL
    assert torch.equal(Y, raw.forward(X))


@pytest.mark.gpu
@pytest.mark.parametrize("router_type", [1, 30])
def test_gguf_half_precision_routers_widen_exactly(tmp_path, ctx, router_type):
    import torch
    from gpeed_b200 import MoeLayer
    z, mats, router = _write_tiny(tmp_path / "t.gguf", blk=0, router_type=router_type)
    with GgufModel(str(tmp_path / "t.gguf")) as m:
        layer = MoeLayer.from_gguf(ctx, m, 0)
    raw = MoeLayer(ctx, layer.cfg).load(router, z["corr"], *mats)
    X = torch.from_numpy(z["X"]).cuda()
    assert torch.equal(layer.forward(X), raw.forward(X))
    ctx.check()


@pytest.mark.gpu
def test_gguf_expert_range_load(tmp_path, ctx):
    import ctypes
    import torch
    from gpeed_b200 import MoeLayer
    from gpeed_b200._capi import call
    z, mats, _ = _write_tiny(tmp_path / "t.gguf", blk=2)
    E, H = int(z["E"]), int(z["H"])
    with GgufModel(str(tmp_path / "t.gguf")) as m:
        full = MoeLayer.from_gguf(ctx, m, 2)
        part = MoeLayer.from_gguf(ctx, m, 2, expert_begin=3, expert_count=4)
    g = torch.Generator().manual_seed(5)
    rows = torch.randn(12, H, generator=g).to(torch.bfloat16).cuda()
    ids = torch.tensor([3, 4, 5, 6, 6, 5, 4, 3, E, E, 3, 6], dtype=torch.int32, device="cuda")
    outs = []
    for layer in (full, part):
        out = torch.empty(12, H, dtype=torch.float32, device="cuda")
        call("gpeed_moe_experts", ctx.handle, layer.layer_id, ctypes.c_void_p(rows.data_ptr()), _capi.DTYPE_BF16, 12,
             ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(out.data_ptr()), None)
        outs.append(out)
    ctx.check()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.gpu
def test_cpp_shim_resolves_names_in_a_gguf_model(tmp_path):
    """gpeed::WeightStore(gpeed::GgufModel) takes the reference's call by tensor name."""
    import subprocess
    z, _, _ = _write_tiny(tmp_path / "t.gguf", blk=4)
    H, I = int(z["H"]), int(z["I"])
    z["X"][0].astype(np.float32).tofile(tmp_path / "x.bin")
    src = tmp_path / "shim.cpp"
    src.write_text(r'''
#include "weight_store.hpp"
#include <cuda_runtime.h>
#include <cstdio>
#include <vector>
int main(int argc, char** argv) {
    const int H = %d, I = %d;
    std::vector<float> x(H), y(I);
    FILE* f = std::fopen(argv[2], "rb");
    if (!f || std::fread(x.data(), 4, H, f) != (size_t)H) return 2;
    std::fclose(f);
    try {
        gpeed::GgufModel model(argv[1]);
        gpeed::WeightStore store(model, 0);
        // the reference's call on host buffers (model.cpp:733)
        store.matvec_quant("blk.4.ffn_gate_exps.weight", 3 * I, H, I, x.data(), y.data());
        // and the device variant gives the same bits
        float *xd, *yd;
        std::vector<float> y2(I);
        cudaMalloc(&xd, 4 * H); cudaMalloc(&yd, 4 * I);
        cudaMemcpy(xd, x.data(), 4 * H, cudaMemcpyHostToDevice);
        store.matvec_quant_device("blk.4.ffn_gate_exps.weight", 3 * I, H, I, xd, yd);
        cudaMemcpy(y2.data(), yd, 4 * I, cudaMemcpyDeviceToHost);
        store.check_device();
        if (y2 != y) return 5;
        try {
            store.matvec_quant("blk.4.no_such.weight", 0, H, I, x.data(), y.data());
            return 4;
        } catch (const std::runtime_error&) {
        }
    } catch (const std::runtime_error& e) {
        std::printf("error: %%s\n", e.what());
        return 3;
    }
    f = std::fopen(argv[3], "wb");
    std::fwrite(y.data(), 4, I, f);
    std::fclose(f);
    return 0;
}
''' % (H, I))
    repo = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    exe = tmp_path / "shim"
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{repo}/gpeed_b200/csrc", "-I/usr/local/cuda/include", str(src),
                    "-o", str(exe), f"-L{repo}/gpeed_b200/lib", "-lgpeed_moe", f"-Wl,-rpath,{repo}/gpeed_b200/lib",
                    "-L/usr/local/cuda/lib64", "-lcudart"], check=True)
    r = subprocess.run([str(exe), str(tmp_path / "t.gguf"), str(tmp_path / "x.bin"), str(tmp_path / "y.bin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    y = np.fromfile(tmp_path / "y.bin", np.float32)
    want = z["matvec_y"]
    assert int(z["matvec_row0"]) == 3 * I
    assert np.linalg.norm(y - want) / np.linalg.norm(want) < 2e-4  # the expert-matrix bar of the GEMV tests
