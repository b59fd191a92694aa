"""The drop-in boundary on the GPU: a C++ program written like a reference
engine caller (glm5::WeightStore::matvec_quant / matmul_quant, weights.h:38-48,
with std::vector host buffers as model.cpp:733-754 and model_batch.cpp:241-279
pass them) compiled against gpeed_b200/csrc/weight_store.hpp and linked to
libgpeed_moe.so, checked against the oracle at the BASELINE expert shapes."""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
GEMV_TOL = 2e-4  # relative L2, one expert matrix (the bar of the other GEMV tests)
REPO = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))

PROGRAM = r'''
// A reference-style caller: expert tensors registered by name, the
// matvec_quant / matmul_quant calls of Model::moe_forward / moe_batch on
// std::vector buffers, errors as std::runtime_error.
#include "weight_store.hpp"
#include <cstdio>
#include <vector>
static std::vector<char> slurp(const char* p) {
    std::vector<char> v;
    FILE* f = std::fopen(p, "rb");
    if (!f) return v;
    std::fseek(f, 0, SEEK_END); v.resize(std::ftell(f)); std::fseek(f, 0, SEEK_SET);
    if (std::fread(v.data(), 1, v.size(), f) != v.size()) v.clear();
    std::fclose(f);
    return v;
}
int main(int argc, char** argv) {
    const int H = 5120, I = 1536, E = 3, T = 5;   // three experts; a 5-token batch
    std::vector<char> gate = slurp(argv[1]), down = slurp(argv[2]), xs = slurp(argv[3]);
    if (gate.size() != (size_t)E * I * (H / 256) * 98 || down.size() != (size_t)E * H * (I / 256) * 98 ||
        xs.size() != (size_t)T * H * 4) return 2;
    const float* X = reinterpret_cast<const float*>(xs.data());
    try {
        gpeed::WeightStore store(0);
        store.add("blk.3.ffn_gate_exps.weight", gate.data(), false, (uint64_t)E * I, H);
        store.add("blk.3.ffn_down_exps.weight", down.data(), false, (uint64_t)E * H, I);
        std::vector<float> g(I), d(H), gb((size_t)T * I);
        store.matvec_quant("blk.3.ffn_gate_exps.weight", 2 * (uint64_t)I, H, I, X, g.data());        // model.cpp:733
        store.matvec_quant("blk.3.ffn_down_exps.weight", 1 * (uint64_t)H, I, H, g.data(), d.data());  // model.cpp:740
        store.matmul_quant("blk.3.ffn_gate_exps.weight", (uint64_t)I, H, I, X, T, gb.data());        // model_batch.cpp:241
        FILE* f = std::fopen(argv[4], "wb");
        std::fwrite(g.data(), 4, g.size(), f);
        std::fwrite(d.data(), 4, d.size(), f);
        std::fwrite(gb.data(), 4, gb.size(), f);
        std::fclose(f);
        try {  // weights.cpp:170: an unknown tensor throws
            store.matvec_quant("blk.3.ffn_up_exps.weight", 0, H, I, X, g.data());
            return 4;
        } catch (const std::runtime_error&) {
        }
        try {  // rows past the tensor are refused, not read
            store.matvec_quant("blk.3.ffn_gate_exps.weight", (uint64_t)E * I - 8, H, I, X, g.data());
            return 5;
        } catch (const std::runtime_error&) {
        }
    } catch (const std::runtime_error& e) {
        std::printf("error: %s\n", e.what());
        return 3;
    }
    return 0;
}
'''


def test_reference_style_cpp_caller_on_host_buffers(tmp_path):
    H, I, E, T = 5120, 1536, 3, 5
    gate = oracle.synth_iq3xxs(71, 1, E * I * H // 256)
    down = oracle.synth_iq3xxs(71, 2, E * H * I // 256)
    X = np.random.default_rng(71).standard_normal((T, H)).astype(np.float32)
    gate.tofile(tmp_path / "gate.bin")
    down.tofile(tmp_path / "down.bin")
    X.tofile(tmp_path / "x.bin")
    src = tmp_path / "caller.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "caller"
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{REPO}/gpeed_b200/csrc", str(src), "-o", str(exe),
                    f"-L{REPO}/gpeed_b200/lib", "-lgpeed_moe", f"-Wl,-rpath,{REPO}/gpeed_b200/lib"], check=True)
    r = subprocess.run([str(exe), *(str(tmp_path / n) for n in ("gate.bin", "down.bin", "x.bin", "out.bin"))],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    out = np.fromfile(tmp_path / "out.bin", np.float32)
    g, d, gb = out[:I], out[I:I + H], out[I + H:].reshape(T, I)
    port = oracle.Checker("port")
    want_g = port.matmul_quant(gate, 2 * I, H, I, X[:1])[0]
    want_d = port.matmul_quant(down, H, I, H, g[None, :])[0]
    want_gb = port.matmul_quant(gate, I, H, I, X)
    assert rel_l2(g, want_g) < GEMV_TOL
    assert rel_l2(d, want_d) < GEMV_TOL
    assert rel_l2(gb, want_gb) < GEMV_TOL


def test_moe_forward_host_buffers_match_the_device_forward():
    """gpeed_moe_forward_host takes and fills host buffers, as the callers of
    Model::moe_forward / moe_batch (model.cpp:692-756, model_batch.cpp:165-281)
    hold them, and gives the device forward's result: one token (the fused
    kernel), 5 tokens in fp32 (one fused launch per token) and 64 tokens (the
    tensor-core path).  The fused kernel's sums into y land in launch order,
    so the comparison is to rounding; the oracle checks of the device forward
    are in test_gpu_parity.py."""
    import torch

    from gpeed_b200 import Context, GpeedError, MoeConfig, MoeLayer
    ctx = Context(0)
    try:
        cfg = MoeConfig()
        rng = np.random.default_rng(31)
        router = (rng.standard_normal((cfg.n_experts, cfg.hidden)) * 0.02).astype(np.float32)
        layer = MoeLayer(ctx, cfg).synth(router, None, 42, 100)
        for n, dt in ((1, torch.bfloat16), (5, torch.float32), (64, torch.bfloat16)):
            x = torch.from_numpy(rng.standard_normal((n, cfg.hidden)).astype(np.float32)).to(dt)
            y_dev = layer.forward(x.cuda()).cpu().numpy()
            y_host = layer.forward_host(x).numpy()
            ctx.check()
            assert np.isfinite(y_host).all()
            assert rel_l2(y_host, y_dev) < 1e-5, (n, rel_l2(y_host, y_dev))
            y_again = layer.forward_host(x).numpy()  # the staging is reused
            assert rel_l2(y_again, y_dev) < 1e-5
        with pytest.raises(GpeedError):
            layer.forward_host(torch.zeros(1, cfg.hidden).cuda())
    finally:
        ctx.close()
