"""CPU checks of the C ABI: the library loads, exports every declared entry
point, and rejects bad arguments before touching a device."""
import ctypes
import os
import re

import pytest

from gpeed_b200 import _capi

HDR = os.path.join(os.path.dirname(__file__), "..", "include", "gpeed_moe.h")


def declared_functions():
    text = open(HDR).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:GPEED_API\s+)?(?:const\s+)?\w+\*?\s+\**(gpeed_\w+)\s*\(", text, re.M)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("gpeed_matvec_quant", "gpeed_matmul_quant", "gpeed_iq3xxs_dequantize", "gpeed_moe_forward",
                 "gpeed_moe_load_layer", "gpeed_ctx_create", "gpeed_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _capi.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # and the binding covers them all
    assert set(declared_functions()) <= set(_capi.SIGNATURES)


def test_argument_errors_need_no_device():
    lib = _capi.load()
    rc = lib.gpeed_iq3xxs_dequantize(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_uint64(255), None)
    assert rc == _capi.ERR_INVALID
    assert b"multiple of block size" in lib.gpeed_last_error()
    rc = lib.gpeed_moe_forward(None, 0, None, 30, 1, None, None, None, None, None)
    assert rc == _capi.ERR_INVALID
    rc = lib.gpeed_moe_forward_host(None, 0, None, 30, 1, None)
    assert rc == _capi.ERR_INVALID
    rc = lib.gpeed_moe_decode_ep(None, 0, None, 30, None, None, None, None)
    assert rc == _capi.ERR_INVALID


def test_ctx_create_fails_cleanly_without_a_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    h = ctypes.c_void_p()
    rc = _capi.load().gpeed_ctx_create(0, ctypes.byref(h))
    assert rc != _capi.OK and not h.value
    with pytest.raises(_capi.GpeedError):
        _capi.check(rc)


def test_cpp_shim_compiles_and_throws_like_the_reference(tmp_path):
    """gpeed_b200/csrc/weight_store.hpp: reference signatures, std::runtime_error on failure."""
    import subprocess
    import torch
    src = tmp_path / "shim.cpp"
    src.write_text(r'''
#include "weight_store.hpp"
#include <cstdio>
int main() {
    try {
        gpeed::WeightStore ws(0);               // throws without a B200
        ws.matvec_quant("blk.3.ffn_gate_exps.weight", 0, 5120, 1536, nullptr, nullptr);
    } catch (const std::runtime_error& e) {
        std::printf("caught: %s\n", e.what());
        return 0;
    }
    return 3;
}
''')
    repo = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    exe = tmp_path / "shim"
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{repo}/gpeed_b200/csrc", str(src), "-o", str(exe),
                    f"-L{repo}/gpeed_b200/lib", "-lgpeed_moe", f"-Wl,-rpath,{repo}/gpeed_b200/lib"], check=True)
    if torch.cuda.is_available():
        pytest.skip("compiled; the throw path needs a machine without a usable device")
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and "caught: gpeed:" in r.stdout
