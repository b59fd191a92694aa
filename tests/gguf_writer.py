"""Minimal GGUF v3 writer for the tests (the public file layout: magic,
version, tensor and key counts, typed key/values, tensor table, then the
tensor data at `general.alignment`).  Test infrastructure only."""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
        I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        etype, items = v
        return struct.pack("<IQ", etype, len(items)) + b"".join(_value(etype, x) for x in items)
    return struct.pack(_FMT[vtype], v)


def write_gguf(path, kvs, tensors, alignment: int = 32, version: int = 3, pad_after_table: bool = True) -> None:
    """kvs: [(key, vtype, value)]; arrays as (ARRAY, (elem_type, [items])).
    tensors: [(name, dims (ne order), ggml type, payload bytes)]."""
    if alignment != 32 and not any(k == "general.alignment" for k, _, _ in kvs):
        kvs = list(kvs) + [("general.alignment", U32, alignment)]
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kvs))
    for k, t, v in kvs:
        head += _str(k) + struct.pack("<I", t) + _value(t, v)
    data = b""
    table = b""
    for name, dims, ttype, payload in tensors:
        data += b"\0" * (-len(data) % alignment)
        table += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        table += struct.pack("<IQ", ttype, len(data))
        data += bytes(payload)
    head += table
    if pad_after_table:
        head += b"\0" * (-len(head) % alignment)
    with open(path, "wb") as fh:
        fh.write(head + data)


def moe_block_tensors(blk: int, router: np.ndarray, corr, gate, up, down, gate_sh, up_sh, down_sh, H: int, I: int,
                      E: int, router_type: int = 0):
    """The tensors Model::moe_forward reads for block `blk`, GGUF shapes (ne order)."""
    if router_type == 0:
        rbytes = np.ascontiguousarray(router, np.float32).tobytes()
    elif router_type == 1:
        rbytes = np.ascontiguousarray(router, np.float16).tobytes()
    else:  # bf16: top half of the fp32 bits (values chosen exactly representable)
        rbytes = (np.ascontiguousarray(router, np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
    p = f"blk.{blk}."
    out = [(p + "ffn_gate_inp.weight", [H, E], router_type, rbytes)]
    if corr is not None:
        out.append((p + "exp_probs_b.bias", [E], 0, np.ascontiguousarray(corr, np.float32).tobytes()))
    out += [(p + "ffn_gate_exps.weight", [H, I, E], 18, gate), (p + "ffn_up_exps.weight", [H, I, E], 18, up),
            (p + "ffn_down_exps.weight", [I, H, E], 18, down)]
    if gate_sh is not None:
        out += [(p + "ffn_gate_shexp.weight", [H, I], 18, gate_sh), (p + "ffn_up_shexp.weight", [H, I], 18, up_sh),
                (p + "ffn_down_shexp.weight", [I, H], 18, down_sh)]
    return out


def moe_metadata(arch: str, H: int, I: int, E: int, K: int, n_shared: int = 1, scale: float = 2.5,
                 norm: bool = True, limit: float = 10.0, gating: int = 2):
    a = arch + "."
    return [("general.architecture", STRING, arch), (a + "embedding_length", U32, H),
            (a + "expert_feed_forward_length", U32, I), (a + "expert_count", U32, E),
            (a + "expert_used_count", U32, K), (a + "expert_shared_count", U32, n_shared),
            (a + "expert_weights_scale", F32, scale), (a + "expert_weights_norm", BOOL, int(norm)),
            (a + "expert_gating_func", U32, gating), (a + "swiglu_clamp_exp", ARRAY, (F32, [limit, limit]))]
