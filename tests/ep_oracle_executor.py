"""Test-only executor for the expert-parallel layer: the device steps done by
the CPU oracle (oracle/), so the exchange logic runs on CPU ranks over gloo.
Never imported by the package."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle


class OracleExecutor:
    def __init__(self, layer: dict, cfg, expert_begin: int, expert_count: int):
        self.layer, self.cfg = layer, cfg
        self.lo, self.cnt = expert_begin, expert_count
        self.chk = oracle.Checker("port")
        self.shape = oracle.Shape(cfg.hidden, cfg.inter, cfg.n_experts, cfg.top_k, cfg.routed_scale,
                                  int(cfg.norm_topk), cfg.swiglu_limit)

    def empty(self, shape, dtype):
        return torch.empty(shape, dtype=dtype)

    def route(self, x):
        _, ids, w = self.chk.moe_batch(self.shape, self.layer, x.float().numpy())
        return torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(w.astype(np.float32))

    def pack(self, ids, x, world):
        # stable bucket order by expert (hence by destination rank), as gpeed_ep_pack
        n, K = ids.shape
        flat = ids.numpy().reshape(-1)
        order = np.argsort(flat, kind="stable")
        slot_of = np.empty(n * K, np.int32)
        slot_of[order] = np.arange(n * K, dtype=np.int32)
        epr = self.cfg.n_experts // world
        counts = np.bincount(flat // epr, minlength=world).astype(np.int32)
        return (x[torch.from_numpy(order // K)].contiguous(), torch.from_numpy(flat[order].astype(np.int32)),
                torch.from_numpy(counts), torch.from_numpy(slot_of.reshape(n, K)))

    def experts(self, rows, ids):
        cfg, L = self.cfg, self.layer
        H, I, E, lim = cfg.hidden, cfg.inter, cfg.n_experts, np.float32(cfg.swiglu_limit)
        X = rows.float().numpy()
        ids = ids.numpy()
        out = np.zeros((X.shape[0], H), np.float32)
        for e in np.unique(ids):
            sel = np.nonzero(ids == e)[0]
            if e == E:
                gate, up, down, rg, rd = L["gate_sh"], L["up_sh"], L["down_sh"], 0, 0
            else:
                assert self.lo <= e < self.lo + self.cnt, f"expert {e} is not held by this rank"
                gate, up, down, rg, rd = L["gate"], L["up"], L["down"], int(e) * I, int(e) * H
            g = self.chk.matmul_quant(gate, rg, H, I, X[sel])
            u = self.chk.matmul_quant(up, rg, H, I, X[sel])
            gi = np.minimum(g, lim)
            h = (gi / (np.float32(1) + np.exp(-gi))) * np.clip(u, -lim, lim)
            out[sel] = self.chk.matmul_quant(down, rd, I, H, h.astype(np.float32))
        return torch.from_numpy(out)

    def combine(self, d_rows, slot_of, w, d_shared):
        d, s, wv = d_rows.numpy(), slot_of.numpy(), w.numpy()
        y = np.zeros((s.shape[0], d.shape[1]), np.float32)
        for k in range(s.shape[1]):
            y = (y + wv[:, k:k + 1] * d[s[:, k]]).astype(np.float32)
        if d_shared is not None:
            y = (y + d_shared.numpy()).astype(np.float32)
        return torch.from_numpy(y)

    def decode_partial(self, x_all, own_tok, y_part=None):
        """gpeed_moe_decode_partial on the oracle: every token's routing, then
        this rank's share: w_k * D_k over the picks whose expert it holds, in
        pick order, plus the shared expert of own_tok."""
        ids, w = self.route(x_all)
        ids, w = ids.numpy(), w.numpy()
        n, K = ids.shape
        out = np.zeros((n, self.cfg.hidden), np.float32)
        for t in range(n):
            for k in range(K):
                e = int(ids[t, k])
                if self.lo <= e < self.lo + self.cnt:
                    d = self.experts(x_all[t:t + 1], torch.tensor([e], dtype=torch.int32)).numpy()[0]
                    out[t] = (out[t] + np.float32(w[t, k]) * d).astype(np.float32)
            if t == own_tok:
                d = self.experts(x_all[t:t + 1], torch.tensor([self.cfg.n_experts], dtype=torch.int32)).numpy()[0]
                out[t] = (out[t] + d).astype(np.float32)
        y = torch.from_numpy(out)
        if y_part is not None:
            y_part.copy_(y)
            return y_part
        return y
