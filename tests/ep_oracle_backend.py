"""CPU backend of the expert-parallel layer for gloo tests: each EP step
restated with the oracle (test infrastructure; the product's steps are the
C ABI calls of chalot_c1_b200.ep.GpuBackend)."""
import numpy as np
import torch

from chalot_c1_b200.ep import local_blob


class OracleBackend:
    def __init__(self, layer, world, rank, orc):
        self.layer, self.world, self.rank, self.orc = layer, world, rank, orc
        self.local = local_blob(layer, world, rank)

    def route(self, x):
        L, o = self.layer, self.orc
        xn = x.numpy()
        T = xn.shape[0]
        sel = np.zeros((T, L.top_k), np.int32)
        selw = np.zeros((T, L.top_k), np.float32)
        xq = np.zeros((T, L.dim), np.int8)
        xs = np.zeros((T,), np.float32)
        for t in range(T):
            logits = np.array([L.router_b[e] + o.dot_f32(L.router_w[e], xn[t]) for e in range(L.n_experts)],
                              np.float32)
            sel[t], selw[t] = o.softmax_top_k(logits, L.top_k)
            xq[t], xs[t] = o.quantize_i8(xn[t])
        return tuple(torch.from_numpy(a) for a in (sel, selw, xq, xs))

    def plan(self, sel):
        E, G = self.layer.n_experts, self.world
        e = sel.numpy().astype(np.int64)
        keys = (e % G) * (E // G) + e // G
        order = np.argsort(keys, kind="stable").astype(np.int32)
        pos = np.empty_like(order)
        pos[order] = np.arange(order.size, dtype=np.int32)
        offs = np.concatenate([[0], np.cumsum(np.bincount(keys, minlength=E))]).astype(np.int32)
        return torch.from_numpy(order), torch.from_numpy(pos), torch.from_numpy(offs)

    def gather(self, xq, xs, order):
        tok = order.numpy() // self.layer.top_k
        return torch.from_numpy(xq.numpy()[tok].copy()), torch.from_numpy(xs.numpy()[tok].copy())

    def experts(self, rows, rs, row_expert):
        L = self.layer
        if rows.shape[0] == 0:
            return torch.zeros((0, L.dim), dtype=torch.float32)
        y = self.orc.expert_rows(rows.numpy(), rs.numpy(), row_expert.numpy(), self.local, L.dim, L.hidden,
                                 L.group)
        return torch.from_numpy(y)

    def combine(self, y, pos, selw):
        yn, pn, wn = y.numpy(), pos.numpy(), selw.numpy()
        T, K = wn.shape
        acc = np.zeros((T, self.layer.dim), np.float32)
        for j in range(K):
            p = (wn[:, j, None] * yn[pn[np.arange(T) * K + j]]).astype(np.float32)
            acc = (acc + p).astype(np.float32)
        return torch.from_numpy(acc)
