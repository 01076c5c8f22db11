"""Expert-parallel MoE layer: experts spread over the ranks of a process
group, tokens exchanged with all-to-alls.

Expert e lives on rank e % G. Per layer call every rank:
  1. routes its own tokens (router, softmax_top_k, quantize x to int8);
  2. orders its (token, choice) slots by destination rank, then by the
     destination's local expert (e // G), and gathers the int8 rows in that
     order;
  3. all-to-all: per-(rank, local expert) slot counts, then the int8 rows and
     their f32 scales (quantization depends only on the token, so shipping
     int8 is exact and 4x smaller than f32);
  4. runs the experts it holds on the rows it received (grouped by source,
     then expert);
  5. all-to-all: the f32 expert outputs back to their sources;
  6. combines them per token in selection order.
Every step keeps the per-token arithmetic of the expert block of
Engine::forward (src/model/engine.rs:334-401), so the result is bit-identical
to the single-GPU layer.

The steps run on a backend: ``GpuBackend`` calls the library's C ABI on CUDA
tensors (collectives over NCCL); tests use a CPU restatement backend over
gloo. ``ep_forward`` takes the collective as a function so the same code also
runs with an in-process exchange (``emulated_forward``).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from .moe import SyntheticMoeLayer


def local_experts(n_experts: int, world: int, rank: int) -> list[int]:
    """Experts held by `rank`, in local order (local index = e // world)."""
    if n_experts % world:
        raise ValueError("n_experts must be a multiple of the number of ranks")
    return [e for e in range(n_experts) if e % world == rank]


def local_blob(layer: SyntheticMoeLayer, world: int, rank: int) -> np.ndarray:
    ex = layer.expert_bytes
    return np.concatenate([layer.experts[e * ex:(e + 1) * ex] for e in local_experts(layer.n_experts, world, rank)])


class GpuBackend:
    """The EP steps on one GPU through the C ABI (device tensors)."""

    def __init__(self, layer: SyntheticMoeLayer, world: int, rank: int, device="cuda"):
        from ._capi import MoeDesc
        self.layer, self.world, self.rank, self.device = layer, world, rank, device
        self.router_w = torch.from_numpy(layer.router_w).to(device)
        self.router_b = torch.from_numpy(layer.router_b).to(device)
        self.local = torch.from_numpy(local_blob(layer, world, rank)).to(device)
        self.desc = MoeDesc(layer.dim, layer.hidden, layer.n_experts, layer.top_k, layer.group,
                            self.router_w.data_ptr(), self.router_b.data_ptr(), 0)
        self.local_desc = MoeDesc(layer.dim, layer.hidden, layer.n_experts // world, layer.top_k, layer.group,
                                  0, 0, self.local.data_ptr())
        self._ws = None

    def _s(self):
        return torch.cuda.current_stream().cuda_stream

    def route(self, x):
        from ._capi import check, lib
        T, K, d = x.shape[0], self.layer.top_k, self.layer.dim
        sel = torch.empty((T, K), dtype=torch.int32, device=self.device)
        selw = torch.empty((T, K), dtype=torch.float32, device=self.device)
        xq = torch.empty((T, d), dtype=torch.int8, device=self.device)
        xs = torch.empty((T,), dtype=torch.float32, device=self.device)
        check(lib().chalot_moe_route(C.byref(self.desc), x.data_ptr(), T, sel.data_ptr(), selw.data_ptr(),
                                     xq.data_ptr(), xs.data_ptr(), self._s()))
        return sel, selw, xq, xs

    def plan(self, sel):
        from ._capi import check, lib
        n = sel.numel()
        E = self.layer.n_experts
        order = torch.empty((n,), dtype=torch.int32, device=self.device)
        pos = torch.empty((n,), dtype=torch.int32, device=self.device)
        offs = torch.empty((E + 1,), dtype=torch.int32, device=self.device)
        check(lib().chalot_moe_plan(sel.data_ptr(), n, E, self.world, order.data_ptr(), pos.data_ptr(),
                                    offs.data_ptr(), self._s()))
        return order, pos, offs

    def gather(self, xq, xs, order):
        from ._capi import check, lib
        n, d = order.numel(), self.layer.dim
        rows = torch.empty((n, d), dtype=torch.int8, device=self.device)
        rs = torch.empty((n,), dtype=torch.float32, device=self.device)
        check(lib().chalot_moe_gather(xq.data_ptr(), xs.data_ptr(), order.data_ptr(), n, self.layer.top_k, d,
                                      rows.data_ptr(), rs.data_ptr(), self._s()))
        return rows, rs

    def experts(self, rows, rs, row_expert):
        from ._capi import check, lib
        n = rows.shape[0]
        y = torch.empty((n, self.layer.dim), dtype=torch.float32, device=self.device)
        if n == 0:
            return y
        need = lib().chalot_moe_experts_workspace_size(C.byref(self.local_desc), n)
        if need == 0:
            check(-1)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        check(lib().chalot_moe_experts(C.byref(self.local_desc), rows.data_ptr(), rs.data_ptr(),
                                       row_expert.data_ptr(), n, y.data_ptr(), self._ws.data_ptr(),
                                       self._ws.numel(), self._s()))
        return y

    def combine(self, y, pos, selw):
        from ._capi import check, lib
        T, K = selw.shape
        out = torch.empty((T, self.layer.dim), dtype=torch.float32, device=self.device)
        check(lib().chalot_moe_combine(y.data_ptr(), pos.data_ptr(), selw.data_ptr(), T, K, self.layer.dim,
                                       out.data_ptr(), self._s()))
        return out


class PeerExpertLayer:
    """chalot_moe_layer_ep: the expert-parallel layer as one library call,
    tokens moved to the experts and back with NVLink peer stores (no host
    round trip, no padding). One instance per rank (one process per GPU);
    construction all-gathers the ranks' exchange-arena handles over
    torch.distributed, and every rank must then call it in lockstep."""

    def __init__(self, layer: SyntheticMoeLayer, rank: int, world: int, max_tokens: int, group=None,
                 device="cuda"):
        import torch.distributed as dist

        from ._capi import MoeDesc, check, lib
        self.layer, self.rank, self.world, self.device = layer, rank, world, device
        self.router_w = torch.from_numpy(layer.router_w).to(device)
        self.router_b = torch.from_numpy(layer.router_b).to(device)
        self.local = torch.from_numpy(local_blob(layer, world, rank)).to(device)
        self.desc = MoeDesc(layer.dim, layer.hidden, layer.n_experts, layer.top_k, layer.group,
                            self.router_w.data_ptr(), self.router_b.data_ptr(), self.local.data_ptr())
        self._comm = C.c_void_p()
        handle = (C.c_uint8 * 64)()
        check(lib().chalot_ep_comm_create(rank, world, C.byref(self.desc), max_tokens, C.byref(self._comm), handle))
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        buf = (C.c_uint8 * (64 * world)).from_buffer_copy(b"".join(handles))
        check(lib().chalot_ep_comm_connect(self._comm, buf))

    def __call__(self, x):
        from ._capi import check, lib
        T, K = x.shape[0], self.layer.top_k
        out = torch.empty((T, self.layer.dim), dtype=torch.float32, device=self.device)
        sel = torch.empty((T, K), dtype=torch.int32, device=self.device)
        selw = torch.empty((T, K), dtype=torch.float32, device=self.device)
        check(lib().chalot_moe_layer_ep(self._comm, C.byref(self.desc), x.data_ptr() if T else None, T,
                                        out.data_ptr() if T else None, sel.data_ptr() if T else None,
                                        selw.data_ptr() if T else None, torch.cuda.current_stream().cuda_stream))
        return out, sel

    def close(self) -> None:
        from ._capi import lib
        if self._comm:
            torch.cuda.synchronize()
            lib().chalot_ep_comm_free(self._comm)
            self._comm = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _counts(offs, world: int, n_local: int):
    c = offs[1:] - offs[:-1]
    return c.reshape(world, n_local)


def _row_experts(recv_cnt, n_local: int, device):
    ids = torch.arange(n_local, dtype=torch.int32, device=device).repeat(recv_cnt.shape[0])
    return torch.repeat_interleave(ids, recv_cnt.reshape(-1).to(torch.int64))


def ep_forward(backend, x, all_to_all, world: int):
    """One expert-parallel layer call on this rank. `all_to_all(out, inp,
    out_splits, in_splits)` is the collective (torch.distributed's
    all_to_all_single signature). Returns (out [T][dim], sel [T][K])."""
    layer = backend.layer
    El = layer.n_experts // world
    sel, selw, xq, xs = backend.route(x)
    order, pos, offs = backend.plan(sel.reshape(-1))
    rows, rs = backend.gather(xq, xs, order)
    send_cnt = _counts(offs, world, El).contiguous()
    recv_cnt = torch.empty_like(send_cnt)
    all_to_all(recv_cnt, send_cnt, None, None)
    out_splits = send_cnt.sum(1).tolist()
    in_splits = recv_cnt.sum(1).tolist()
    n_in = int(sum(in_splits))
    recv_rows = torch.empty((n_in, layer.dim), dtype=torch.int8, device=rows.device)
    recv_rs = torch.empty((n_in,), dtype=torch.float32, device=rows.device)
    all_to_all(recv_rows, rows, in_splits, out_splits)
    all_to_all(recv_rs, rs, in_splits, out_splits)
    y = backend.experts(recv_rows, recv_rs, _row_experts(recv_cnt, El, rows.device))
    y_back = torch.empty((rows.shape[0], layer.dim), dtype=torch.float32, device=rows.device)
    all_to_all(y_back, y, out_splits, in_splits)
    return backend.combine(y_back, pos, selw), sel


def dist_all_to_all(group=None):
    import torch.distributed as dist

    def a2a(out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)
    return a2a


def emulated_forward(backends, xs):
    """Runs ep_forward for all ranks in one process, the all-to-alls done by
    slicing (each rank's calls in lockstep). Returns the per-rank outputs."""
    import threading
    world = len(backends)
    # a barrier-based exchange: every rank posts its send buffer, then takes its parts
    lock = threading.Condition()
    state = {"posted": {}, "round": 0, "taken": 0}

    def make(rank):
        def a2a(out, inp, out_splits, in_splits):
            with lock:
                r = state["round"]
                state["posted"][(r, rank)] = (inp, in_splits)
                lock.notify_all()
                lock.wait_for(lambda: all((r, k) in state["posted"] for k in range(world)))
            parts = []
            for src in range(world):
                sinp, ssplits = state["posted"][(r, src)]
                if ssplits is None:  # equal splits
                    n = sinp.shape[0] // world
                    parts.append(sinp[rank * n:(rank + 1) * n])
                else:
                    off = int(sum(ssplits[:rank]))
                    parts.append(sinp[off:off + int(ssplits[rank])])
            out.copy_(torch.cat(parts, 0).to(out.device))
            with lock:
                state["taken"] += 1
                if state["taken"] == world:
                    state["taken"] = 0
                    for k in range(world):
                        del state["posted"][(r, k)]
                    state["round"] += 1
                    lock.notify_all()
                else:
                    lock.wait_for(lambda: state["round"] > r)
        return a2a

    results = [None] * world
    errors = []

    def run(rank):
        try:
            results[rank] = ep_forward(backends[rank], xs[rank], make(rank), world)
        except Exception as e:  # surfaced below
            errors.append(e)
            with lock:
                lock.notify_all()

    ts = [threading.Thread(target=run, args=(k,)) for k in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    if errors:
        raise errors[0]
    return results
