"""Engine: the reference's inference API over the B200 library.

Mirrors ``Engine`` in src/model/engine.rs: ``Engine.load(path)`` (:94),
``forward(token, pos) -> int`` (:173), ``generate(tokens, max_new, sampling)``
(:497), ``sample_from_logits(sampling, history)`` (:551) and the public
``state.logits`` (state.rs:20), exposed here as ``logits()``. Errors the
reference reports as ``Err(String)`` or panics on raise ``ChalotError``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from ._capi import ModelConfig, Opts, Sampling, check, lib

GREEDY, TOP_K, TOP_P, MIN_P = 0, 1, 2, 3


@dataclass
class SamplingConfig:
    """SamplingConfig (src/model/engine.rs:37-62) plus the seed of the draws
    (0: from the clock, as the reference). The default here is greedy without
    a penalty (the reference's default is TopP with penalty 1.15)."""
    strategy: int = GREEDY
    temperature: float = 0.7
    top_k: int = 40
    top_p: float = 0.9
    min_p: float = 0.05
    repetition_penalty: float = 1.0
    repetition_window: int = 64
    stop_tokens: Sequence[int] = field(default_factory=list)
    seed: int = 0

    def _c(self):
        stops = (C.c_uint32 * max(1, len(self.stop_tokens)))(*self.stop_tokens)
        s = Sampling(self.strategy, self.temperature, self.top_k, self.top_p, self.min_p,
                     self.repetition_penalty, self.repetition_window,
                     C.cast(stops, C.POINTER(C.c_uint32)), len(self.stop_tokens), self.seed)
        return s, stops


class EpHub:
    """An in-process expert-parallel group of `world` engines (chalot_ep_hub)."""

    def __init__(self, world: int):
        self.world = world
        self._h = lib().chalot_ep_hub_create(world)
        if not self._h:
            check(-1)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().chalot_ep_hub_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


class Engine:
    def __init__(self, handle: C.c_void_p):
        self._h = handle
        self._ep = None
        self._cap = 0
        cfg = ModelConfig()
        check(lib().chalot_get_config(self._h, C.byref(cfg)))
        self.config = cfg.as_dict()

    @classmethod
    def load(cls, path: str, device: int = 0, use_cuda_graph: bool = True) -> "Engine":
        h = C.c_void_p()
        opts = Opts(device, int(use_cuda_graph))
        check(lib().chalot_load(path.encode(), C.byref(opts), C.byref(h)))
        return cls(h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().chalot_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def forward(self, token: int, pos: int) -> int:
        out = C.c_uint32()
        check(lib().chalot_forward(self._h, int(token), int(pos), C.byref(out)))
        return int(out.value)

    def logits(self) -> np.ndarray:
        v = np.empty(self.config["vocab_size"], np.float32)
        check(lib().chalot_get_logits(self._h, v.ctypes.data_as(C.c_void_p), v.size))
        return v

    def generate(self, tokens: Sequence[int], max_new: int,
                 sampling: SamplingConfig | None = None) -> list[int]:
        p = _u32(list(tokens) or [0])
        out = np.zeros(max(1, max_new), np.uint32)
        n = C.c_size_t()
        sp = None
        keep = None
        if sampling is not None:
            sp, keep = sampling._c()
        check(lib().chalot_generate(self._h, p.ctypes.data_as(C.c_void_p), len(tokens), max_new,
                                    C.byref(sp) if sp is not None else None,
                                    out.ctypes.data_as(C.c_void_p), C.byref(n)))
        del keep
        return out[: n.value].tolist()

    # ---- batched decode: many sequences, one KV slot each ----

    def reserve_batch(self, max_seqs: int) -> None:
        check(lib().chalot_batch_reserve(self._h, max_seqs))
        self._cap = max(self._cap, max_seqs)

    def reserve_batch_paged(self, max_seqs: int, n_pages: int, page_tokens: int = 16) -> None:
        """The batch with a paged f32 K/V cache (chalot_batch_reserve_paged):
        n_pages pages of page_tokens positions shared by the slots, taken as
        positions are written and returned by release_slot."""
        check(lib().chalot_batch_reserve_paged(self._h, max_seqs, n_pages, page_tokens))
        self._cap = max(self._cap, max_seqs)

    def release_slot(self, slot: int) -> None:
        """Returns a slot's K/V pages to the pool (chalot_batch_release)."""
        check(lib().chalot_batch_release(self._h, slot))

    def kv_pages(self) -> dict:
        """Pool state of a paged reserve: free, total, page_tokens (zeros for the flat cache)."""
        f, t, p = C.c_uint32(), C.c_uint32(), C.c_uint32()
        check(lib().chalot_batch_kv_pages(self._h, C.byref(f), C.byref(t), C.byref(p)))
        return {"free": f.value, "total": t.value, "page_tokens": p.value}

    def scheduler(self, max_rows: int | None = None) -> "Scheduler":
        """A continuous-batching scheduler over this engine's batch slots."""
        return Scheduler(self, max_rows or self._cap)

    # ---- expert parallelism of the batched forward ----

    def attach_ep_nccl(self, rank: int, world: int, group=None) -> None:
        """Joins an expert-parallel group of `world` engines over NCCL (one
        process per GPU). The NCCL id travels over torch.distributed (the
        default process group, or `group`), from rank 0 to the others."""
        import torch
        import torch.distributed as dist
        idb = (C.c_uint8 * 128)()
        if rank == 0:
            check(lib().chalot_ep_nccl_id(idb))
        t = torch.tensor(list(bytes(idb)), dtype=torch.uint8)
        if dist.get_backend(group) == "nccl":
            t = t.cuda()
        dist.broadcast(t, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        idb = (C.c_uint8 * 128)(*t.cpu().tolist())
        check(lib().chalot_ep_attach_nccl(self._h, rank, world, idb))
        self._ep = (rank, world)

    def attach_ep_hub(self, hub: "EpHub", rank: int) -> None:
        """Joins an in-process group (engines on threads of this process)."""
        check(lib().chalot_ep_attach_hub(self._h, hub._h, rank))
        self._ep = (rank, hub.world)

    def detach_ep(self) -> None:
        check(lib().chalot_ep_detach(self._h))
        self._ep = None

    def forward_batch(self, slots: Sequence[int], tokens: Sequence[int], positions: Sequence[int]) -> list[int]:
        """Engine::forward for several sequences at once (one token each)."""
        s, t, p = _u32(slots), _u32(tokens), _u32(positions)
        out = np.zeros(max(1, s.size), np.uint32)
        check(lib().chalot_forward_batch(self._h, s.ctypes.data_as(C.c_void_p), t.ctypes.data_as(C.c_void_p),
                                         p.ctypes.data_as(C.c_void_p), s.size, out.ctypes.data_as(C.c_void_p)))
        return out[: s.size].tolist()

    def batch_logits(self, row: int) -> np.ndarray:
        v = np.empty(self.config["vocab_size"], np.float32)
        check(lib().chalot_get_batch_logits(self._h, row, v.ctypes.data_as(C.c_void_p), v.size))
        return v

    @staticmethod
    def batch_steps(prompts: Sequence[Sequence[int]], max_new: int) -> int:
        """forward_batch calls generate_batch makes for these prompts."""
        if not prompts:
            return 0
        return max(len(list(p) or [0]) for p in prompts) + max(max_new - 1, 0)

    def generate_batch(self, prompts: Sequence[Sequence[int]], max_new: int, reserve: int | None = None,
                       steps: int | None = None) -> list[list[int]]:
        """Greedy Engine::generate (engine.rs:497-548) of every prompt at once:
        sequence i uses slot i; each call advances every sequence that still
        has a prompt token or a token to decode. Returns the new tokens.
        In an expert-parallel group every rank must make the same number of
        forward_batch calls: pass `steps` = the group's maximum of
        batch_steps(), and `reserve` = the group's common max_seqs."""
        n = len(prompts)
        self.reserve_batch(reserve or max(n, 1))
        prompts = [list(p) or [0] for p in prompts]
        nxt = [0] * n
        out = [[] for _ in range(n)]
        own = self.batch_steps(prompts, max_new)
        total = own if steps is None else steps
        if total < own:
            raise ValueError("steps is below this rank's own step count")
        for step in range(total):
            slots, toks, pos, who = [], [], [], []
            for i, p in enumerate(prompts):
                if step < len(p):
                    tok = p[step]
                elif step - len(p) < max_new - 1 and len(out[i]) < max_new:
                    tok = nxt[i]
                else:
                    continue
                slots.append(i)
                toks.append(tok)
                pos.append(step)
                who.append(i)
            if not slots and not self._ep:
                break
            res = self.forward_batch(slots, toks, pos)
            for i, r in zip(who, res):
                nxt[i] = r
                if step >= len(prompts[i]) - 1 and len(out[i]) < max_new:
                    out[i].append(r)
        return out

    def prefill_rows(self, slot: int, tokens: Sequence[int], pos0: int) -> int:
        """Runs tokens at positions pos0, pos0+1, ... of the sequence in `slot`
        as rows of chalot_forward_batch (as many per call as the batch holds);
        returns the argmax after the last token (Engine::forward over each in
        turn, engine.rs:173)."""
        if not tokens:
            raise ValueError("prefill_rows: no tokens")
        cap = self._cap
        out = None
        for i in range(0, len(tokens), cap):
            chunk = list(tokens[i:i + cap])
            out = self.forward_batch([slot] * len(chunk), chunk, range(pos0 + i, pos0 + i + len(chunk)))[-1]
        return out

    def generate_speculative(self, tokens: Sequence[int], max_new: int, draft: "Engine", k: int = 4) -> tuple:
        """Greedy generate with speculative decoding (src/model/speculative.rs:
        100-249): `draft` (a cheaper engine with the same vocabulary) proposes
        k tokens, this engine verifies all of them in one chalot_forward_batch
        over k+1 positions of the sequence, and the longest agreeing prefix
        plus this engine's own next token are kept. The reference verifies one
        candidate per forward; the tokens are this engine's greedy tokens
        either way. Uses KV slot 0 of both engines. Returns (tokens, accepted,
        proposed)."""
        if k < 1:
            raise ValueError("k must be >= 1")
        for e in (self, draft):
            e.reserve_batch(max(k + 1, e._cap or 1))
        prompt = list(tokens) or [0]
        room = self.config["max_seq_len"]
        out = [self.prefill_rows(0, prompt, 0)]
        draft.prefill_rows(0, prompt, 0)
        d_have = len(prompt)  # the draft's cache holds positions < d_have
        accepted = proposed = 0
        while len(out) < max_new:
            pos = len(prompt) + len(out) - 1  # position of out[-1]
            kk = min(k, room - 1 - pos, max_new - len(out))
            if kk < 1:
                break
            seq = prompt + out
            drafts = [draft.prefill_rows(0, seq[d_have:pos + 1], d_have)]
            for i in range(1, kk):
                drafts.append(draft.forward_batch([0], [drafts[-1]], [pos + i])[0])
            verdict = self.forward_batch([0] * (kk + 1), [out[-1]] + drafts, range(pos, pos + kk + 1))
            j = 0
            while j < kk and drafts[j] == verdict[j]:
                j += 1
            out.extend(drafts[:j] + [verdict[j]])
            accepted += j
            proposed += kk
            d_have = pos + 1 + min(j, kk - 1)
        return out[:max_new], accepted, proposed

    def sample_from_logits(self, sampling: SamplingConfig | None, history: Sequence[int]) -> int:
        h = _u32(list(history) or [0])
        tok = C.c_uint32()
        sp, keep = (sampling or SamplingConfig())._c()
        check(lib().chalot_sample_from_logits(self._h, C.byref(sp), h.ctypes.data_as(C.c_void_p),
                                              len(history), C.byref(tok)))
        del keep
        return int(tok.value)

    def last_timing(self) -> dict:
        a, b = C.c_double(), C.c_double()
        n1, n2 = C.c_uint32(), C.c_uint32()
        check(lib().chalot_last_timing(self._h, C.byref(a), C.byref(b), C.byref(n1), C.byref(n2)))
        return {"prefill_ms": a.value, "decode_ms": b.value, "n_prefill": n1.value,
                "n_decode": n2.value}

    def profile_forward(self, token: int, pos: int) -> dict:
        """Per-kernel device ms of one forward, summed by kernel kind."""
        n = 2 + 6 * self.config["n_layers"] + 1
        ms = np.zeros(n, np.float32)
        cnt = C.c_int()
        check(lib().chalot_profile_forward(self._h, token, pos, ms.ctypes.data_as(C.c_void_p), n,
                                           C.byref(cnt)))
        names = ["embed"] + ["qkv", "attn_scores", "attn_pv", "oproj_route", "gateup", "down"] * \
            self.config["n_layers"] + ["lmhead"]
        out: dict = {}
        for k, v in zip(names, ms[: cnt.value]):
            out[k] = out.get(k, 0.0) + float(v)
        return out

    def decode_trace(self):
        """Phase timestamps (ns) of the last decode step of the persistent
        kernel as an array [n_layers + 1][16] (see chalot_decode_trace), or
        None when the engine runs the multi-kernel chain."""
        n = C.c_size_t()
        rc = lib().chalot_decode_trace(self._h, None, 0, C.byref(n))
        if rc != 0:
            return None
        buf = np.zeros(n.value, np.uint64)
        check(lib().chalot_decode_trace(self._h, buf.ctypes.data_as(C.c_void_p), n.value, C.byref(n)))
        return buf.reshape(-1, 32)

    def bench_moe_layers(self, reps: int = 20) -> tuple[float, float]:
        ms, by = C.c_double(), C.c_double()
        check(lib().chalot_bench_moe_layers(self._h, reps, C.byref(ms), C.byref(by)))
        return ms.value, by.value


class Scheduler:
    """Continuous batching (chalot_sched_*): submit prompts at any time, call
    step() to run one batched forward (decoding sequences one row each,
    prefilling ones in prompt chunks, new ones admitted as slots and K/V pages
    free up), poll() each sequence's greedy tokens. Every sequence's tokens are
    those of Engine.generate on its prompt alone (engine.rs:497-548)."""

    def __init__(self, engine: Engine, max_rows: int):
        self.engine = engine
        h = C.c_void_p()
        check(lib().chalot_sched_create(engine._h, max_rows, C.byref(h)))
        self._h = h

    def submit(self, prompt: Sequence[int], max_new: int, stop: Sequence[int] = ()) -> int:
        p, st = _u32(list(prompt)), _u32(list(stop))
        i = C.c_uint64()
        check(lib().chalot_sched_submit(self._h, p.ctypes.data_as(C.c_void_p), p.size, max_new,
                                        st.ctypes.data_as(C.c_void_p) if st.size else None, st.size, C.byref(i)))
        return i.value

    def step(self) -> dict:
        r, w, n = C.c_uint32(), C.c_uint32(), C.c_uint32()
        check(lib().chalot_sched_step(self._h, C.byref(r), C.byref(w), C.byref(n)))
        return {"running": r.value, "waiting": w.value, "rows": n.value}

    def poll(self, seq_id: int, cap: int = 1 << 16) -> tuple[list[int], bool]:
        """(tokens so far, done); a done sequence is forgotten once polled."""
        buf = np.zeros(max(cap, 1), np.uint32)
        n, done = C.c_size_t(), C.c_int()
        check(lib().chalot_sched_poll(self._h, seq_id, buf.ctypes.data_as(C.c_void_p), cap, C.byref(n),
                                      C.byref(done)))
        return buf[: min(n.value, cap)].tolist(), bool(done.value)

    def run(self, max_steps: int = 1 << 30) -> None:
        """Steps until nothing runs or waits."""
        for _ in range(max_steps):
            st = self.step()
            if not st["running"] and not st["waiting"]:
                return

    def close(self) -> None:
        if self._h:
            lib().chalot_sched_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
