"""Benchmark of the MoE decode hot path on B200.

Workload (default): Qwen2.5-0.5B-shaped synthetic MoE (dim 896, 24 layers,
14 heads, vocab 151936, 8 experts top-2, int4 group 32, weights N(0, 0.02)
seed 1), batch 1, a 512-token uniform-random prompt (numpy default_rng(1))
prefilled token by token as the reference does, then 512 greedy tokens.
One step = one such generate call.

  value      decode tok/s: decoded tokens / decode-phase device time (CUDA
             events on the engine's stream), weights resident in HBM.
  e2e        decode tok/s through the public API (chalot_generate via
             Engine.generate) with the prompt in host memory and the tokens
             copied back: decoded tokens / (wall time of the call - its
             device prefill time), i.e. every host<->device copy, launch and
             sync of the call is charged to decoding.
  roofline   the MoE expert GEMV (gate/up + SwiGLU kernel and down + combine
             kernel of the top-2 experts), timed with CUDA events over the
             24 layers' distinct experts: algorithmic bytes = 2 experts x
             8,171,520 B per layer, against the measured HBM copy bandwidth.
  cpu_baseline  the CPU restatement of the reference (oracle/), 1 thread +
             one thread per selected expert as the reference's rayon use,
             timing decode forwards at positions 512.. (a bounded sample).

Multi-GPU: batch-1 decode does not shard (each forward depends on the last),
so --gpus N runs N independent replicas, one per rank, and reports the total
tok/s ("scaling": "weak"). Rank 0 prints one JSON line.

--impl reference times the reference's CPU path (the oracle restatement, all
host threads) on the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_LEN = 512
NEW_TOKENS = 512
KERNELS_PER_LAYER = 6  # qkv, attn scores, attn softmax+PV, o-proj + routing, gate/up, down


def model_dir() -> str:
    return os.environ.get("CHALOT_MODEL_DIR", os.path.join(tempfile.gettempdir(), "chalot_models"))


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class Clocks:
    """Samples nvidia-smi during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.p = None
        self.path = os.path.join(tempfile.gettempdir(), f"chalot_clocks_{os.getpid()}.csv")

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-i", str(self.index), "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()
            self.f.close()

    def summary(self) -> dict:
        if not self.p or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch.distributed as dist
        # gloo for the host-side timing reductions, NCCL for the expert-parallel exchange
        dist.init_process_group("cpu:gloo,cuda:nccl", timeout=datetime.timedelta(seconds=240))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def allmax(ws, v: float) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def prepare_model(ws, rank) -> str:
    import chalot_c1_b200 as cb
    path = None
    if rank == 0:
        path = cb.ensure_shape(model_dir(), "qwen")
    barrier(ws)
    if path is None:
        path = cb.ensure_shape(model_dir(), "qwen")
    return path


def cpu_sample(path: str, threads: int, n_tokens: int = 4, start: int = 512):
    """Times `n_tokens` reference-path forwards at positions start.. on the
    host (KV positions [0, start) filled with seeded values)."""
    from oracle import oracle as orc
    e = orc.OracleEngine(path, threads=threads)
    e.fill_kv_random(start)
    e.forward(1, start)  # warm the page cache
    t0 = time.perf_counter()
    for i in range(n_tokens):
        e.forward(100 + i, start + 1 + i)
    dt = time.perf_counter() - t0
    e.close()
    return n_tokens / dt, dt


def run_reference(args, ws, rank):
    if rank != 0:
        return
    import numpy as np  # noqa: F401

    from chalot_c1_b200.myai import SHAPES  # shape constants only: the CUDA library stays unloaded
    from oracle import oracle as orc
    orc.build()
    # the model file through the oracle's copy of the writer (the same bytes the
    # library writes), so this CPU-only process never loads the CUDA library
    path = orc.ensure_model(model_dir(), "qwen", SHAPES["qwen"])
    threads = orc.hw_threads()
    for _ in range(args.warmup):
        cpu_sample(path, threads, n_tokens=1)
    vals = []
    for _ in range(args.steps):
        v, _dt = cpu_sample(path, threads, n_tokens=16)
        vals.append(v)
    value = statistics.mean(vals)
    line = {
        "impl": "reference", "metric": "decode tok/s", "value": value, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 16 / value * 1000, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8/int4 weights, f32 activations", "data": "synthetic",
        "config": {"workload": "qwen2.5-0.5b-shaped MoE decode, batch 1, 512 prompt + 512 greedy",
                   "sample": "16 decode forwards per step at positions 513-528"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": "16 decode forwards per step at positions 513-528, KV [0,512) filled"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, ws, rank, local):
    import numpy as np
    import torch

    import chalot_c1_b200 as cb
    from chalot_c1_b200 import build as b
    b.build()
    torch.cuda.set_device(local)
    path = prepare_model(ws, rank)
    eng = cb.Engine.load(path, device=local)
    cfg = eng.config
    prompt = np.random.default_rng(1).integers(0, cfg["vocab_size"], PROMPT_LEN).tolist()
    for _ in range(args.warmup):
        eng.generate(prompt, NEW_TOKENS)
    # dominant kernel: expert GEMV over the layers' experts
    moe_ms, moe_bytes = eng.bench_moe_layers(reps=10)
    barrier(ws)
    torch.cuda.synchronize()
    dev_decode_ms, dev_prefill_ms, wall, n_dec = 0.0, 0.0, 0.0, 0
    toks = None
    with Clocks(local) as clk:
        t_all = time.perf_counter()
        for _ in range(args.steps):
            t0 = time.perf_counter()
            toks = eng.generate(prompt, NEW_TOKENS)
            wall += time.perf_counter() - t0
            t = eng.last_timing()
            dev_decode_ms += t["decode_ms"]
            dev_prefill_ms += t["prefill_ms"]
            n_dec += t["n_decode"]
        t_all = time.perf_counter() - t_all
        moe_ms2, _ = eng.bench_moe_layers(reps=10)
    torch.cuda.synchronize()
    barrier(ws)
    clocks = clk.summary()
    ep_res = bench_moe_ep(ws, rank) if ws > 1 else None
    bep = None
    if ws > 1:
        try:
            bep = bench_batch_ep(ws, rank, local)
        except Exception as ex:  # reported in the line; every rank still takes the reductions below
            bep = {"dt": float("nan"), "decode_steps": 0, "error": str(ex)[:300]}
    bep_dt = allmax(ws, bep["dt"]) if ws > 1 else None
    # every reduction runs on every rank, before rank 0 alone builds the line
    decode_s = allmax(ws, dev_decode_ms / 1000.0)
    prefill_s = allmax(ws, dev_prefill_ms / 1000.0)
    e2e_s = allmax(ws, wall - dev_prefill_ms / 1000.0)
    step_s = allmax(ws, t_all / args.steps)
    moe_ms = min(moe_ms, moe_ms2)
    if rank != 0:
        return
    pk = peaks()
    achieved = moe_bytes / (moe_ms * 1e-3) / 1e9
    prof = os.path.join(ROOT, "profiles", "moe_expert_gemv_traffic.json")
    traffic = json.load(open(prof))["bytes_per_layer"] if os.path.exists(prof) else None
    cpu_v, cpu_dt = cpu_sample(path, 0, n_tokens=48)
    from oracle import oracle as orc
    value = n_dec * ws / decode_s
    fwd = (PROMPT_LEN + NEW_TOKENS) * args.steps
    line = {
        "metric": "decode tok/s", "value": value, "unit": "tok/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1000.0,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8/int4 weights (dp4a int32 dots), f32 activations", "data": "synthetic",
        "config": {"workload": "qwen2.5-0.5b-shaped MoE decode (d896 L24 H14 V151936 E8 top-2 g32), "
                               "batch 1, 512-token prompt prefilled token by token + 512 greedy tokens",
                   "replicas": ws, "l2": "inputs larger than L2: 607 MB of weights streamed per token",
                   "prefill_tok_s": PROMPT_LEN * args.steps * ws / prefill_s,
                   "moe_layer_ms": moe_ms, "tokens_checksum": int(np.asarray(toks, np.uint64).sum())},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"], "traffic": traffic,
                     "kernel": "expert GEMV: k_gateup + k_down, 2 experts x 8,171,520 B per layer",
                     "peak_source": pk["source"]},
        "cpu_baseline": {"value": cpu_v, "unit": "tok/s", "cores": 1, "kind": "port",
                         "sample": f"48 decode forwards at positions 513-560 ({cpu_dt:.2f} s), "
                                   f"1 thread + 1 thread per selected expert, of "
                                   f"{orc.hw_threads()} host threads"},
        "e2e": {"value": n_dec * ws / e2e_s, "unit": "tok/s",
                "h2d_bytes_per_step": PROMPT_LEN * 4 + 32, "d2h_bytes_per_step": (PROMPT_LEN + NEW_TOKENS) * 4},
        "gpu_launches": fwd * ws * (1 + cfg["n_layers"] * KERNELS_PER_LAYER + 2),
        "clocks": clocks,
    }
    if ep_res is not None:
        line["moe_layer_prefill_ep"] = dict(ep_res, workload="expert-parallel MoE layer prefill over NVLink peer memory, "
                                            "4096 tokens per rank, experts e on rank e % n_gpus", scaling="weak")
    if bep is not None and "error" in bep:
        line["batch_decode_ep"] = {"error": bep["error"]}
    elif bep is not None:
        line["batch_decode_ep"] = {
            "workload": "1B-class MoE (d2048 L16 E16 top-2) batched decode, 64 sequences after 256-token "
                        "prompts split over the ranks, experts e on rank e % n_gpus, token rows over NCCL",
            "tok_s": BT_SEQS * bep["decode_steps"] / bep_dt, "ms_per_step": bep_dt / bep["decode_steps"] * 1000,
            "scaling": "strong", "parallelism": f"ep{ws}"}
    eng.close()
    if ws == 1:
        td = bench_tiny()
        line["tiny_decode"] = td
        mo = bench_moe_prefill(reps=10, warmup=3, cpu_tokens=1024)
        try:  # measured int8 tensor-core peak of this GPU (tcgen05.mma.kind::i8 stream)
            from chalot_c1_b200 import ops
            i8 = ops.probe_int8_mma()
            i8_peak, i8_src = i8["tops"], "measured (int8 MMA probe, 1 CTA/SM, M128xN256xK32 from smem)"
        except Exception as ex:
            i8_peak, i8_src = 4500.0, f"nominal dense int8 (probe failed: {str(ex)[:80]})"
        line["moe_layer_prefill"] = {
            "workload": "single MoE layer, 4096 tokens N(0,1) at dim 896, router 896->8, experts int4 g32 "
                        "SwiGLU 896->4864->896, top-2 (tensor-core path)",
            "tok_s": mo["tok_s"], "ms": mo["ms"], "e2e_tok_s": mo["e2e_tok_s"],
            "roofline": {"bound": "cuda-core f32 group epilogue (exact per-group order); int8 tensor ops",
                         "achieved": mo["tops"], "unit": "TOP/s", "peak": i8_peak,
                         "peak_source": i8_src, "frac": mo["tops"] / i8_peak, "nominal_peak": 4500.0},
            "cpu_baseline": mo.get("cpu")}
        bt = bench_batch(decode_steps=32, warmup=3)
        line["batch_decode"] = {
            "workload": "1B-class MoE (d2048 L16 H16 V32000 E16 top-2 g32) batched decode, 64 sequences after "
                        "256-token prompts, one KV slot each, 32 decode steps of 64 tokens",
            "tok_s": bt["tok_s"], "ms_per_step": bt["ms_per_step"],
            "e2e": {"value": bt["e2e_tok_s"], "unit": "tok/s", "h2d_bytes_per_step": BT_SEQS * 12,
                    "d2h_bytes_per_step": BT_SEQS * 4},
            "roofline": {"bound": "hbm", "achieved": bt["gbs"], "unit": "GB/s", "peak": pk["hbm_gbs"],
                         "frac": bt["gbs"] / pk["hbm_gbs"], "peak_source": pk["source"],
                         "bytes_per_step": bt["bytes_per_step"],
                         "bytes": "all 16 experts x 16 layers + dense weights + f32 K/V of 64 sequences"},
            "served": bt["served"],
            "cpu_baseline": bt["cpu_baseline"]}
        pg = bench_paged(reps=5, warmup=3)
        cpu_tok_s, cpu_sample_s = paged_cpu_sample()
        line["paged_kv_attention"] = {
            "workload": "24 layers of decode-step attention, 32 sequences x 8192 cached tokens, pages of 16, "
                        "14 heads x 64, int8 K/V per (page, K|V, head)",
            "tok_s": pg["tok_s"], "ms": pg["ms"], "e2e_tok_s": pg["e2e_tok_s"],
            "roofline": {"bound": "hbm", "achieved": pg["gbs"], "unit": "GB/s", "peak": pk["hbm_gbs"],
                         "frac": pg["gbs"] / pk["hbm_gbs"], "peak_source": pk["source"],
                         "bytes_per_step": pg["kv_gb"] * 1e9},
            "cpu_baseline": {"value": cpu_tok_s, "unit": "tok/s", "cores": orc.hw_threads(), "kind": "port",
                             "sample": cpu_sample_s}}
    print(json.dumps(line), flush=True)


def bench_tiny() -> dict:
    """Config 1: the tiny MoE (d256 L4 E8 top-2 g32, seed 0), a 32-token
    prompt (numpy seed 0) and 128 greedy tokens. The weights (19 MB) sit in L2,
    so this is a latency figure: device decode time per token."""
    import numpy as np

    import chalot_c1_b200 as cb
    path = cb.ensure_shape(model_dir(), "tiny")
    eng = cb.Engine.load(path)
    prompt = np.random.default_rng(0).integers(0, 4096, 32).tolist()
    for _ in range(3):
        eng.generate(prompt, 128)
    dec, n, wall_dec = 0.0, 0, 0.0
    for _ in range(5):
        t0 = time.perf_counter()
        eng.generate(prompt, 128)  # host prompt in, host tokens out
        wall = time.perf_counter() - t0
        t = eng.last_timing()
        dec += t["decode_ms"]
        n += t["n_decode"]
        wall_dec += wall - t["prefill_ms"] / 1000.0  # copies, launches and syncs charged to decoding
    eng.close()
    from oracle import oracle as orc
    o = orc.OracleEngine(path, threads=0)
    t0 = time.perf_counter()
    o.generate(prompt, 128)
    cdt = time.perf_counter() - t0
    o.close()
    return {"workload": "tiny MoE d256 L4 E8, 32-token prompt + 128 greedy tokens", "tok_s": n / (dec / 1000),
            "us_per_token": dec * 1000 / n,
            "e2e": {"value": n / wall_dec, "unit": "tok/s", "h2d_bytes_per_step": 32 * 4 + 32,
                    "d2h_bytes_per_step": (32 + 128) * 4},
            "cpu_baseline": {"value": 128 / cdt, "unit": "tok/s (prompt + 128 tokens)", "cores": 1, "kind": "port",
                             "sample": f"one generate of 32 + 128 tokens ({cdt:.2f} s)"}}


def paged_cpu_sample():
    """The oracle's paged attention on the host: 2 sequences x 8192 tokens,
    one layer, all host threads; returned as tok/s of a 24-layer step."""
    import numpy as np
    from oracle import oracle as orc
    rng = np.random.default_rng(5)
    P, H, hd, L = PG_P, PG_H, PG_HD, PG_TOK
    npg = 2 * L // P
    data = rng.integers(-127, 128, (npg, 2, H, P, hd)).astype(np.int8)
    sc = rng.uniform(0.01, 0.03, (npg, 2, H)).astype(np.float32)
    table = np.arange(npg, dtype=np.int32).reshape(2, L // P)
    q = rng.standard_normal((2, H, hd), dtype=np.float32)
    t0, n = time.perf_counter(), 0
    while time.perf_counter() - t0 < 8.0:  # a bounded sample: about 8 s of host work
        orc.paged_attention(data, sc, table, [L, L], P, H, hd, q, threads=orc.hw_threads())
        n += 1
    dt = (time.perf_counter() - t0) / n
    return 2 / (dt * PG_LAYERS), (f"{n} runs of 2 sequences x 8192 tokens, 1 layer ({dt * 1e3:.1f} ms each), "
                                  f"scaled to a 24-layer step")


def bench_moe_ep(ws: int, rank: int, reps: int = 10, warmup: int = 3) -> dict:
    """Expert-parallel MoE layer prefill (chalot_moe_layer_ep: tokens to the
    experts and back over NVLink peer memory): every rank holds 4096 tokens
    (weak scaling) and experts e % ws == rank of the Qwen-shaped layer. Device
    time per call (CUDA events on the calling stream), max over ranks."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from chalot_c1_b200 import ep, moe
    layer = moe.synthetic_moe_layer(MOE_DIM, MOE_H, MOE_E, MOE_K, 32, seed=3)
    x = torch.from_numpy(np.random.default_rng(100 + rank).standard_normal((MOE_T, MOE_DIM),
                                                                           dtype=np.float32)).cuda()
    pl = ep.PeerExpertLayer(layer, rank, ws, max_tokens=MOE_T)
    try:
        for _ in range(warmup):
            pl(x)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            pl(x)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
    finally:
        pl.close()
    ms = allmax(ws, ms)
    return {"tokens_per_rank": MOE_T, "ms": ms, "tok_s": MOE_T * ws / (ms * 1e-3),
            "tops": MOE_OPS * ws / (ms * 1e-3) / 1e12,
            "exchange": "int8 rows to the experts and f32 outputs back by NVLink peer stores in "
                        "chalot_moe_layer_ep (counts on the device, no host round trip)"}


def run_profile(args):
    """A short decode for profilers: 32 prompt tokens + 8 new tokens on the
    Qwen-shaped model (40 forwards, 147 kernel launches each: embed, 6 per
    layer, lm_head, advance), run twice; the second run is the one to capture
    (skip the first 5880 launches)."""
    import numpy as np

    import chalot_c1_b200 as cb
    path = prepare_model(1, 0)
    eng = cb.Engine.load(path)
    prompt = np.random.default_rng(1).integers(0, eng.config["vocab_size"], 32).tolist()
    for _ in range(2):
        toks = eng.generate(prompt, 8)
    print(json.dumps({"profile_tokens": toks}))
    for pos in (40, 768):  # per-kernel device times (no programmatic overlap)
        prof = eng.profile_forward(100, pos)
        print(json.dumps({"pos": pos, "total_ms": sum(prof.values()),
                          "per_kind_us": {k: round(v * 1000, 2) for k, v in prof.items()}}))
    eng.close()


MOE_T, MOE_DIM, MOE_H, MOE_E, MOE_K = 4096, 896, 4864, 8, 2
# int dot work of one layer call: T tokens x top-2 x (gate+up+down = 3 x dim x H) MACs x 2
MOE_OPS = MOE_T * MOE_K * 3 * MOE_DIM * MOE_H * 2


def bench_moe_prefill(reps: int = 10, warmup: int = 3, path: str | None = None,
                      cpu_tokens: int = 0) -> dict:
    """Single MoE layer prefill: 4096 tokens of N(0,1) activations (seed 3)
    through chalot_moe_layer with the Qwen-shaped layer (router 896->8
    N(0,0.02), experts int4 g32 SwiGLU 896->4864->896, top-2). Device time
    by CUDA events around each call (inputs resident), plus an end-to-end
    time with the activations copied in from pinned host memory and the
    output copied back."""
    import numpy as np
    import torch
    from chalot_c1_b200 import moe
    old = os.environ.get("CHALOT_MOE_PATH")
    if path:
        os.environ["CHALOT_MOE_PATH"] = path
    try:
        layer = moe.synthetic_moe_layer(MOE_DIM, MOE_H, MOE_E, MOE_K, 32, seed=3)
        xh = np.random.default_rng(3).standard_normal((MOE_T, MOE_DIM), dtype=np.float32)
        dev = moe.MoeLayer(layer, MOE_T)
        x = torch.from_numpy(xh).cuda()
        out = torch.empty((MOE_T, MOE_DIM), dtype=torch.float32, device="cuda")
        x_pin = torch.from_numpy(xh).pin_memory()
        out_pin = torch.empty((MOE_T, MOE_DIM), dtype=torch.float32).pin_memory()
        for _ in range(warmup):
            dev(x, out=out)
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * reps)]
        for i in range(reps):
            ev[2 * i].record()
            dev(x, out=out)
            ev[2 * i + 1].record()
        torch.cuda.synchronize()
        ms = statistics.median(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(reps))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            x.copy_(x_pin, non_blocking=True)
            dev(x, out=out)
            out_pin.copy_(out, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / reps
        res = {"tokens": MOE_T, "ms": ms, "tok_s": MOE_T / (ms * 1e-3),
               "tops": MOE_OPS / (ms * 1e-3) / 1e12, "e2e_ms": e2e_ms,
               "e2e_tok_s": MOE_T / (e2e_ms * 1e-3),
               "path": os.environ.get("CHALOT_MOE_PATH", "auto")}
        if cpu_tokens:
            from oracle import oracle as orc
            blob = layer.layer_bytes()
            t0, n = time.perf_counter(), 0
            while time.perf_counter() - t0 < 8.0:  # a bounded sample: about 8 s of host work
                orc.moe_forward(xh[:cpu_tokens], blob, MOE_DIM, MOE_H, MOE_E, MOE_K, 32, threads=orc.hw_threads())
                n += 1
            dt = time.perf_counter() - t0
            res["cpu"] = {"tok_s": n * cpu_tokens / dt, "cores": orc.hw_threads(), "kind": "port",
                          "sample": f"{n} x {cpu_tokens} tokens ({dt:.1f} s)"}
        return res
    finally:
        if path:
            if old is None:
                os.environ.pop("CHALOT_MOE_PATH", None)
            else:
                os.environ["CHALOT_MOE_PATH"] = old


PG_SEQ, PG_TOK, PG_P, PG_H, PG_HD, PG_LAYERS = 32, 8192, 16, 14, 64, 24


def bench_paged(reps: int = 5, warmup: int = 3, layers: int = PG_LAYERS) -> dict:
    """Long-context paged int8 KV attention: 32 sequences x 8192 cached tokens,
    pages of 16 tokens, 14 heads of 64; K/V ~ N(0,1) (torch generator seed 5)
    quantized per (page, K|V, head); queries ~ N(0,1). One step = decode-step
    attention of all sequences in each of 24 layers (one pool per layer).
    The pools (11.3 GB) are far larger than L2, so no flush is needed."""
    import numpy as np
    import torch
    from chalot_c1_b200 import paged
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    pages_per_seq = PG_TOK // PG_P
    n_pages = PG_SEQ * pages_per_seq
    pools = []
    chunk = 2048
    for _ in range(layers):
        pool = paged.PagedKVPool(n_pages, PG_P, PG_H, PG_HD)
        for c0 in range(0, n_pages, chunk):
            n = min(chunk, n_pages - c0)
            k = torch.randn((n, PG_P, PG_H, PG_HD), generator=g, device="cuda")
            v = torch.randn((n, PG_P, PG_H, PG_HD), generator=g, device="cuda")
            pool.store(torch.arange(c0, c0 + n, dtype=torch.int32, device="cuda"), k, v)
        pools.append(pool)
        del k, v
    # sequence s owns a shuffled set of pages (numpy seed 5)
    perm = np.random.default_rng(5).permutation(n_pages).astype(np.int32).reshape(PG_SEQ, pages_per_seq)
    table = torch.from_numpy(perm).cuda()
    lens = torch.full((PG_SEQ,), PG_TOK, dtype=torch.int32, device="cuda")
    q = torch.randn((layers, PG_SEQ, PG_H, PG_HD), generator=g, device="cuda")
    out = torch.empty_like(q)
    for p in pools:
        p.workspace(PG_SEQ, pages_per_seq)

    def step():
        for li, p in enumerate(pools):
            p.attention(q[li], table, lens, out=out[li])

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in evs:
        a.record()
        step()
        b.record()
    torch.cuda.synchronize()
    ms = statistics.median(a.elapsed_time(b) for a, b in evs)
    kv_bytes = layers * n_pages * (pools[0].page_bytes + 2 * PG_H * 4)
    q_pin = q.cpu().pin_memory()
    out_pin = torch.empty(out.shape, dtype=torch.float32).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        q.copy_(q_pin, non_blocking=True)
        step()
        out_pin.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / reps
    return {"seqs": PG_SEQ, "tokens": PG_TOK, "layers": layers, "ms": ms,
            "kv_gb": kv_bytes / 1e9, "gbs": kv_bytes / (ms * 1e-3) / 1e9, "e2e_ms": e2e_ms,
            "tok_s": PG_SEQ / (ms * 1e-3), "e2e_tok_s": PG_SEQ / (e2e_ms * 1e-3)}


def run_paged(args):
    print(json.dumps(bench_paged(reps=args.steps, warmup=args.warmup, layers=args.paged_layers)), flush=True)


BT_SEQS, BT_PROMPT, BT_NEW = 64, 256, 256


def bench_batch(decode_steps: int = 64, warmup: int = 3, cpu: bool = True) -> dict:
    """Batched decode of the 1B-class MoE (d2048 L16 H16 V32000 E16 top-2
    g32, seed 2): 64 sequences with 256-token prompts (numpy seed 2) prefilled
    together, position by position, then decoded together. `decode_steps`
    batched decode forwards (64 tokens each) after the prompt: device time
    from CUDA events on the engine's stream (chalot_last_timing), and the
    end-to-end wall time of the chalot_forward_batch calls with host tokens in
    and out. Roofline: algorithmic HBM bytes of a step (every expert of every
    layer, which 64 tokens x top-2 over 16 experts touch; the dense weights;
    the f32 K/V rows the 64 sequences attend over) per device second."""
    import numpy as np
    import torch

    import chalot_c1_b200 as cb
    path = cb.ensure_shape(model_dir(), "1b")
    eng = cb.Engine.load(path)
    cfg = eng.config
    V, L, D, E = cfg["vocab_size"], cfg["n_layers"], cfg["dim"], cfg["n_experts"]
    prompts = np.random.default_rng(2).integers(0, V, (BT_SEQS, BT_PROMPT))
    eng.reserve_batch(BT_SEQS)
    slots = list(range(BT_SEQS))
    nxt = None
    for p in range(BT_PROMPT):
        nxt = eng.forward_batch(slots, prompts[:, p].tolist(), [p] * BT_SEQS)
    pos = BT_PROMPT
    for _ in range(warmup):
        nxt = eng.forward_batch(slots, nxt, [pos] * BT_SEQS)
        pos += 1
    torch.cuda.synchronize()
    dev_ms, kv_bytes, pos0 = 0.0, 0.0, pos
    t0 = time.perf_counter()
    for _ in range(decode_steps):
        nxt = eng.forward_batch(slots, nxt, [pos] * BT_SEQS)
        dev_ms += eng.last_timing()["decode_ms"]
        kv_bytes += BT_SEQS * L * (pos + 1) * D * 4 * 2
        pos += 1
    dt = time.perf_counter() - t0
    eng.close()
    # the same job served end to end by the continuous-batching scheduler on
    # a paged K/V pool: prompts submitted at once, prefilled in 64-row chunks,
    # decoded together; wall time of the whole job from submit to last token
    eng = cb.Engine.load(path)
    eng.reserve_batch_paged(BT_SEQS, n_pages=BT_SEQS * (BT_PROMPT + BT_NEW) // 16, page_tokens=16)
    sch = eng.scheduler(BT_SEQS)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    ids = [sch.submit(prompts[i].tolist(), BT_NEW) for i in range(BT_SEQS)]
    sch.run()
    sched_s = time.perf_counter() - t1
    n_gen = sum(len(sch.poll(i)[0]) for i in ids)
    sch.close()
    expert_bytes = cfg["expert_bytes"]
    dense = cfg["total_bytes"] - L * E * expert_bytes - V * (D + 4)  # all but the experts and the embedding table
    step_bytes = L * E * expert_bytes + dense + kv_bytes / decode_steps
    eng.close()
    served = {"tok_s": n_gen / sched_s, "seconds": sched_s, "generated": n_gen,
              "workload": f"{BT_SEQS} sequences x ({BT_PROMPT}-token prompt + {BT_NEW} greedy tokens) through "
                          "chalot_sched (continuous batching, 64 rows per forward, chunked prefill) on a paged "
                          "f32 K/V pool of 16-token pages; wall time from submit to the last token"}
    res = {"seqs": BT_SEQS, "prompt": BT_PROMPT, "decode_steps": decode_steps, "positions": [pos0, pos - 1],
           "ms_per_step": dev_ms / decode_steps, "tok_s": BT_SEQS * decode_steps / (dev_ms / 1000.0),
           "e2e_tok_s": BT_SEQS * decode_steps / dt, "e2e_ms_per_step": dt / decode_steps * 1000,
           "bytes_per_step": step_bytes, "gbs": step_bytes / (dev_ms / decode_steps / 1000.0) / 1e9,
           "served": served}
    if cpu:
        # the reference runs one Engine per sequence, one after another: its
        # rate is one sequence's decode rate on all host threads
        from oracle import oracle as orc
        v, cdt = cpu_sample(path, orc.hw_threads(), n_tokens=8, start=BT_PROMPT)
        res["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": orc.hw_threads(), "kind": "port",
                               "sample": f"8 decode forwards of one sequence at positions 257-264 ({cdt:.1f} s); "
                                         "the reference decodes the 64 sequences one after another"}
    return res


def bench_batch_ep(ws: int, rank: int, local: int, decode_steps: int = 16, warmup: int = 2) -> dict:
    """The batched decode of bench_batch, expert-parallel over the ws ranks:
    each rank decodes BT_SEQS/ws of the 64 sequences (the 64-sequence job split
    over the group: strong scaling) on its GPU, its engine computing the
    experts e with e % ws == rank and exchanging token rows over NCCL at every
    MoE layer. Returns this rank's decode wall time; the caller takes the max
    over ranks."""
    import numpy as np
    import torch

    import chalot_c1_b200 as cb
    torch.cuda.set_device(local)
    if rank == 0:
        cb.ensure_shape(model_dir(), "1b")  # written once, by rank 0
    barrier(ws)
    path = cb.ensure_shape(model_dir(), "1b")
    eng = cb.Engine.load(path, device=local)
    try:
        eng.attach_ep_nccl(rank, ws)
        V = eng.config["vocab_size"]
        prompts = np.random.default_rng(2).integers(0, V, (BT_SEQS, BT_PROMPT))
        mine = list(range(rank, BT_SEQS, ws))  # the sequences of this rank
        eng.reserve_batch(-(-BT_SEQS // ws))
        slots = list(range(len(mine)))
        nxt = None
        for p in range(BT_PROMPT):
            nxt = eng.forward_batch(slots, prompts[mine, p].tolist(), [p] * len(mine))
        pos = BT_PROMPT
        for _ in range(warmup):
            nxt = eng.forward_batch(slots, nxt, [pos] * len(mine))
            pos += 1
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(decode_steps):
            nxt = eng.forward_batch(slots, nxt, [pos] * len(mine))
            pos += 1
        dt = time.perf_counter() - t0
        eng.detach_ep()
    finally:
        eng.close()
    return {"dt": dt, "decode_steps": decode_steps}


def run_batch(args):
    ws, rank, local = dist_setup()
    try:
        if ws == 1:
            print(json.dumps(bench_batch(decode_steps=max(args.steps, 8), warmup=args.warmup)), flush=True)
            return
        r = bench_batch_ep(ws, rank, local, decode_steps=max(args.steps, 8), warmup=args.warmup)
        dt = allmax(ws, r["dt"])
        if rank == 0:
            print(json.dumps({"seqs": BT_SEQS, "prompt": BT_PROMPT, "n_gpus": ws, "decode_steps": r["decode_steps"],
                              "ms_per_step": dt / r["decode_steps"] * 1000,
                              "tok_s": BT_SEQS * r["decode_steps"] / dt, "parallelism": f"ep{ws}",
                              "scaling": "strong"}), flush=True)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


def run_moe(args):
    for path in ("tc", "simt"):
        r = bench_moe_prefill(reps=args.steps, warmup=args.warmup, path=path,
                              cpu_tokens=1024 if path == "tc" else 0)
        print(json.dumps(r), flush=True)


def run_kernels(args):
    """Small cases of the batched-decode kernels, sized for ncu captures:
    one MoE layer at the 1B shape (dim 2048, hidden 5632, 16 experts, top-2)
    for 64 tokens through chalot_moe_layer (the few-slot expert kernels), and
    six chalot_forward_batch steps of 64 sequences of the Qwen-shaped model on
    a paged K/V pool of 128 pages (the tcgen05 dense GEMMs, the batched
    attention). Prints the layer time and the step time."""
    import numpy as np
    import torch

    import chalot_c1_b200 as cb
    from chalot_c1_b200 import moe
    layer = moe.synthetic_moe_layer(2048, 5632, 16, 2, 32, seed=2)
    x = torch.from_numpy(np.random.default_rng(5).standard_normal((64, 2048), dtype=np.float32)).cuda()
    dev = moe.MoeLayer(layer, max_tokens=64)
    for _ in range(max(args.warmup, 1)):
        out, sel, selw = dev(x)
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(max(args.steps, 1)):
        dev(x, out=out, sel=sel, selw=selw)
    en.record()
    torch.cuda.synchronize()
    layer_ms = st.elapsed_time(en) / max(args.steps, 1)
    del dev
    path = cb.ensure_shape(model_dir(), "qwen")
    e = cb.Engine.load(path)
    e.reserve_batch_paged(64, n_pages=128, page_tokens=16)
    rng = np.random.default_rng(0)
    step_ms = []
    for p in range(6):
        e.forward_batch(list(range(64)), rng.integers(0, 151936, 64).tolist(), [p] * 64)
        step_ms.append(e.last_timing()["decode_ms"])
    e.close()
    print(json.dumps({"moe_layer_1b_64tok_ms": layer_ms, "qwen_batch64_step_ms": step_ms}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="bench", choices=["bench", "profile", "moe", "paged", "batch", "kernels"])
    ap.add_argument("--paged-layers", type=int, default=PG_LAYERS,
                    help="--mode paged: layers (one 470 MB page pool each)")
    a = ap.parse_args()
    if a.mode == "profile":
        run_profile(a)
        return
    if a.mode == "moe":
        run_moe(a)
        return
    if a.mode == "paged":
        run_paged(a)
        return
    if a.mode == "batch":
        run_batch(a)
        return
    if a.mode == "kernels":
        run_kernels(a)
        return
    ws, rank, local = dist_setup()
    try:
        if a.impl == "reference":
            run_reference(a, ws, rank)
        else:
            run_ours(a, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
