#!/usr/bin/env python3
"""Decode benchmark for the B200 path: batch-1 tok/s on the Llama-3.1-8B-shape
Q4_K_M model, with the Q4_K GEMV's HBM roofline fraction.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--shape llama8b|llama70b] [--prompt P] [--kv-fill auto|tokens|synthetic]

One step = one decoded token: embed -> L layers (RMSNorm+QKV+RoPE GEMV,
Q8_0 append + split-K attention, O GEMV + residual, RMSNorm+gate/up GEMV +
SwiGLU, down GEMV + residual) -> lm_head GEMV -> first-index argmax, with the
token fed back on the device.  Weights (4.9 GB for the 8B shape, 44.4 GB for
70B) are synthetic, seeded, and generated in HBM.  The 8B shape's KV cache is
prefilled with a 512-token random prompt decoded token by token; the 70B
shape's 8192-position context is N(0,1) K/V rows quantised straight into the
Q8_0 cache (decoding 8192 prompt tokens one by one would take minutes and
times nothing different).  Weights exceed L2 (126 MB), so no flush is needed
between steps.

At --gpus N > 1 the same single sequence is decoded tensor-parallel over N
GPUs (one process per GPU; Wq/Wk/Wv/gate/up split by output rows, Wo/down by
input columns, KV heads local to a rank, output head split by vocabulary rows;
NCCL all-reduce after O and down inside the captured step; `--p2p-allreduce`
sends the partial rows straight into every rank's exchange buffer over NVLink
and lets the next GEMV sum them instead): strong scaling,
timed as the max over ranks.  Each rank generates its shard's synthetic
weights directly (same distributions, rank-seeded).
``--impl reference`` times the reference's own C implementation of the path
(oracle/_ref, compiled from the reference sources; else the oracle port) on
host cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s bs1, 8B-shape Q4_K_M; Q4_K/Q6_K GEMV HBM GB/s vs peak"
PROMPT = 512
PROMPTS = {"llama8b": 512, "llama70b": 8192}  # the context each model shape is measured at
PART_NAMES = ("rmsnorm_qkv_rope", "append_attention", "o_proj_residual", "rmsnorm_gateup_swiglu",
              "down_residual", "lm_head")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--shape", default="llama8b")
    ap.add_argument("--prompt", type=int, default=None,
                    help="KV context before the timed decode (default: 512 for the 8B shape, 8192 for 70B)")
    ap.add_argument("--kv-fill", default="auto", choices=["auto", "tokens", "synthetic"],
                    help="how the context is built: the prompt decoded token by token, or N(0,1) K/V rows "
                         "appended straight into the Q8_0 cache (auto: synthetic above 1024 positions)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--p2p-allreduce", action="store_true",
                    help="tensor parallel: the peer-memory exchange inside the GEMVs instead of NCCL all-reduce")
    ap.add_argument("--tp-allreduce", default="ll", choices=["ll", "nccl"],
                    help="tensor parallel: one-shot all-reduce kernel over NVLink peer memory with the flags in "
                         "the data words (ll, default) or NCCL's all-reduce")
    a = ap.parse_args()
    if a.prompt is None:
        a.prompt = PROMPTS.get(a.shape, PROMPT)
    if a.kv_fill == "auto":
        a.kv_fill = "synthetic" if a.prompt > 1024 else "tokens"
    return a


def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def recorded_traffic(shape: str, part: str):
    """DRAM bytes (read + write) per launch of a decode part, as one ncu
    capture of the current kernels measured them (profiles/dram_traffic.json:
    per workload and part, the bytes and the capture command), or None."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if not os.path.exists(p):
        return None
    rec = json.load(open(p)).get(shape, {}).get(part)
    if not rec:
        return None
    return {"bytes": rec["dram_bytes_per_launch"], "source": rec["capture"]}


def part_kernel(part: str) -> str:
    """The kernel that runs a decode part in the bench's weight layouts."""
    from shukuchi_b200.synth_device import TILED_DEFAULT
    proj = {"rmsnorm_qkv_rope": "qkv", "o_proj_residual": "o", "rmsnorm_gateup_swiglu": "gateup",
            "down_residual": "down", "lm_head": "output"}.get(part)
    if proj is None:
        return "attn_cluster_kernel"
    if proj in TILED_DEFAULT:
        return f"mmv_kernel (tensor-core matvec, row-tiled) {part}"
    return f"gemv_kernel (dp4a, GGUF / planar rows) {part}"


class ClockSampler:
    """nvidia-smi clocks + throttle reasons while the timed region runs."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int):
        self.dev, self.proc, self.lines = dev, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------- CPU side
def cpu_sample(steps: int, warmup: int, shape_name: str, prompt: int):
    """Reference (or oracle) CPU path on a bounded sample of the token: each
    step runs 2 of the model's L layers (forward_layer_view at the current
    position, KV prefilled to `prompt`) plus 2/L of the output-head rows; one
    token costs L/2 such steps.  Returns (tok/s, kind, sample text, per-step
    tok/s)."""
    import numpy as np
    from oracle.oracle_py import Oracle, Reference
    from shukuchi_b200 import synth

    s = synth.SHAPES[shape_name]
    f = s.n_layers / 2.0  # steps per token
    rng = np.random.default_rng(0)
    layers = [synth.make_layer(rng, s) for _ in range(2)]
    head_rows = int(round(s.n_vocab / f))
    head = synth.quant_matrix(rng, s.t_out, head_rows, s.n_embd)
    sub = synth.Model(s, layers, np.zeros(1, np.uint8), np.zeros(1, np.float32), head)
    import dataclasses
    sub.shape = dataclasses.replace(s, n_layers=2)
    hidden = rng.normal(0, 1, s.n_embd).astype(np.float32)
    kvd = s.n_kv_heads * s.head_dim
    max_seq = prompt + steps + warmup + 2
    if Reference.available():
        R = Reference()
        kind = "reference"
        h, step_fn = R.forward_layer_fn(sub, max_seq)
        kvh = R.L.ref_engine_kv(h)
        for p in range(prompt):
            kk = rng.normal(0, 1, kvd).astype(np.float32)
            for layer in range(2):
                R.L.ref_kv_append(kvh, layer, p, kk.ctypes.data, kk.ctypes.data)

        def layer_fwd(layer, pos):
            step_fn(layer, pos, hidden)

        def head_fn():
            R.matvec(s.t_out, head, hidden, head_rows, s.n_embd)
    else:
        O = Oracle(threads=1)
        kind = "port"
        ms = O.model_struct(sub)
        kv = O.kv_create(2, s.n_kv_heads, s.head_dim, max_seq)
        for p in range(prompt):
            kk = rng.normal(0, 1, kvd).astype(np.float32)
            for layer in range(2):
                O.L.orc_kv_append(kv, layer, p, kk.ctypes.data, kk.ctypes.data)
        import ctypes

        def layer_fwd(layer, pos):
            assert O.L.orc_forward_layer(ctypes.byref(ms), kv, layer, pos, hidden.ctypes.data) == 0

        def head_fn():
            O.matvec(s.t_out, head, hidden, head_rows, s.n_embd)

    pos = prompt
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        layer_fwd(0, pos)
        layer_fwd(1, pos)
        head_fn()
        dt = time.perf_counter() - t0
        np.clip(hidden, -1e4, 1e4, out=hidden)
        pos += 1
        if i >= warmup:
            times.append(dt)
    per_token = f * sum(times) / len(times)
    sample = (f"{steps} steps of 2/{s.n_layers} layers of {s.name} at positions {prompt}+ plus "
              f"{head_rows}/{s.n_vocab} output-head rows; token time = {f:g} x step time")
    return 1.0 / per_token, kind, sample, [1.0 / (f * t) for t in times]


def host_info() -> dict:
    """Cores and load of the host the CPU baseline ran on."""
    return {"host_nproc": os.cpu_count(), "host_loadavg_1m": round(os.getloadavg()[0], 2)}


PARITY_SHAPE = ("tp-hd128", 2, 1024, 8, 4, 2048, 1024)  # 2 layers, d 1024, 8/4 heads x 128, ffn 2048


def parity_check(ctx, ws, rank, local, allreduce="ll"):
    """The decode path of this run (same context, same rank layout) on a small
    synthetic model against the oracle: 5 prompt ids + 8 greedy tokens,
    greedy ids and max|dlogit| / std(logits).  Rank 0 runs the oracle; every
    rank's ids are gathered.  Returns the JSON object (rank 0) or None."""
    import numpy as np
    from shukuchi_b200 import synth
    from shukuchi_b200 import tp as tpl
    from shukuchi_b200.device_model import GpuDecoder

    shape = synth.ModelShape(*PARITY_SHAPE)
    model = synth.make_model(shape, seed=21)
    prompt = np.random.default_rng(7).integers(0, shape.n_vocab, 5).astype(np.uint32)
    n_dec = 8
    if ws > 1:
        mr, lay = tpl.shard_model(model, rank, ws)
        tp_rows = (lay.o_lo, lay.o_hi, lay.v_lo, lay.v_hi)
    else:
        mr, tp_rows = model, None
    from shukuchi_b200.synth_device import TILED_DEFAULT
    gather = None
    if ws > 1 and allreduce == "ll":
        import torch.distributed as dist

        def gather(h):
            hs = [None] * ws
            dist.all_gather_object(hs, h)
            return hs
    # the layouts and the all-reduce the timed run uses
    dec = GpuDecoder(ctx, mr, len(prompt) + n_dec + 1, device=f"cuda:{local}", tp_rows=tp_rows,
                     tiled=TILED_DEFAULT, ll_exchange=gather)
    try:
        logits = np.zeros((n_dec, shape.n_vocab), np.float32)
        ids = dec.generate(prompt, n_dec, logits)
        ctx.check()
    finally:
        dec.close()
    all_ids = [ids.tolist()]
    if ws > 1:
        import torch.distributed as dist
        all_ids = [None] * ws
        dist.all_gather_object(all_ids, ids.tolist())
    if rank != 0:
        return None
    from oracle.oracle_py import Oracle
    t_ref, l_ref = Oracle().generate(model, prompt, n_dec)
    dl = max(float(np.max(np.abs(logits[t] - l_ref[t]))) / float(np.std(l_ref[t])) for t in range(n_dec))
    return {"model": f"{shape.name} (2 layers, d 1024, 8/4 heads x 128, ffn 2048, vocab 1024), "
                     f"5 prompt + {n_dec} greedy ids vs the oracle",
            "ids_match": all(list(r) == t_ref.tolist() for r in all_ids),
            "ranks": ws, "allreduce": allreduce if ws > 1 else None, "max_dlogit_over_std": dl,
            "tolerance": 1e-2}


def workload_config(args, ws):
    from shukuchi_b200 import synth
    s = synth.SHAPES[args.shape]
    ctx = (f"after a {args.prompt}-token prompt" if args.kv_fill == "tokens" else
           f"at a {args.prompt}-position context of N(0,1) K/V rows appended to the cache")
    return {"workload": f"{s.name} Q4_K_M decode bs1 {ctx}, Q8_0 KV",
            "model": s.name, "global_batch": 1, "seq_len": args.prompt, "kv_fill": args.kv_fill,
            "parallelism": f"tp{ws}" if ws > 1 else "single",
            "l2": f"no flush: {synth.token_bytes(s) / 1e9:.1f} GB of weights per step exceed the 126 MB L2"}


def run_reference(args, ws, rank):
    if rank != 0:
        return
    v, kind, sample, per_step = cpu_sample(args.steps, args.warmup, args.shape, args.prompt)
    spread = {"min": min(per_step), "max": max(per_step), "steps": len(per_step)}
    line = {
        "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, 1),
        "impl": "reference",
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": 1, "kind": kind, "sample": sample,
                         "per_step_tok_s": spread, **host_info()},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU side
def run_ours(args, ws, rank, local):
    import torch
    import torch.distributed as dist
    from shukuchi_b200 import cuda as sc
    from shukuchi_b200 import synth
    from shukuchi_b200 import tp as tpl
    from shukuchi_b200 import synth_device
    from shukuchi_b200.synth_device import make_device_model

    torch.cuda.set_device(local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    shape = synth.SHAPES[args.shape]
    ctx = sc.Context(local)
    lay = tpl.layout(shape, rank, ws)
    lshape = tpl.local_shape(shape, lay)
    if ws > 1:
        obj = [sc.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.tp_init(rank, ws, obj[0])
    # correctness of this exact path before it is timed (small model, oracle on rank 0)
    parity = parity_check(ctx, ws, rank, local, args.tp_allreduce) if not args.p2p_allreduce else None
    wts = make_device_model(lshape, seed=1234 + rank, device=f"cuda:{local}",
                            o_rows=lay.o_hi - lay.o_lo, out_rows=lay.v_hi - lay.v_lo, ctx=ctx,
                            tiled=(synth_device.TILED_DEFAULT if not args.p2p_allreduce else False))
    total = args.prompt + 2 * (args.warmup + args.steps) + 8
    kv = sc.KvCache(ctx, lshape.n_layers, lshape.n_kv_heads, lshape.head_dim, total)
    m = sc.DeviceModel(ctx, kv, wts.desc)
    if ws > 1:
        m.set_tp_rows(lay.o_lo, lay.o_hi, lay.v_lo, lay.v_hi)
        if args.p2p_allreduce:  # all-reduce over NVLink peer memory inside the GEMVs
            hs = [None] * ws
            dist.all_gather_object(hs, m.tp_p2p_export())
            m.tp_p2p_import(hs, [(L.o_lo, L.o_hi) for L in (tpl.layout(shape, r, ws) for r in range(ws))])
        elif args.tp_allreduce == "ll":  # one-shot all-reduce kernel, flags in the data words
            hs = [None] * ws
            dist.all_gather_object(hs, m.tp_ll_export())
            m.tp_ll_import(hs)
    for i, lv in enumerate(wts.layers):
        m.set_layer(i, lv)
    stream = torch.cuda.ExternalStream(ctx.stream, device=f"cuda:{local}")

    import numpy as np
    rng = np.random.default_rng(0)  # one sequence, the same on every rank
    if args.kv_fill == "tokens":
        # prompt, token by token (the reference has no batched prefill)
        prompt = rng.integers(0, shape.n_vocab, args.prompt).astype(np.uint32)
        nxt = 0
        for i, t in enumerate(prompt):
            nxt = m.token_step(int(t), i, want_next=(i == len(prompt) - 1))
    else:
        # the context as N(0,1) K/V rows quantised into the cache (this rank's
        # KV heads), then decode from a random token
        kvd_l = lshape.n_kv_heads * lshape.head_dim
        gen = torch.Generator(device=f"cuda:{local}")
        gen.manual_seed(77 + rank)
        with torch.cuda.stream(stream):
            for layer in range(lshape.n_layers):
                for p0 in range(0, args.prompt, 2048):
                    n = min(2048, args.prompt - p0)
                    kk = torch.randn((n, kvd_l), device=f"cuda:{local}", generator=gen)
                    vv = torch.randn((n, kvd_l), device=f"cuda:{local}", generator=gen)
                    kv.append_range(layer, p0, n, kk.data_ptr(), vv.data_ptr(), stream=ctx.stream)
                    ctx.sync()
        nxt = int(rng.integers(0, shape.n_vocab))
    pos = args.prompt

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # warm-up
    m.decode_steps(nxt, pos, args.warmup)
    pos += args.warmup
    nxt = m.last_token()
    barrier()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        ev0.record(stream)
        torch.cuda.nvtx.range_push("decode")  # lets ncu --nvtx-include "decode/" pick the timed launches
        m.decode_steps(nxt, pos, args.steps)
        torch.cuda.nvtx.range_pop()
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
    ctx.check()
    ms = ev0.elapsed_time(ev1)
    pos += args.steps
    nxt = m.last_token()
    t_max = torch.tensor([ms], device="cuda")
    if ws > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms_max = float(t_max.item())
    ms_per_step = ms_max / args.steps
    value = args.steps / (ms_max / 1000.0)

    # end to end through the public call: host token in (pinned H2D), host
    # token out (D2H), one call per token
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        nxt = m.token_step(int(nxt), pos, want_next=True)
        pos += 1
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = torch.tensor([e0.elapsed_time(e1)], device="cuda")
    if ws > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e = args.steps / (float(e_ms.item()) / 1000.0)

    # Per-part device time of one token: each part launched alone over all
    # layers (the second of two passes timed), CUDA events on the launching
    # stream; the weights of 32 layers exceed L2, so no launch finds its
    # weights there.  Bytes per launch: weights + x + y for a projection, the
    # Q8_0 K/V of one layer's KV heads at the current context for attention.
    # The roofline reports the part that takes the most time per token.
    # (Tensor parallel with the peer-memory exchange inside the GEMVs: the
    # parts wait on the peers, so they are not launched alone.)
    solo_parts = ws == 1 or not args.p2p_allreduce
    peak, peak_kind = peaks()
    hd = shape.head_dim
    qd, kvd = lshape.n_heads * hd, lshape.n_kv_heads * hd
    io = {0: (shape.n_embd, qd + 2 * kvd), 2: (qd, lay.o_hi - lay.o_lo), 3: (shape.n_embd, 2 * lshape.n_ff),
          4: (lshape.n_ff, shape.n_embd), 5: (shape.n_embd, lay.v_hi - lay.v_lo)}
    parts, part_rl = {}, {}
    for part, name in enumerate(PART_NAMES if solo_parts else ()):
        evs = []
        n = 1 if part == 5 else shape.n_layers
        wb = 0
        for rep in range(2):
            for layer in range(n):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                wb = m.launch_part(layer, part)
                b.record(stream)
                if rep == 1:
                    evs.append((a, b))
        torch.cuda.synchronize()
        us = sum(a.elapsed_time(b) for a, b in evs) * 1000.0
        parts[name] = round(us, 1)
        if part == 1:
            nb = synth.kv_bytes_per_pos(lshape) // lshape.n_layers * (pos + 1)
        else:
            k_in, m_out = io[part]
            nb = wb + 4 * k_in + 4 * m_out
        gbs = nb / (us / n * 1e-6) / 1e9
        part_rl[name] = {"us_per_launch": round(us / n, 3), "bytes_per_launch": nb, "gbs": round(gbs, 1),
                         "frac": round(gbs / peak, 4)}
    ctx.check()
    dom = max((nm for nm in part_rl if nm != "append_attention"), key=lambda nm: parts[nm], default=None)
    traffic = recorded_traffic(args.shape, dom) if dom and ws == 1 else None
    # whole-step bytes at the mean context of the timed region, summed over
    # ranks (tensor parallel duplicates a few rows), against ws x the peak
    mean_ctx = args.prompt + args.warmup + args.steps / 2
    if ws == 1:
        step_bytes = synth.token_bytes(shape) + synth.kv_bytes_per_pos(shape) * mean_ctx
    else:
        wb, kvb = tpl.rank_token_bytes(shape, lay)
        tb = torch.tensor([wb + kvb * mean_ctx], dtype=torch.float64, device="cuda")
        dist.all_reduce(tb)
        step_bytes = float(tb.item())
    step_gbs = step_bytes / (ms_per_step / 1000.0) / 1e9

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        # three repeats of a 4-step sample: the median is the value, the
        # spread shows host noise (one compute thread, as the reference uses)
        reps = []
        for _ in range(3):
            v, kind, sample, _ = cpu_sample(4, 1, args.shape, args.prompt)
            reps.append(v)
        cpu = {"value": statistics.median(reps), "unit": "tok/s", "cores": 1, "kind": kind,
               "sample": sample + "; median of 3 repeats", "repeats": reps, **host_info()}

    launches_per_step = 1 + 5 * shape.n_layers + 2 + (1 if lay.v_hi - lay.v_lo < shape.n_vocab else 0)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, ws),
        "clocks": clk.summary(),
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": ({"bound": "hbm", "kernel": part_kernel(dom), "part": dom,
                      "achieved": part_rl[dom]["gbs"], "peak": peak, "unit": "GB/s", "frac": part_rl[dom]["frac"],
                      "peak_kind": peak_kind, "bytes_per_launch": part_rl[dom]["bytes_per_launch"],
                      "us_per_launch": part_rl[dom]["us_per_launch"],
                      "traffic": traffic["bytes"] if traffic else None,
                      "traffic_source": traffic["source"] if traffic else None}
                     if dom else
                     {"bound": "hbm", "kernel": "whole decode step (tensor parallel, summed over ranks)",
                      "achieved": step_gbs, "peak": ws * peak, "unit": "GB/s", "frac": step_gbs / (ws * peak),
                      "peak_kind": peak_kind, "bytes_per_launch": step_bytes, "traffic": None}),
        "parts_roofline": part_rl,
        "token_parts_us": parts,
        "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_gbs,
                          "frac": step_gbs / (ws * peak)},
        "cpu_baseline": cpu,
        "parity": parity,
        "nccl_nranks": ctx.tp_comm_size() if ws > 1 else None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    m.close()
    kv.close()
    ctx.close()
    if ws > 1:
        dist.destroy_process_group()


def main():
    # NCCL's log (its version banner and, at INFO, the communicator lines that
    # name every rank) goes to stderr, so stdout carries the one JSON line
    os.environ.setdefault("NCCL_DEBUG", "INFO")
    os.environ["NCCL_DEBUG_FILE"] = "/dev/stderr"
    args = parse()
    ws, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, ws, rank)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
