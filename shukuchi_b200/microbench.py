"""Kernel microbenchmarks on one GPU.

  python -m shukuchi_b200.microbench gemv [--shapes QT,M,K ...] [--reps R]
      Batch-1 dequant-matvec sweep (Q4_K = 12, Q6_K = 14), fp32 x ~ N(0,1),
      seeded random blocks; Q6_K matrices repacked once to the planar layout
      the decode path uses (shk_cuda_q6k_repack), outside the timed graph.  Each launch reads a different copy of the weights
      (copies totalling >= 4x the L2 size, at least 2), launches captured in a
      CUDA graph, CUDA-event timing on the launching stream.
      Bytes per launch = weights + 4*K (x) + 4*M (y).

  python -m shukuchi_b200.microbench prefill [--shapes QT,M,K ...] [--tokens T]
      Batched (prefill) dequantise-matmul of T tokens (default 512) on the
      tensor cores over the GEMV sweep's matrices; TFLOP/s = 2 M K T / time
      against the measured dense bf16 peak.

  python -m shukuchi_b200.microbench kv [--ctx C ...] [--batch B ...]
      Q8_0 KV cache: 64 query / 8 KV heads, head_dim 128, K/V ~ N(0,1).
      One step = for each of B independent sequences, append one new K/V row
      (quantise-on-append) and attend over all c+1 positions.  A pool of
      sequences larger than 4x L2 is rotated so no step finds its cache in L2.
      Bytes per sequence = (c+1)*2304 (Q8_0 K+V read) + 2304 (append write)
      + 8 KB (new K/V fp32) + 32 KB (q) + 32 KB (out).

  python -m shukuchi_b200.microbench parts [--shape llama8b] [--layers 8] [--prompt 512]
      One decode token split into its kernels: a model of the given shape
      with `--layers` distinct layers (more than 4x L2 of weights) is run
      through a prompt, then each part (RMSNorm+QKV+RoPE GEMV, append +
      attention, O + residual, RMSNorm + gate/up + SwiGLU, down + residual,
      lm_head) is captured for all layers in a CUDA graph and timed per launch.

  python -m shukuchi_b200.microbench timeline [--shape llama8b] [--layers 32] [--prompt 512]
      The persistent decode kernel's own timeline: one decode_steps launch of
      --steps tokens with CTA 0 recording %globaltimer around every grid
      barrier; reports per phase kind the mean wall time (barrier to barrier)
      and the part of it CTA 0 spent waiting at the barrier.

  python -m shukuchi_b200.microbench prompt [--shape llama8b] [--tokens 512]
      A T-token prompt through the model as one batched prefill
      (shk_cuda_prefill: tensor-core matmuls, row-batched glue) against T
      token steps (timed on a prefix, scaled): prefill ms, tok/s, speed-up.

  python -m shukuchi_b200.microbench loader [--shape llama8b] [--prompt 8] [--decode 16] [--depth 3]
      The C engine on a GGUF file of the shape (written once under --dir):
      HBM-resident mode (every layer pread -> pinned -> HBM once, then the
      captured step) and ring mode (SHUKUCHI_HBM_RESIDENT=0: every layer
      streamed through `depth` device slots on every token, as the reference
      streams them from disk): open and first-generation times, tok/s,
      streamed GB/s and the prefetch hit / miss statistics.

One JSON line per case; `frac` is achieved GB/s over the measured HBM copy
bandwidth (MEASURED_PEAKS.json when present).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from . import cuda as sc
from .synth import BLOCK_BYTES, QK
from .synth_device import _fill_blocks

GEMV_SHAPES = [(12, 4096, 4096), (12, 14336, 4096), (12, 4096, 14336), (14, 4096, 14336),
               (14, 128256, 4096), (13, 4096, 4096), (13, 14336, 4096), (13, 4096, 14336)]
_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def hbm_peak() -> tuple[float, str]:
    p = os.path.join(_ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def l2_bytes() -> int:
    return torch.cuda.get_device_properties(0).L2_cache_size


def _time_graph(g: torch.cuda.CUDAGraph, stream, reps: int) -> float:
    """ms per replay."""
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(reps):
            g.replay()
        b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def gemv(args, ctx) -> None:
    peak, kind = hbm_peak()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    shapes = [tuple(int(v) for v in s.split(",")) for s in args.shapes] if args.shapes else GEMV_SHAPES
    for qt, m, k in shapes:
        row = (k // QK) * BLOCK_BYTES[qt]
        stride = (row + 15) // 16 * 16
        wb = m * stride
        ncopy = max(2, min(64, math.ceil(4 * l2_bytes() / wb)))
        ws = []
        for _ in range(ncopy):
            t = torch.empty(wb, dtype=torch.uint8, device="cuda")
            _fill_blocks(t, qt, m, k, stride, gen)
            ws.append(t)
        if stride != row:
            raise SystemExit(f"rows of {qt},{m},{k} are not 16-byte multiples; use the C ABI row_stride")
        dt = qt
        if args.tiled and qt == 13:
            continue  # Q5_K has no row-tiled form: it runs on GGUF rows
        if args.tiled:  # row-tiled copies for the tensor-core matvec
            torch.cuda.synchronize()
            tw = []
            for t in ws:
                d = torch.empty(sc.tiled_bytes(qt, m, k), dtype=torch.uint8, device="cuda")
                ctx.tile(qt, t.data_ptr(), m, k, d.data_ptr(), stride)
                tw.append(d)
            ctx.sync()
            ws = tw
            dt = sc.DTYPE_Q4_K_TILED if qt == 12 else sc.DTYPE_Q6_K_TILED
        elif qt == 14:  # the layout the decode path registers Q6_K weights in
            torch.cuda.synchronize()
            for t in ws:
                ctx.q6k_repack(t.data_ptr(), m, k, stride, True)
            ctx.sync()
            dt = sc.DTYPE_Q6_K_PLANAR
        x = torch.randn(k, device="cuda", generator=gen)
        y = torch.empty(m, device="cuda")
        s = torch.cuda.Stream()
        nl = max(ncopy, args.launches)
        with torch.cuda.stream(s):
            for i in range(3):  # warm-up (also loads the kernels)
                ctx.matvec(dt, ws[i % ncopy].data_ptr(), x.data_ptr(), y.data_ptr(), m, k, stream=s.cuda_stream)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for i in range(nl):
                    ctx.matvec(dt, ws[i % ncopy].data_ptr(), x.data_ptr(), y.data_ptr(), m, k,
                               stream=s.cuda_stream)
        ms = _time_graph(g, s, args.reps)
        ctx.check()
        us = ms * 1000.0 / nl
        alg = m * row + 4 * k + 4 * m
        gbs = alg / (us * 1e-6) / 1e9
        print(json.dumps({"bench": "gemv", "qtype": {12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}[qt], "m": m, "k": k,
                          "layout": "tiled" if args.tiled else ("planar" if qt == 14 else "gguf"),
                          "us": round(us, 3), "bytes": alg, "gbs": round(gbs, 1),
                          "frac": round(gbs / peak, 4), "peak_gbs": peak, "peak_kind": kind,
                          "copies": ncopy}), flush=True)
        del g, ws
        torch.cuda.empty_cache()


def bf16_peak() -> tuple[float, str]:
    p = os.path.join(_ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def prefill(args, ctx) -> None:
    """Batched dequantise-matmul on the tensor cores: T tokens through each
    matrix of the GEMV sweep that it takes (Q4_K, Q6_K); one call = the f16
    conversion of x (a power-of-two scale per token) + the tcgen05 kernel.
    TFLOP/s = 2 M K T / time."""
    peak, kind = bf16_peak()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    shapes = [tuple(int(v) for v in s.split(",")) for s in args.shapes] if args.shapes else GEMV_SHAPES
    shapes = [s for s in shapes if s[0] in (12, 14)]
    T = args.tokens
    for qt, m, k in shapes:
        row = (k // QK) * BLOCK_BYTES[qt]
        stride = (row + 15) // 16 * 16
        w = torch.empty(m * stride, dtype=torch.uint8, device="cuda")
        _fill_blocks(w, qt, m, k, stride, gen)
        dt = qt
        if qt == 14:
            torch.cuda.synchronize()
            ctx.q6k_repack(w.data_ptr(), m, k, stride, True)
            ctx.sync()
            dt = sc.DTYPE_Q6_K_PLANAR
        x = torch.randn(T, k, device="cuda", generator=gen)
        y = torch.empty(T, m, device="cuda")
        s = torch.cuda.Stream()
        n = args.launches
        with torch.cuda.stream(s):
            for _ in range(3):
                ctx.prefill_matmul(dt, w.data_ptr(), x.data_ptr(), y.data_ptr(), m, k, T, row_stride=stride,
                                   stream=s.cuda_stream)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(n):
                    ctx.prefill_matmul(dt, w.data_ptr(), x.data_ptr(), y.data_ptr(), m, k, T, row_stride=stride,
                                       stream=s.cuda_stream)
        ms = _time_graph(g, s, args.reps)
        ctx.check()
        us = ms * 1000.0 / n
        tf = 2.0 * m * k * T / (us * 1e-6) / 1e12
        print(json.dumps({"bench": "prefill", "qtype": "Q4_K" if qt == 12 else "Q6_K", "m": m, "k": k,
                          "tokens": T, "us": round(us, 2), "tflops": round(tf, 1), "frac": round(tf / peak, 4),
                          "peak_tflops": peak, "peak_kind": kind}), flush=True)
        del g
        torch.cuda.empty_cache()


def kv(args, ctx) -> None:
    peak, kind = hbm_peak()
    H, KV, HD = 64, 8, 128
    row = KV * HD
    per_pos = 2 * KV * (HD + 4 * HD // 32)  # K + V Q8_0 bytes per position: 2304
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    for c in args.ctx:
        for B in args.batch:
            seq_bytes = (c + 8) * per_pos
            pool = max(B, min(4096, math.ceil(4 * l2_bytes() / seq_bytes)))
            pool = math.ceil(pool / B) * B
            cache = sc.KvCache(ctx, pool, KV, HD, c + 8)
            chunk = 8192
            kbuf = torch.empty(chunk * row, device="cuda")
            vbuf = torch.empty(chunk * row, device="cuda")
            for sidx in range(pool):
                for p0 in range(0, c, chunk):
                    n = min(chunk, c - p0)
                    kbuf.normal_(generator=gen)
                    vbuf.normal_(generator=gen)
                    cache.append_range(sidx, p0, n, kbuf.data_ptr(), vbuf.data_ptr())
            q = torch.randn(B, H * HD, device="cuda", generator=gen)
            kn = torch.randn(B, row, device="cuda", generator=gen)
            vn = torch.randn(B, row, device="cuda", generator=gen)
            out = torch.empty(B, H * HD, device="cuda")
            torch.cuda.synchronize()
            s = torch.cuda.Stream()
            steps = pool // B
            scale = 1.0 / math.sqrt(HD)
            def attend(first):  # the batch's B sequences (cache layers first..) in one launch
                if B == 1:
                    cache.attend(first, q[0].data_ptr(), out[0].data_ptr(), H, c + 1, scale,
                                 kn[0].data_ptr(), vn[0].data_ptr(), stream=s.cuda_stream)
                else:
                    cache.attend_batch(first, B, q.data_ptr(), out.data_ptr(), H, c + 1, scale,
                                       kn.data_ptr(), vn.data_ptr(), stream=s.cuda_stream)
            with torch.cuda.stream(s):
                attend(0)  # warm-up (sizes the batch scratch outside the capture)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for st in range(steps):
                        attend(st * B)
            ms = _time_graph(g, s, args.reps)
            ctx.check()
            us = ms * 1000.0 / steps
            alg = B * ((c + 1) * per_pos + per_pos + 2 * 4 * row + 2 * 4 * H * HD)
            gbs = alg / (us * 1e-6) / 1e9
            print(json.dumps({"bench": "kv", "ctx": c, "batch": B, "us_per_step": round(us, 3),
                              "bytes": alg, "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                              "peak_gbs": peak, "peak_kind": kind, "pool": pool,
                              "launches_per_step": 1}), flush=True)
            del g
            cache.close()
            torch.cuda.empty_cache()


PART_NAMES = ("rmsnorm_qkv_rope", "append_attention", "o_proj_residual", "rmsnorm_gateup_swiglu",
              "down_residual", "lm_head")


def parts(args, ctx) -> None:
    import dataclasses

    import numpy as np

    from . import synth
    from .synth_device import make_device_model

    peak, kind = hbm_peak()
    shape = dataclasses.replace(synth.SHAPES[args.shape], n_layers=args.layers)
    wts = make_device_model(shape, seed=7, ctx=ctx)
    kv = sc.KvCache(ctx, shape.n_layers, shape.n_kv_heads, shape.head_dim, args.prompt + 16)
    m = sc.DeviceModel(ctx, kv, wts.desc)
    try:
        for i, lv in enumerate(wts.layers):
            m.set_layer(i, lv)
        rng = np.random.default_rng(0)
        for i, t in enumerate(rng.integers(0, shape.n_vocab, args.prompt)):
            m.token_step(int(t), i, want_next=(i == args.prompt - 1))
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        for part, name in enumerate(PART_NAMES):
            n = 1 if part == 5 else shape.n_layers
            reps = 8 if part == 5 else 1
            with torch.cuda.stream(s):
                wb = [m.launch_part(layer, part, stream=s.cuda_stream) for layer in range(n)]
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for _ in range(reps):
                        for layer in range(n):
                            m.launch_part(layer, part, stream=s.cuda_stream)
            torch.cuda.nvtx.range_push(name)  # ncu --nvtx --nvtx-include "<part>/" picks one part
            ms = _time_graph(g, s, args.reps)
            torch.cuda.nvtx.range_pop()
            ctx.check()
            us = ms * 1000.0 / (n * reps)
            gbs = wb[0] / (us * 1e-6) / 1e9
            print(json.dumps({"bench": "parts", "shape": shape.name, "part": name, "us": round(us, 2),
                              "weight_bytes": wb[0], "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                              "peak_gbs": peak, "peak_kind": kind, "ctx": args.prompt}), flush=True)
            del g
    finally:
        m.close()
        kv.close()


def timeline(args, ctx) -> None:
    import dataclasses

    import numpy as np

    from . import synth
    from .synth_device import make_device_model

    shape = dataclasses.replace(synth.SHAPES[args.shape], n_layers=args.layers)
    wts = make_device_model(shape, seed=7, ctx=ctx)
    ctx = sc.Context(0, flags=sc.FLAG_PERSISTENT)
    kv = sc.KvCache(ctx, shape.n_layers, shape.n_kv_heads, shape.head_dim, args.prompt + args.steps + 8)
    m = sc.DeviceModel(ctx, kv, wts.desc)
    try:
        for i, lv in enumerate(wts.layers):
            m.set_layer(i, lv)
        rng = np.random.default_rng(0)
        nxt = 0
        for i, t in enumerate(rng.integers(0, shape.n_vocab, args.prompt)):
            nxt = m.token_step(int(t), i, want_next=(i == args.prompt - 1))
        per_tok = 1 + 5 * shape.n_layers + 2
        m.trace_enable(per_tok * args.steps)
        m.decode_steps(nxt, args.prompt, args.steps)
        torch.cuda.synchronize()
        ctx.check()
        tr = m.trace_read(1 + 2 * per_tok * args.steps)
        m.trace_enable(0)
        kinds = ["embed"] + ["qkv", "attention", "o_proj", "gate_up", "down"] * shape.n_layers + ["lm_head", "argmax"]
        wall, wait = {}, {}
        prev = tr[0]
        for i in range((len(tr) - 1) // 2):
            arrive, leave = tr[1 + 2 * i], tr[2 + 2 * i]
            k = kinds[i % per_tok]
            wall.setdefault(k, []).append(leave - prev)
            wait.setdefault(k, []).append(leave - arrive)
            prev = leave
        total_us = (tr[-1] - tr[0]) / 1000.0
        out = {"bench": "timeline", "shape": shape.name, "ctx": args.prompt, "steps": args.steps,
               "us_per_token": round(total_us / args.steps, 1), "phases": {}}
        for k in wall:
            out["phases"][k] = {"wall_us": round(float(np.mean(wall[k])) / 1000.0, 2),
                                "cta0_wait_us": round(float(np.mean(wait[k])) / 1000.0, 2),
                                "count_per_token": len(wall[k]) // args.steps}
        print(json.dumps(out), flush=True)
    finally:
        m.close()
        kv.close()
        ctx.close()


def prompt(args, ctx) -> None:
    """Prompt of T tokens at the model shape: one batched prefill
    (shk_cuda_prefill) against T token steps, device time by CUDA events."""
    import numpy as np

    from . import synth
    from .synth_device import make_device_model

    shape = synth.SHAPES[args.shape]
    wts = make_device_model(shape, seed=7, ctx=ctx, tiled=False)  # the prefill reads GGUF / planar rows
    kv = sc.KvCache(ctx, shape.n_layers, shape.n_kv_heads, shape.head_dim, args.tokens + 8)
    m = sc.DeviceModel(ctx, kv, wts.desc)
    try:
        for i, lv in enumerate(wts.layers):
            m.set_layer(i, lv)
        rng = np.random.default_rng(0)
        toks = rng.integers(0, shape.n_vocab, args.tokens).astype(np.uint32)
        s = torch.cuda.ExternalStream(ctx.stream)
        m.prefill(toks[:64], 0)  # warm-up (kernel loads, scratch)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        first_pf = m.prefill(toks, 0)
        b.record(s)
        torch.cuda.synchronize()
        pf_ms = a.elapsed_time(b)
        kv.clear()
        n_steps = min(args.tokens, args.steps)  # token steps timed on a prefix, scaled to T
        m.token_step(int(toks[0]), 0, want_next=False)
        torch.cuda.synchronize()
        a.record(s)
        nxt = 0
        for i in range(1, n_steps):
            nxt = m.token_step(int(toks[i]), i, want_next=(i == n_steps - 1))
        b.record(s)
        torch.cuda.synchronize()
        step_ms = a.elapsed_time(b) / max(1, n_steps - 1)
        ctx.check()
        D, hd = shape.n_embd, shape.head_dim
        qd, kvd, F = shape.n_heads * hd, shape.n_kv_heads * hd, shape.n_ff
        layer_w = D * qd + 2 * D * kvd + qd * D + 3 * D * F  # weights of the seven matmuls
        flops = 2.0 * args.tokens * layer_w * shape.n_layers
        print(json.dumps({"bench": "prompt", "shape": shape.name, "tokens": args.tokens,
                          "prefill_ms": round(pf_ms, 3), "prefill_tok_s": round(args.tokens / (pf_ms / 1e3), 1),
                          "token_step_ms": round(step_ms, 4),
                          "token_by_token_ms": round(step_ms * args.tokens, 2),
                          "speedup": round(step_ms * args.tokens / pf_ms, 2), "first_token": int(first_pf),
                          "matmul_tflops": round(flops / (pf_ms / 1e3) / 1e12, 1)}), flush=True)
    finally:
        m.close()
        kv.close()


def loader(args, ctx) -> None:
    import ctypes as C
    import time

    import numpy as np

    from . import gguf, synth

    class Stats(C.Structure):
        _fields_ = [("layer_loads", C.c_uint64), ("layer_bytes_read", C.c_uint64), ("max_layer_size", C.c_size_t),
                    ("peak_buffer_usage", C.c_size_t), ("peak_rss", C.c_size_t),
                    ("max_concurrent_buffers", C.c_uint32), ("prefetch_hits", C.c_uint32),
                    ("prefetch_misses", C.c_uint32)]

    class Config(C.Structure):
        _fields_ = [("n_threads", C.c_uint32), ("batch_size", C.c_uint32), ("prefetch_depth", C.c_uint32),
                    ("kv_block_size", C.c_uint32), ("kv_quant", C.c_uint32), ("use_mmap", C.c_int)]

    L = C.CDLL(os.path.join(os.path.dirname(os.path.abspath(__file__)), "engine", "libshukuchi.so"))
    L.engine_open.restype = C.c_void_p
    L.engine_open.argtypes = [C.c_char_p, C.POINTER(Config)]
    L.engine_generate_ids.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p]
    L.engine_get_streaming_stats.argtypes = [C.c_void_p, C.POINTER(Stats)]
    L.engine_close.argtypes = [C.c_void_p]
    s = synth.SHAPES[args.shape]
    os.makedirs(args.dir, exist_ok=True)
    path = os.path.join(args.dir, f"{args.shape}.gguf")
    write_s = 0.0
    if not os.path.exists(path):
        t = time.perf_counter()
        gguf.write_model(path, synth.make_model(s, seed=3))
        write_s = time.perf_counter() - t
    size = os.path.getsize(path)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, s.n_vocab, args.prompt).astype(np.uint32)
    n = args.prompt + args.decode
    ids = np.zeros(args.decode, np.uint32)
    for mode in ("resident", "ring"):
        os.environ["SHUKUCHI_HBM_RESIDENT"] = "1" if mode == "resident" else "0"
        os.environ["SHUKUCHI_MAX_SEQ"] = str(n + 8)
        t0 = time.perf_counter()
        h = L.engine_open(path.encode(), C.byref(Config(4, 1, args.depth, 32, 0, 0)))
        t1 = time.perf_counter()
        if not h:
            raise SystemExit("engine_open failed")
        try:
            rc = L.engine_generate_ids(h, prompt.ctypes.data, prompt.size, args.decode, ids.ctypes.data, None)
            t2 = time.perf_counter()
            rc2, t3 = rc, t2
            if mode == "resident":  # a second generation: the layers are in HBM already
                rc2 = L.engine_generate_ids(h, prompt.ctypes.data, prompt.size, args.decode, ids.ctypes.data, None)
                t3 = time.perf_counter()
            st = Stats()
            L.engine_get_streaming_stats(h, C.byref(st))
        finally:
            L.engine_close(h)
        if rc != args.decode or rc2 != args.decode:
            raise SystemExit(f"generation failed ({mode})")
        gen = t2 - t1
        line = {"bench": "loader", "shape": s.name, "mode": mode, "file_bytes": size, "file_write_s": round(write_s, 2),
                "depth": args.depth, "tokens": n, "open_s": round(t1 - t0, 3), "first_generation_s": round(gen, 3),
                "first_generation_tok_s": round(n / gen, 2), "layer_loads": st.layer_loads,
                "layer_bytes_read": st.layer_bytes_read, "max_layer_size": st.max_layer_size,
                "peak_buffer_usage": st.peak_buffer_usage, "max_concurrent_buffers": st.max_concurrent_buffers,
                "prefetch_hits": st.prefetch_hits, "prefetch_misses": st.prefetch_misses,
                "prefetch_hit_rate": round(st.prefetch_hits / max(1, st.prefetch_hits + st.prefetch_misses), 4)}
        if mode == "resident":
            warm = t3 - t2
            line["warm_generation_tok_s"] = round(n / warm, 2)
            # staging: the first generation's extra time over the warm one
            line["staging_s"] = round(max(gen - warm, 1e-9), 3)
            line["staged_gbs"] = round(st.layer_bytes_read / max(gen - warm, 1e-9) / 1e9, 2)
        else:
            line["streamed_gbs"] = round(st.layer_bytes_read / gen / 1e9, 2)
        print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("gemv")
    g.add_argument("--shapes", nargs="*")
    g.add_argument("--launches", type=int, default=20)
    g.add_argument("--reps", type=int, default=5)
    g.add_argument("--tiled", action="store_true", help="row-tiled weights on the tensor-core matvec")
    k = sub.add_parser("kv")
    pf = sub.add_parser("prefill")
    pf.add_argument("--shapes", nargs="*")
    pf.add_argument("--tokens", type=int, default=512)
    pf.add_argument("--launches", type=int, default=10)
    pf.add_argument("--reps", type=int, default=5)
    k.add_argument("--ctx", type=int, nargs="*", default=[1024, 4096, 16384, 32768])
    k.add_argument("--batch", type=int, nargs="*", default=[1, 8, 32])
    k.add_argument("--reps", type=int, default=5)
    pp = sub.add_parser("parts")
    pp.add_argument("--shape", default="llama8b")
    pp.add_argument("--layers", type=int, default=8)
    pp.add_argument("--prompt", type=int, default=512)
    pp.add_argument("--reps", type=int, default=5)
    tl = sub.add_parser("timeline")
    tl.add_argument("--shape", default="llama8b")
    tl.add_argument("--layers", type=int, default=32)
    tl.add_argument("--prompt", type=int, default=512)
    tl.add_argument("--steps", type=int, default=4)
    pr = sub.add_parser("prompt")
    pr.add_argument("--shape", default="llama8b")
    pr.add_argument("--tokens", type=int, default=512)
    pr.add_argument("--steps", type=int, default=64)
    ld = sub.add_parser("loader")
    ld.add_argument("--shape", default="llama8b")
    ld.add_argument("--prompt", type=int, default=8)
    ld.add_argument("--decode", type=int, default=16)
    ld.add_argument("--depth", type=int, default=3)
    ld.add_argument("--dir", default="/tmp/shk_gguf")
    args = ap.parse_args()
    torch.cuda.set_device(0)
    ctx = sc.Context(0)
    try:
        {"gemv": gemv, "kv": kv, "parts": parts, "timeline": timeline, "prefill": prefill,
         "loader": loader, "prompt": prompt}[args.cmd](args, ctx)
    finally:
        ctx.close()


if __name__ == "__main__":
    main()
