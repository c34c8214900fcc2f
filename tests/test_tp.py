"""Tensor parallelism: the rank layout and weight shards of shukuchi_b200.tp,
and the decode of `world` ranks that all-reduce their partial O and down
projections and merge their argmax over vocabulary slices.

CPU: `world` gloo processes each run the oracle's operators on their shard
(numpy glue, the same per-rank schedule as the CUDA path: rank 0 adds the
residual, the others contribute their partial sums); greedy ids must equal
the oracle's single-device decode and logits stay within 1e-2 * std.
GPU: the same through libshk_cuda (NCCL all-reduce inside the captured
decode graphs), one process per GPU; skipped with fewer GPUs than ranks.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from shukuchi_b200 import synth, tp

TP_SHAPE = synth.ModelShape("tp-hd128", 2, 1024, 8, 4, 2048, 1024)


def _shape(name):
    return TP_SHAPE if name == "tp-hd128" else synth.SHAPES[name]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# --------------------------------------------------------------- layout
@pytest.mark.parametrize("name,world", [("llama8b", 2), ("llama8b", 4), ("llama8b", 8), ("llama70b", 8),
                                        ("tinyllama", 2), ("tinyllama", 4), ("small", 2), ("tp-hd128", 4)])
def test_layout_covers_every_row_once(name, world):
    s = _shape(name)
    lays = [tp.layout(s, r, world) for r in range(world)]
    A = lays[0].group_size
    # every (query head, O output row) pair is computed by exactly one rank
    cover = np.zeros((s.n_heads, s.n_embd), np.int32)
    for L in lays:
        assert L.kv_hi - L.kv_lo == s.n_kv_heads * A // world
        for h in L.q_heads:
            assert L.kv_lo <= h % s.n_kv_heads < L.kv_hi  # modulo GQA (engine/src/ops.c:421)
            cover[h, L.o_lo:L.o_hi] += 1
        # Wo column ranges are whole 256-blocks
        loc = tp.local_shape(s, L)
        assert (loc.n_heads * loc.head_dim) % synth.QK == 0 and loc.head_dim == s.head_dim
    assert np.all(cover == 1)
    f = np.zeros(s.n_ff, np.int32)
    for L in lays:
        assert L.f_lo % synth.QK == 0 and L.f_hi % synth.QK == 0
        f[L.f_lo:L.f_hi] += 1
    assert np.all(f == 1)
    v = np.zeros(s.n_vocab, np.int32)
    for L in lays:
        v[L.v_lo:L.v_hi] += 1
    assert np.all(v == 1) or all(L.v_hi - L.v_lo == s.n_vocab for L in lays)


def test_shard_bytes_are_the_rows_and_columns(oracle):
    """Dequantised shards equal the corresponding slices of the full matrices."""
    s = TP_SHAPE
    m = synth.make_model(s, seed=3, n_layers=1)
    L = m.layers[0]
    hd = s.head_dim
    for world in (2, 4):
        for r in range(world):
            lay = tp.layout(s, r, world)
            Ls = tp.shard_layer(L, s, lay)

            def deq(t, w, rows, cols):
                rb = (cols // synth.QK) * synth.BLOCK_BYTES[t]
                return np.stack([oracle.dequant(t, w[i * rb:(i + 1) * rb], cols) for i in range(rows)])

            q = deq(s.t_q, L.wq, s.n_heads * hd, s.n_embd)
            qs = deq(s.t_q, Ls.wq, len(lay.q_heads) * hd, s.n_embd)
            want = np.concatenate([q[h * hd:(h + 1) * hd] for h in lay.q_heads])
            assert np.array_equal(qs, want)
            o = deq(s.t_o, L.wo, s.n_embd, s.n_heads * hd)
            os_ = deq(s.t_o, Ls.wo, lay.o_hi - lay.o_lo, len(lay.q_heads) * hd)
            cols = np.concatenate([np.arange(h * hd, (h + 1) * hd) for h in lay.q_heads])
            assert np.array_equal(os_, o[lay.o_lo:lay.o_hi][:, cols])
            d = deq(s.t_down, L.wd, s.n_embd, s.n_ff)
            ds = deq(s.t_down, Ls.wd, s.n_embd, lay.f_hi - lay.f_lo)
            assert np.array_equal(ds, d[:, lay.f_lo:lay.f_hi])


# --------------------------------------------------------------- CPU ranks
def _q8_roundtrip(oracle, x):
    """Q8_0 quantise (engine/src/kv_cache.c:28-55) then dequantise (:57-69)."""
    b = oracle.q8_quantize(x).reshape(-1, 36)
    scale = b[:, :4].copy().view(np.float32)
    q = b[:, 4:].copy().view(np.int8).astype(np.float32)
    return (q * scale).reshape(-1)[: x.size]


def rank_decode(oracle, mr, lay, prompt, n_dec, all_reduce, all_gather):
    """One rank's greedy decode with the oracle's operators: the reference's
    token schedule (engine/src/engine.c:306-501) on a shard, partial sums
    all-reduced after O and down, logits slices gathered before the argmax."""
    s = mr.shape
    D, hd, Hl, KVl, F = s.n_embd, s.head_dim, s.n_heads, s.n_kv_heads, s.n_ff
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    kc = [[] for _ in range(s.n_layers)]
    vc = [[] for _ in range(s.n_layers)]

    def layer(li, pos, hidden):
        Lw = mr.layers[li]
        x = oracle.rmsnorm(hidden, Lw.attn_norm)
        q = oracle.matvec(s.t_q, Lw.wq, x, Hl * hd, D)
        k = oracle.matvec(s.t_k, Lw.wk, x, KVl * hd, D)
        v = oracle.matvec(s.t_v, Lw.wv, x, KVl * hd, D)
        q = oracle.rope(q, Hl, hd, pos)
        k = oracle.rope(k, KVl, hd, pos)
        kc[li].append(_q8_roundtrip(oracle, k))
        vc[li].append(_q8_roundtrip(oracle, v))
        att = oracle.attention(q, np.concatenate(kc[li]), np.concatenate(vc[li]), Hl, KVl, hd, pos + 1, scale)
        proj = oracle.matvec(s.t_o, Lw.wo, att, lay.o_hi - lay.o_lo, Hl * hd)
        part = hidden.copy() if lay.rank == 0 else np.zeros(D, np.float32)
        part[lay.o_lo:lay.o_hi] = (part[lay.o_lo:lay.o_hi] + proj) if lay.rank == 0 else proj
        hidden = all_reduce(part)
        x = oracle.rmsnorm(hidden, Lw.ffn_norm)
        g = oracle.matvec(s.t_gate, Lw.wg, x, F, D)
        u = oracle.matvec(s.t_up, Lw.wu, x, F, D)
        proj = oracle.matvec(s.t_down, Lw.wd, oracle.swiglu(g, u), D, F)
        part = (hidden + proj) if lay.rank == 0 else proj
        return all_reduce(part.astype(np.float32))

    def step(tok, pos):
        h = oracle.embed(mr.tok_embd, s.t_embd, int(tok), D)
        for li in range(s.n_layers):
            h = layer(li, pos, h)
        return h

    def head(h):
        loc = oracle.matvec(s.t_out, mr.output, h, lay.v_hi - lay.v_lo, D)
        return loc if lay.v_hi - lay.v_lo == s.n_vocab else all_gather(loc)

    pos = 0
    h = None
    for t in prompt:
        h = step(t, pos)
        pos += 1
    ids = np.zeros(n_dec, np.uint32)
    logits = np.zeros((n_dec, s.n_vocab), np.float32)
    for t in range(n_dec):
        logits[t] = head(h)
        ids[t] = oracle.argmax(logits[t])
        if t + 1 < n_dec:
            h = step(ids[t], pos)
            pos += 1
    return ids, logits


def _cpu_rank(rank, world, port, name, seed, prompt, n_dec, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    from oracle.oracle_py import Oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        model = synth.make_model(_shape(name), seed=seed)
        mr, lay = tp.shard_model(model, rank, world)

        def all_reduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        def all_gather(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            out = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(out, t)
            return torch.cat(out).numpy()

        ids, logits = rank_decode(Oracle(), mr, lay, prompt, n_dec, all_reduce, all_gather)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), ids=ids, logits=logits)
    finally:
        dist.destroy_process_group()


def _run_ranks(target, world, args, timeout):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs]


def _check(oracle, name, seed, prompt, n_dec, world, out_dir):
    model = synth.make_model(_shape(name), seed=seed)
    t_ref, l_ref = oracle.generate(model, prompt, n_dec)
    for r in range(world):
        z = np.load(os.path.join(out_dir, f"r{r}.npz"))
        assert np.array_equal(z["ids"], t_ref), (r, z["ids"], t_ref)
        for t in range(n_dec):
            assert np.max(np.abs(z["logits"][t] - l_ref[t])) <= 1e-2 * np.std(l_ref[t]), (r, t)


@pytest.mark.parametrize("name,world", [("small", 2), ("tp-hd128", 2), ("tp-hd128", 4)])
def test_tp_ranks_match_oracle_cpu(oracle, tmp_path, name, world):
    prompt = np.random.default_rng(7).integers(0, _shape(name).n_vocab, 5).astype(np.uint32)
    n_dec = 6
    codes = _run_ranks(_cpu_rank, world, (name, 21, prompt, n_dec, str(tmp_path)), 240)
    assert codes == [0] * world
    _check(oracle, name, 21, prompt, n_dec, world, str(tmp_path))


# --------------------------------------------------------------- GPU ranks
def _gpu_rank(rank, world, port, name, seed, prompt, n_dec, out_dir, mode="nccl"):
    import datetime

    import torch
    import torch.distributed as dist

    from shukuchi_b200 import cuda as sc
    from shukuchi_b200.device_model import GpuDecoder
    from shukuchi_b200.synth_device import TILED_DEFAULT
    torch.cuda.set_device(rank)
    # gloo carries only the communicator id; the decode's collectives are NCCL
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    ctx = sc.Context(rank)
    try:
        obj = [sc.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.tp_init(rank, world, obj[0])
        model = synth.make_model(_shape(name), seed=seed)
        mr, lay = tp.shard_model(model, rank, world)
        def gather(h):
            hs = [None] * world
            dist.all_gather_object(hs, h)
            return hs
        o_ranges = [(L.o_lo, L.o_hi) for L in (tp.layout(model.shape, r, world) for r in range(world))]
        # the bench's weight layouts (O and down row-tiled): this ill-conditioned
        # model (logits ~1e4) turns any change of rounding into a visible drift
        dec = GpuDecoder(ctx, mr, len(prompt) + n_dec + 1, device=f"cuda:{rank}", tiled=TILED_DEFAULT,
                         tp_rows=(lay.o_lo, lay.o_hi, lay.v_lo, lay.v_hi),
                         p2p_exchange=gather if mode == "p2p" else None, o_ranges=o_ranges,
                         ll_exchange=gather if mode == "ll" else None)
        try:
            logits = np.zeros((n_dec, model.shape.n_vocab), np.float32)
            ids = dec.generate(prompt, n_dec, logits)
            # the captured decode loop (argmax merged over ranks on the device)
            dec.m.decode_steps(int(ids[0]), len(prompt), n_dec - 1)
            last = dec.m.last_token()
            ctx.check()
        finally:
            dec.close()
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), ids=ids, logits=logits, last=last)
    finally:
        ctx.close()
        dist.destroy_process_group()


# Four ranks with the one-shot all-reduce only (the layout that shares KV
# heads between pairs of ranks; the bench's parity check runs the same case):
# the C engine's four-rank run over NCCL did not finish on four GPUs for a
# cause not yet found, so the NCCL and peer-exchange modes stay at two ranks.
@pytest.mark.gpu
@pytest.mark.parametrize("name,world,mode", [(n, 2, m) for n in ("small", "tp-hd128") for m in ("nccl", "p2p", "ll")]
                         + [("tp-hd128", 4, "ll")])
def test_tp_ranks_match_oracle_gpu(oracle, tmp_path, name, world, mode):
    """nccl: all-reduce kernels between the GEMVs; p2p: partials pushed into
    peer memory by the O / down GEMVs and summed by the next GEMV; ll: a
    one-shot all-reduce kernel over peer memory with the flags in the data
    words."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    prompt = np.random.default_rng(7).integers(0, _shape(name).n_vocab, 5).astype(np.uint32)
    n_dec = 8
    codes = _run_ranks(_gpu_rank, world, (name, 21, prompt, n_dec, str(tmp_path), mode), 300)
    assert codes == [0] * world
    _check(oracle, name, 21, prompt, n_dec, world, str(tmp_path))
    for r in range(world):
        z = np.load(os.path.join(str(tmp_path), f"r{r}.npz"))
        assert int(z["last"]) == int(z["ids"][-1])
