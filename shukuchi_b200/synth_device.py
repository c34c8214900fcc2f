"""Seeded synthetic K-quant weights generated directly in HBM with torch's
device RNG (same value distributions as ``synth.py``, different stream).

Used where a full-size model would take too long to build on the host
(e.g. the 4.9 GB Llama-3.1-8B-shape model for the decode benchmark).  Q6_K
rows that are not 16-byte multiples are padded.
"""
from __future__ import annotations

import dataclasses

import torch

from . import cuda as sc
from .synth import BLOCK_BYTES, QK, ModelShape, T_Q4K, T_Q5K, T_Q6K


def _fill_blocks(buf: torch.Tensor, qtype: int, rows: int, cols: int, stride: int, gen) -> None:
    """buf: uint8 view of rows * stride bytes."""
    nb = cols // QK
    bb = BLOCK_BYTES[qtype]
    v = buf.view(rows, stride)[:, : nb * bb]
    v.copy_(torch.randint(0, 256, v.shape, dtype=torch.uint8, device=buf.device, generator=gen))
    blocks = v.view(rows, nb, bb)
    if qtype in (T_Q4K, T_Q5K):
        d = (torch.randn((rows, nb, 2), device=buf.device, generator=gen) * 0.002).abs().half()
        blocks[:, :, 0:4] = d.view(torch.uint8).view(rows, nb, 4)
    else:
        sc8 = torch.randint(-32, 32, (rows, nb, 16), dtype=torch.int8, device=buf.device, generator=gen)
        blocks[:, :, 192:208] = sc8.view(torch.uint8)
        d = (torch.randn((rows, nb, 1), device=buf.device, generator=gen) * 0.0005).abs().half()
        blocks[:, :, 208:210] = d.view(torch.uint8).view(rows, nb, 2)


def _matrix(qtype, rows, cols, device, gen, keep, ctx=None, tiled=False):
    """Returns (device pointer, row stride or 0, dtype to register).  Matrices
    are generated in GGUF blocks; with a context they are converted on the
    device to the row-tiled layout of the tensor-core matvec (tiled) or, for
    Q6_K, repacked in place to the planar layout of the staged GEMV."""
    rb = (cols // QK) * BLOCK_BYTES[qtype]
    stride = (rb + 15) // 16 * 16
    t = torch.zeros(rows * stride, dtype=torch.uint8, device=device)
    _fill_blocks(t, qtype, rows, cols, stride, gen)
    if ctx is not None and tiled:
        dst = torch.empty(sc.tiled_bytes(qtype, rows, cols), dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)
        ctx.tile(qtype, t.data_ptr(), rows, cols, dst.data_ptr(), stride)
        ctx.sync()
        del t
        keep.append(dst)
        return dst.data_ptr(), 0, (sc.DTYPE_Q4_K_TILED if qtype == T_Q4K else sc.DTYPE_Q6_K_TILED)
    keep.append(t)
    dt = qtype
    if ctx is not None and qtype == T_Q6K:
        torch.cuda.synchronize(device)
        ctx.q6k_repack(t.data_ptr(), rows, cols, stride, True)
        ctx.sync()
        dt = sc.DTYPE_Q6_K_PLANAR
    return t.data_ptr(), (0 if stride == rb else stride), dt


# Projections whose matrices go row-tiled (tensor-core matvec) by default: the
# ones where it measured faster than the staged dp4a GEMV on the 8B decode
# step (O: 8.2 vs 9.0 us, down: 19.0 vs 21.1 us per layer); QKV, gate/up and
# the output head stay GGUF / planar rows.
TILED_DEFAULT = frozenset({"o", "down"})
PROJECTIONS = frozenset({"qkv", "o", "gateup", "down", "output"})


def tiled_set(tiled) -> frozenset:
    """True: every projection; False: none; else an iterable of names from
    PROJECTIONS (QKV and gate/up are planned as one launch each, so their
    matrices share a layout)."""
    if tiled is True:
        return PROJECTIONS
    if tiled is False or tiled is None:
        return frozenset()
    t = frozenset(tiled)
    assert t <= PROJECTIONS, t - PROJECTIONS
    return t


@dataclasses.dataclass
class DeviceWeights:
    shape: ModelShape
    keep: list
    layers: list
    desc: sc.ModelDesc

    def layer_bytes(self) -> int:
        return sum(t.numel() for t in self.keep) // max(1, self.shape.n_layers)


def make_device_model(shape: ModelShape, seed: int = 0, device="cuda:0",
                      distinct_layers: int | None = None, o_rows: int | None = None,
                      out_rows: int | None = None, ctx: sc.Context | None = None,
                      tiled=TILED_DEFAULT) -> DeviceWeights:
    """All weights in HBM.  distinct_layers < n_layers reuses layer buffers
    cyclically (only for smoke-sized runs; the benchmark uses distinct layers).
    o_rows / out_rows: rows of the O projection and of the output head when
    they differ from n_embd / n_vocab (a tensor-parallel rank's shard, whose
    `shape` is the local one of shukuchi_b200.tp.local_shape).  ctx: the
    context whose stream converts the matrices (required for a model the
    library runs; without it the matrices stay GGUF blocks).  tiled: which
    projections are row-tiled for the tensor-core matvec (tiled_set); the
    others keep GGUF rows (Q6_K planar) for the staged GEMV."""
    ts = tiled_set(tiled)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    keep: list = []
    s = shape
    hd = s.head_dim
    nd = distinct_layers or s.n_layers
    made = []
    for _ in range(nd):
        an = (1 + 0.02 * torch.randn(s.n_embd, device=device, generator=gen)).float()
        fn = (1 + 0.02 * torch.randn(s.n_embd, device=device, generator=gen)).float()
        keep += [an, fn]
        q, _, tq = _matrix(s.t_q, s.n_heads * hd, s.n_embd, device, gen, keep, ctx, "qkv" in ts)
        k, _, tk = _matrix(s.t_k, s.n_kv_heads * hd, s.n_embd, device, gen, keep, ctx, "qkv" in ts)
        v, sv, tv = _matrix(s.t_v, s.n_kv_heads * hd, s.n_embd, device, gen, keep, ctx, "qkv" in ts)
        o, _, to = _matrix(s.t_o, o_rows or s.n_embd, s.n_heads * hd, device, gen, keep, ctx, "o" in ts)
        g, _, tg = _matrix(s.t_gate, s.n_ff, s.n_embd, device, gen, keep, ctx, "gateup" in ts)
        u, _, tu = _matrix(s.t_up, s.n_ff, s.n_embd, device, gen, keep, ctx, "gateup" in ts)
        dn, sd, td = _matrix(s.t_down, s.n_embd, s.n_ff, device, gen, keep, ctx, "down" in ts)
        made.append(sc.LayerDesc(an.data_ptr(), fn.data_ptr(), q, k, v, o, g, u, dn,
                                 tq, tk, tv, to, tg, tu, td, sv, sd))
    layers = [made[i % nd] for i in range(s.n_layers)]
    te, _, _ = _matrix(s.t_embd, s.n_vocab, s.n_embd, device, gen, keep)
    out, so, tout = _matrix(s.t_out, out_rows or s.n_vocab, s.n_embd, device, gen, keep, ctx, "output" in ts)
    assert so == 0, "output head rows must be 16-byte multiples"
    desc = sc.ModelDesc(s.n_layers, s.n_embd, s.n_heads, s.n_kv_heads, hd, s.n_ff, s.n_vocab, 0.0,
                        te, s.t_embd, out, tout)
    torch.cuda.synchronize(device)
    return DeviceWeights(s, keep, layers, desc)
