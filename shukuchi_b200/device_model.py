"""Uploads an in-memory llama-shaped model to HBM and wires it to the C ABI.

By default (tiled=True) every Q4_K / Q6_K matrix is uploaded as GGUF rows and
converted on the device into the row-tiled layout of the tensor-core matvec
(shk_cuda_tile, SHK_DTYPE_Q4_K_TILED / SHK_DTYPE_Q6_K_TILED).  With
tiled=False weights keep their GGUF block bytes for the staged dp4a GEMV: Q6_K
rows whose byte length is not a multiple of 16 (e.g. 22 blocks per row) are
padded to the next 16-byte multiple and converted in place to the planar
layout (shk_cuda_q6k_repack, SHK_DTYPE_Q6_K_PLANAR); an output head whose rows
stay unaligned keeps the GGUF layout (plain-load kernel).  torch is only the
allocator here.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

from . import cuda as sc
from .synth import BLOCK_BYTES, QK, Model, T_Q5K, T_Q6K


def _dev(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def upload_matrix(w: np.ndarray, qtype: int, rows: int, cols: int, device) -> tuple[torch.Tensor, int]:
    """Returns (device tensor, row stride in bytes; 0 when rows are dense)."""
    rb = (cols // QK) * BLOCK_BYTES[qtype]
    if rb % 16 == 0:
        return _dev(w, device), 0
    stride = (rb + 15) // 16 * 16
    padded = np.zeros((rows, stride), np.uint8)
    padded[:, :rb] = np.asarray(w).reshape(rows, rb)
    return _dev(padded.reshape(-1), device), stride


@dataclasses.dataclass
class Uploaded:
    model: Model
    tensors: list
    layers: list          # LayerDesc per layer
    desc: sc.ModelDesc


def to_planar(ctx: sc.Context, t: torch.Tensor, qtype: int, rows: int, cols: int, stride: int) -> int:
    """Repacks a Q6_K matrix in place when its rows are 16-byte aligned;
    returns the dtype to register it with."""
    if qtype != T_Q6K:
        return qtype
    rb = stride or (cols // QK) * BLOCK_BYTES[qtype]
    if rb % 16 or t.data_ptr() % 16:
        return qtype
    ctx.q6k_repack(t.data_ptr(), rows, cols, rb, True, ctx.stream)
    return sc.DTYPE_Q6_K_PLANAR


def to_tiled(ctx: sc.Context, w: np.ndarray, qtype: int, rows: int, cols: int, device) -> tuple[torch.Tensor, int]:
    """GGUF rows -> a device tensor in the row-tiled layout; returns (tensor, dtype)."""
    src = _dev(np.asarray(w).reshape(-1), device)
    dst = torch.empty(sc.tiled_bytes(qtype, rows, cols), dtype=torch.uint8, device=device)
    ctx.tile(qtype, src.data_ptr(), rows, cols, dst.data_ptr(), 0, ctx.stream)
    ctx.sync()
    return dst, (sc.DTYPE_Q4_K_TILED if qtype == 12 else sc.DTYPE_Q6_K_TILED)


def upload(model: Model, device: str | torch.device = "cuda:0", ctx: sc.Context | None = None,
           out_rows: int | None = None, tiled=True) -> Uploaded:
    """ctx: the context whose stream runs the layout conversions (required for
    a model the library runs).  out_rows: rows of the output head (a
    tensor-parallel rank's vocabulary slice).  tiled: which projections are
    row-tiled for the tensor-core matvec (synth_device.tiled_set: True = all,
    the default here, False = none); the others keep GGUF / planar rows."""
    from .synth_device import tiled_set
    ts = tiled_set(tiled) if ctx is not None else frozenset()
    s = model.shape
    keep = []

    def put(a):
        t = _dev(a, device)
        keep.append(t)
        return t.data_ptr()

    def mat(w, qt, rows, cols, proj):
        if proj in ts and qt != T_Q5K:  # Q5_K stays in GGUF rows (its own matvec)
            t, dt = to_tiled(ctx, w, qt, rows, cols, device)
            keep.append(t)
            return t.data_ptr(), 0, dt
        t, stride = upload_matrix(w, qt, rows, cols, device)
        keep.append(t)
        dt = to_planar(ctx, t, qt, rows, cols, stride) if ctx is not None else qt
        return t.data_ptr(), stride, dt

    layers = []
    hd = s.head_dim
    D, F, qd, kvd = s.n_embd, s.n_ff, s.n_heads * hd, s.n_kv_heads * hd
    o_rows = len(np.asarray(model.layers[0].wo).reshape(-1)) // ((qd // QK) * BLOCK_BYTES[s.t_o]) \
        if model.layers else D
    for Lw in model.layers:
        q, _, tq = mat(Lw.wq, s.t_q, qd, D, "qkv")
        k, _, tk = mat(Lw.wk, s.t_k, kvd, D, "qkv")
        v, sv, tv = mat(Lw.wv, s.t_v, kvd, D, "qkv")
        o, _, to = mat(Lw.wo, s.t_o, o_rows, qd, "o")
        g, _, tg = mat(Lw.wg, s.t_gate, F, D, "gateup")
        u, _, tu = mat(Lw.wu, s.t_up, F, D, "gateup")
        d, sd, td = mat(Lw.wd, s.t_down, D, F, "down")
        layers.append(sc.LayerDesc(put(Lw.attn_norm), put(Lw.ffn_norm), q, k, v, o, g, u, d,
                                   tq, tk, tv, to, tg, tu, td, sv, sd))
    nv = out_rows or s.n_vocab
    if "output" in ts and s.t_out != T_Q5K:
        out, t_out = to_tiled(ctx, model.output, s.t_out, nv, D, device)
    else:
        out = _dev(model.output, device)
        t_out = to_planar(ctx, out, s.t_out, nv, D, 0) if ctx is not None else s.t_out
    keep.append(out)
    desc = sc.ModelDesc(s.n_layers, s.n_embd, s.n_heads, s.n_kv_heads, hd, s.n_ff, s.n_vocab, 0.0,
                        put(model.tok_embd), s.t_embd, out.data_ptr(), t_out)
    if ctx is not None:
        ctx.sync()
    return Uploaded(model, keep, layers, desc)


class GpuDecoder:
    """A DeviceModel + KV cache for a synthetic model, ready for token steps."""

    def __init__(self, ctx: sc.Context, model: Model, max_seq: int, device="cuda:0", tp_rows=None,
                 p2p_exchange=None, o_ranges=None, tiled=True, ll_exchange=None):
        """tp_rows: (o_lo, o_hi, v_lo, v_hi) of a tensor-parallel rank whose
        context has joined its group (the model is that rank's shard).
        p2p_exchange: for the all-reduce over peer memory, a function taking
        this rank's handle and returning every rank's in rank order (an
        all-gather); o_ranges: every rank's (o_lo, o_hi).  ll_exchange: the
        same all-gather for the all-reduce with flags in the data words
        (shk_cuda_model_tp_ll_*), which replaces NCCL's."""
        s = model.shape
        out_rows = tp_rows[3] - tp_rows[2] if tp_rows is not None else None
        # the peer-memory exchange runs in the staged GEMV's epilogue (GGUF / planar rows)
        self.up = upload(model, device, ctx=ctx, out_rows=out_rows, tiled=tiled if p2p_exchange is None else False)
        self.kv = sc.KvCache(ctx, s.n_layers, s.n_kv_heads, s.head_dim, max_seq)
        self.m = sc.DeviceModel(ctx, self.kv, self.up.desc)
        if tp_rows is not None:
            self.m.set_tp_rows(*tp_rows)
        if p2p_exchange is not None:
            self.m.tp_p2p_import(p2p_exchange(self.m.tp_p2p_export()), o_ranges)
        if ll_exchange is not None:
            self.m.tp_ll_import(ll_exchange(self.m.tp_ll_export()))
        for i, lv in enumerate(self.up.layers):
            self.m.set_layer(i, lv)

    def close(self):
        self.m.close()
        self.kv.close()

    def generate(self, prompt, n_decode, logits_out: np.ndarray | None = None):
        """Same token schedule as the reference engine_generate: prompt tokens
        one at a time, then n_decode greedy tokens; the last decoded token is
        also run through all layers."""
        pos = 0
        nxt = 0
        for i, t in enumerate(prompt):
            last = i == len(prompt) - 1
            ptr = logits_out[0].ctypes.data if (last and logits_out is not None) else None
            nxt = self.m.token_step(int(t), pos, want_next=last, logits_host_ptr=ptr)
            pos += 1
        out = []
        for j in range(n_decode):
            out.append(nxt)
            want = j + 1 < n_decode
            ptr = logits_out[j + 1].ctypes.data if (want and logits_out is not None) else None
            nxt2 = self.m.token_step(int(nxt), pos, want_next=want, logits_host_ptr=ptr)
            pos += 1
            if want:
                nxt = nxt2
        return np.array(out, np.uint32)
