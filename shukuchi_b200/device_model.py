"""Uploads an in-memory llama-shaped model to HBM and wires it to the C ABI.

Weights keep their GGUF block bytes.  Q6_K rows whose byte length is not a
multiple of 16 (e.g. 22 blocks per row) are padded to the next 16-byte
multiple so the staged GEMV can move whole rows with bulk copies; the row
stride is passed to the library.  torch is only the allocator here.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

from . import cuda as sc
from .synth import BLOCK_BYTES, QK, Model, T_Q6K


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


def upload(model: Model, device: str | torch.device = "cuda:0") -> Uploaded:
    s = model.shape
    keep = []

    def put(a):
        t = _dev(a, device)
        keep.append(t)
        return t.data_ptr()

    layers = []
    hd = s.head_dim
    for Lw in model.layers:
        wv, sv = upload_matrix(Lw.wv, s.t_v, s.n_kv_heads * hd, s.n_embd, device)
        wd, sd = upload_matrix(Lw.wd, s.t_down, s.n_embd, s.n_ff, device)
        keep += [wv, wd]
        layers.append(sc.LayerDesc(
            put(Lw.attn_norm), put(Lw.ffn_norm), put(Lw.wq), put(Lw.wk), wv.data_ptr(), put(Lw.wo),
            put(Lw.wg), put(Lw.wu), wd.data_ptr(),
            s.t_q, s.t_k, s.t_v, s.t_o, s.t_gate, s.t_up, s.t_down, sv, sd))
    desc = sc.ModelDesc(s.n_layers, s.n_embd, s.n_heads, s.n_kv_heads, hd, s.n_ff, s.n_vocab, 0.0,
                        put(model.tok_embd), s.t_embd, put(model.output), s.t_out)
    return Uploaded(model, keep, layers, desc)


class GpuDecoder:
    """A DeviceModel + KV cache for a synthetic model, ready for token steps."""

    def __init__(self, ctx: sc.Context, model: Model, max_seq: int, device="cuda:0", tp_rows=None):
        """tp_rows: (o_lo, o_hi, v_lo, v_hi) of a tensor-parallel rank whose
        context has joined its group (the model is that rank's shard)."""
        s = model.shape
        self.up = upload(model, device)
        self.kv = sc.KvCache(ctx, s.n_layers, s.n_kv_heads, s.head_dim, max_seq)
        self.m = sc.DeviceModel(ctx, self.kv, self.up.desc)
        if tp_rows is not None:
            self.m.set_tp_rows(*tp_rows)
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
