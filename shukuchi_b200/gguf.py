"""Minimal GGUF (v3) writer for synthetic llama-architecture models.

Writes the metadata keys and tensor names the Shukuchi engine reads
(engine/src/model_loader.c:97-111, 336-346; engine/src/llama_tensor_map.c:
66-129): llama.block_count, llama.embedding_length, llama.attention.head_count,
llama.attention.head_count_kv, tokenizer.ggml.tokens (fixed-width "t%05d"
strings, so greedy longest match maps a prompt text to exact ids), and the
tensors token_embd / blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_output,
ffn_norm, ffn_gate, ffn_up, ffn_down} / output_norm / output, data aligned to
32 bytes.  No BOS key is written, so no BOS token is prepended.
"""
from __future__ import annotations

import struct

import numpy as np

from .synth import Model

GGUF_MAGIC = b"GGUF"
T_UINT32, T_FLOAT32, T_STRING, T_ARRAY = 4, 6, 8, 9
GGML_F32 = 0
ALIGN = 32


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv_u32(key: str, v: int) -> bytes:
    return _str(key) + struct.pack("<II", T_UINT32, v)


def _kv_f32(key: str, v: float) -> bytes:
    return _str(key) + struct.pack("<If", T_FLOAT32, v)


def _kv_str(key: str, v: str) -> bytes:
    return _str(key) + struct.pack("<I", T_STRING) + _str(v)


def _kv_str_array(key: str, vals: list[str]) -> bytes:
    out = [_str(key), struct.pack("<IIQ", T_ARRAY, T_STRING, len(vals))]
    out += [_str(v) for v in vals]
    return b"".join(out)


def token_text(i: int) -> str:
    return f"t{i:05d}"


def model_tensors(model: Model):
    """(name, ggml type, dims (ne0 = columns first), bytes) in file order."""
    s = model.shape
    D, hd = s.n_embd, s.head_dim
    t = [("token_embd.weight", s.t_embd, (D, s.n_vocab), model.tok_embd)]
    for i, L in enumerate(model.layers):
        p = f"blk.{i}."
        t += [(p + "attn_norm.weight", GGML_F32, (D,), L.attn_norm),
              (p + "attn_q.weight", s.t_q, (D, s.n_heads * hd), L.wq),
              (p + "attn_k.weight", s.t_k, (D, s.n_kv_heads * hd), L.wk),
              (p + "attn_v.weight", s.t_v, (D, s.n_kv_heads * hd), L.wv),
              (p + "attn_output.weight", s.t_o, (s.n_heads * hd, D), L.wo),
              (p + "ffn_norm.weight", GGML_F32, (D,), L.ffn_norm),
              (p + "ffn_gate.weight", s.t_gate, (D, s.n_ff), L.wg),
              (p + "ffn_up.weight", s.t_up, (D, s.n_ff), L.wu),
              (p + "ffn_down.weight", s.t_down, (s.n_ff, D), L.wd)]
    t += [("output_norm.weight", GGML_F32, (D,), model.output_norm),
          ("output.weight", s.t_out, (D, s.n_vocab), model.output)]
    return t


def write_model(path: str, model: Model, rope_theta: float = 10000.0, tokens: list | None = None,
                bos: int | None = None) -> None:
    """tokens: the vocabulary strings (default: fixed-width token_text ids);
    bos: tokenizer.ggml.bos_token_id (default: none, so no BOS is prepended)."""
    s = model.shape
    tensors = model_tensors(model)
    vocab = tokens if tokens is not None else [token_text(i) for i in range(s.n_vocab)]
    assert len(vocab) == s.n_vocab
    kvs = [_kv_str("general.architecture", "llama"), _kv_u32("general.alignment", ALIGN),
           _kv_u32("llama.block_count", s.n_layers), _kv_u32("llama.embedding_length", s.n_embd),
           _kv_u32("llama.feed_forward_length", s.n_ff), _kv_u32("llama.attention.head_count", s.n_heads),
           _kv_u32("llama.attention.head_count_kv", s.n_kv_heads),
           _kv_f32("llama.rope.freq_base", rope_theta),
           _kv_str_array("tokenizer.ggml.tokens", vocab)]
    if bos is not None:
        kvs.append(_kv_u32("tokenizer.ggml.bos_token_id", bos))
    infos, offs, off = [], [], 0
    for name, typ, dims, data in tensors:
        off = (off + ALIGN - 1) // ALIGN * ALIGN
        offs.append(off)
        infos.append(_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
                     + struct.pack("<IQ", typ, off))
        off += np.ascontiguousarray(data).nbytes
    head = GGUF_MAGIC + struct.pack("<IQQ", 3, len(tensors), len(kvs)) + b"".join(kvs) + b"".join(infos)
    data_start = (len(head) + ALIGN - 1) // ALIGN * ALIGN
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data_start - len(head)))
        pos = 0
        for (name, typ, dims, data), o in zip(tensors, offs):
            f.write(b"\0" * (o - pos))
            b = np.ascontiguousarray(data).tobytes()
            f.write(b)
            pos = o + len(b)
