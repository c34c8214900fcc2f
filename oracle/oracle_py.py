"""Python access to the oracle libraries (TEST INFRASTRUCTURE ONLY).

* ``Oracle``    -- oracle/liboracle.so, the C restatement of the reference path.
* ``Reference`` -- oracle/_ref/libshkref.so, the unmodified reference sources
  compiled in place (only where they were built).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline / reference
leg import this module.  The product path never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libshkref.so")
REF_CLI = os.path.join(HERE, "_ref", "shukuchi_ref")

P, U32, U64, I, F = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int, C.c_float


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class OrcLayer(C.Structure):
    _fields_ = [("attn_norm", P), ("ffn_norm", P), ("wq", P), ("wk", P), ("wv", P), ("wo", P),
                ("wg", P), ("wu", P), ("wd", P), ("tq", U32), ("tk", U32), ("tv", U32),
                ("to", U32), ("tg", U32), ("tu", U32), ("td", U32)]


class OrcModel(C.Structure):
    _fields_ = [("n_layers", U32), ("n_embd", U32), ("n_heads", U32), ("n_kv_heads", U32),
                ("head_dim", U32), ("n_ff", U32), ("n_vocab", U32), ("rope_theta", F),
                ("layers", C.POINTER(OrcLayer)), ("tok_embd", P), ("tok_embd_type", U32),
                ("output", P), ("output_type", U32)]


def build(ref: bool = False) -> None:
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


class Oracle:
    def __init__(self, threads: int | None = None):
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        sig = {
            "orc_set_threads": (None, [I]),
            "orc_half_to_float": (F, [C.c_uint16]),
            "orc_dequant_q4k": (None, [P, P, U32]),
            "orc_dequant_q5k": (None, [P, P, U32]),
            "orc_dequant_q6k": (None, [P, P, U32]),
            "orc_matvec": (I, [U32, P, P, P, U32, U32]),
            "orc_rmsnorm": (I, [P, P, P, U32]),
            "orc_rope": (I, [P, U32, U32, U32, F]),
            "orc_q8_quantize": (None, [P, U32, P]),
            "orc_q8_dequantize": (None, [P, U32, P]),
            "orc_attention": (I, [P, P, P, P, U32, U32, U32, U32, F]),
            "orc_swiglu": (None, [P, P, P, U32]),
            "orc_embed": (I, [P, U32, U32, P, U32]),
            "orc_argmax": (U32, [P, U32]),
            "orc_kv_create": (P, [U32, U32, U32, U32, U32]),
            "orc_kv_destroy": (None, [P]),
            "orc_kv_append": (I, [P, U32, U32, P, P]),
            "orc_kv_read_range": (I, [P, U32, U32, U32, P, P]),
            "orc_kv_token_blocks": (P, [P, U32, U32, I]),
            "orc_kv_clear": (None, [P]),
            "orc_kv_seq_len": (U32, [P, U32]),
            "orc_forward_layer": (I, [C.POINTER(OrcModel), P, U32, U32, P]),
            "orc_generate": (I, [C.POINTER(OrcModel), P, P, U32, U32, P, P]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        self.L = L
        L.orc_set_threads(threads or max(1, min(32, os.cpu_count() or 1)))

    def half_to_float(self, h: int) -> float:
        return self.L.orc_half_to_float(h)

    def dequant(self, qtype: int, blocks: np.ndarray, k: int) -> np.ndarray:
        y = np.empty(k, np.float32)
        fn = {12: self.L.orc_dequant_q4k, 13: self.L.orc_dequant_q5k, 14: self.L.orc_dequant_q6k}[qtype]
        fn(_ptr(blocks), _ptr(y), k)
        return y

    def matvec(self, qtype: int, w: np.ndarray, x: np.ndarray, m: int, k: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(m, np.float32)
        assert self.L.orc_matvec(qtype, _ptr(w), _ptr(x), _ptr(y), m, k) == 0
        return y

    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.L.orc_rmsnorm(_ptr(x), _ptr(np.ascontiguousarray(w, np.float32)), _ptr(y), x.size)
        return y

    def rope(self, qk, n_heads, head_dim, pos, theta=10000.0):
        v = np.array(qk, np.float32, copy=True)
        self.L.orc_rope(_ptr(v), n_heads, head_dim, pos, theta)
        return v

    def q8_quantize(self, x) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(((x.size + 31) // 32) * 36, np.uint8)
        self.L.orc_q8_quantize(_ptr(x), x.size, _ptr(out))
        return out

    def attention(self, q, k, v, n_heads, n_kv, hd, seq, scale):
        out = np.empty(n_heads * hd, np.float32)
        assert self.L.orc_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), n_heads, n_kv, hd, seq, scale) == 0
        return out

    def swiglu(self, g, u):
        h = np.empty_like(g)
        self.L.orc_swiglu(_ptr(g), _ptr(u), _ptr(h), g.size)
        return h

    def embed(self, table, dtype, token, n_embd):
        out = np.empty(n_embd, np.float32)
        assert self.L.orc_embed(_ptr(table), dtype, token, _ptr(out), n_embd) == 0
        return out

    def argmax(self, x) -> int:
        x = np.ascontiguousarray(x, np.float32)
        return self.L.orc_argmax(_ptr(x), x.size)

    # ---- model ----
    def model_struct(self, model):
        """Builds an OrcModel for a shukuchi_b200.synth.Model (keeps refs)."""
        s = model.shape
        arr = (OrcLayer * s.n_layers)()
        for i, Lw in enumerate(model.layers):
            arr[i] = OrcLayer(_ptr(Lw.attn_norm), _ptr(Lw.ffn_norm), _ptr(Lw.wq), _ptr(Lw.wk),
                              _ptr(Lw.wv), _ptr(Lw.wo), _ptr(Lw.wg), _ptr(Lw.wu), _ptr(Lw.wd),
                              s.t_q, s.t_k, s.t_v, s.t_o, s.t_gate, s.t_up, s.t_down)
        m = OrcModel(s.n_layers, s.n_embd, s.n_heads, s.n_kv_heads, s.head_dim, s.n_ff, s.n_vocab,
                     10000.0, arr, _ptr(model.tok_embd), s.t_embd, _ptr(model.output), s.t_out)
        m._keep = (arr, model)
        return m

    def kv_create(self, n_layers, n_kv, hd, max_seq, block=32):
        return self.L.orc_kv_create(n_layers, n_kv, hd, block, max_seq)

    def kv_destroy(self, kv):
        self.L.orc_kv_destroy(kv)

    def kv_token_blocks(self, kv, layer, pos, which, nbytes) -> np.ndarray:
        p = self.L.orc_kv_token_blocks(kv, layer, pos, which)
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), (nbytes,)).copy()

    def generate(self, model, prompt, n_decode, max_seq=None):
        s = model.shape
        ms = self.model_struct(model)
        kv = self.kv_create(s.n_layers, s.n_kv_heads, s.head_dim, max_seq or (len(prompt) + n_decode + 1))
        toks = np.zeros(n_decode, np.uint32)
        logits = np.zeros((n_decode, s.n_vocab), np.float32)
        pr = np.ascontiguousarray(prompt, np.uint32)
        try:
            assert self.L.orc_generate(C.byref(ms), kv, _ptr(pr), pr.size, n_decode, _ptr(toks), _ptr(logits)) == 0
        finally:
            self.kv_destroy(kv)
        return toks, logits

    def forward_layers(self, model, token, pos, kv, hidden=None):
        """embed(token) (if hidden is None) then every layer at pos; returns hidden."""
        s = model.shape
        ms = self.model_struct(model)
        if hidden is None:
            hidden = self.embed(model.tok_embd, s.t_embd, token, s.n_embd)
        hidden = np.array(hidden, np.float32, copy=True)
        for layer in range(s.n_layers):
            assert self.L.orc_forward_layer(C.byref(ms), kv, layer, pos, _ptr(hidden)) == 0
        return hidden


class Reference:
    """The reference's own C code, compiled from its sources (oracle/_ref)."""

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def __init__(self):
        L = C.CDLL(REF_SO)
        sig = {
            "ref_matmul": (I, [U32, P, P, P, U32, U32]),
            "ref_rmsnorm": (I, [P, P, P, U32]),
            "ref_rope": (I, [P, U32, U32, U32, F]),
            "ref_attention": (I, [P, P, P, P, U32, U32, U32, U32, F]),
            "ref_softmax": (I, [P, U32]),
            "ref_embed": (I, [P, U32, U32, P, U32]),
            "ref_mlp_swiglu": (I, [P, P, P, P, P, U32, U32]),
            "ref_q8_quantize": (None, [P, U32, P]),
            "ref_kv_create": (P, [U32, U32, U32, U32, U32]),
            "ref_kv_destroy": (None, [P]),
            "ref_kv_append": (I, [P, U32, U32, P, P]),
            "ref_kv_read_range": (I, [P, U32, U32, U32, P, P]),
            "ref_kv_token_blocks": (P, [P, U32, U32, I]),
            "ref_engine_new": (P, [U32, U32, U32, U32, U32]),
            "ref_engine_free": (None, [P]),
            "ref_engine_kv": (P, [P]),
            "ref_forward_layer": (I, [P, P, P, P, U32, U32, P]),
            "ref_generate_file": (I, [C.c_char_p, U32, P, U32, U32, P, P, P]),
            "ref_tokenize": (I, [C.c_char_p, C.c_char_p, P, U32]),
            "ref_now": (C.c_double, []),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        self.L = L

    def matvec(self, qtype, w, x, m, k):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(m, np.float32)
        assert self.L.ref_matmul(qtype, _ptr(w), _ptr(x), _ptr(y), m, k) == 0
        return y

    def rmsnorm(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.L.ref_rmsnorm(_ptr(x), _ptr(np.ascontiguousarray(w, np.float32)), _ptr(y), x.size)
        return y

    def rope(self, qk, n_heads, head_dim, pos, theta=10000.0):
        v = np.array(qk, np.float32, copy=True)
        self.L.ref_rope(_ptr(v), n_heads, head_dim, pos, theta)
        return v

    def q8_quantize(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(((x.size + 31) // 32) * 36, np.uint8)
        self.L.ref_q8_quantize(_ptr(x), x.size, _ptr(out))
        return out

    def attention(self, q, k, v, n_heads, n_kv, hd, seq, scale):
        out = np.empty(n_heads * hd, np.float32)
        assert self.L.ref_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), n_heads, n_kv, hd, seq, scale) == 0
        return out

    def embed(self, table, dtype, token, n_embd):
        out = np.empty(n_embd, np.float32)
        assert self.L.ref_embed(_ptr(table), dtype, token, _ptr(out), n_embd) == 0
        return out

    def tokenize_file(self, path, text: bytes, cap=1 << 16):
        out = np.zeros(cap, np.uint32)
        n = self.L.ref_tokenize(path.encode(), text, _ptr(out), cap)
        assert n >= 0
        return out[:min(n, cap)].copy()

    def generate_file(self, path, prompt, n_decode, n_vocab, depth=3):
        pr = np.ascontiguousarray(prompt, np.uint32)
        ids = np.zeros(n_decode, np.uint32)
        logits = np.zeros((n_decode, n_vocab), np.float32)
        stats = np.zeros(8, np.uint64)
        rc = self.L.ref_generate_file(path.encode(), depth, _ptr(pr), pr.size, n_decode, _ptr(ids),
                                      _ptr(logits), _ptr(stats))
        assert rc == 0, "reference generation failed"
        return ids, logits, stats

    def forward_layer_fn(self, model, max_seq):
        """Returns (engine_handle, step(layer, pos, hidden)) driving the reference
        forward_layer_view on in-memory weights."""
        s = model.shape
        h = self.L.ref_engine_new(s.n_layers, s.n_embd, s.n_heads, s.n_kv_heads, max_seq)
        assert h
        keep = []

        def step(layer, pos, hidden):
            Lw = model.layers[layer]
            ptrs = (P * 9)(*[_ptr(a) for a in (Lw.attn_norm, Lw.wq, Lw.wk, Lw.wv, Lw.wo,
                                                Lw.ffn_norm, Lw.wg, Lw.wu, Lw.wd)])
            types = (U32 * 9)(0, s.t_q, s.t_k, s.t_v, s.t_o, 0, s.t_gate, s.t_up, s.t_down)
            sizes = (U64 * 9)(*[a.nbytes for a in (Lw.attn_norm, Lw.wq, Lw.wk, Lw.wv, Lw.wo,
                                                    Lw.ffn_norm, Lw.wg, Lw.wu, Lw.wd)])
            keep.append((ptrs, types, sizes))
            assert self.L.ref_forward_layer(h, ptrs, types, sizes, layer, pos, _ptr(hidden)) == 0
            keep.clear()

        return h, step
