"""Seeded synthetic K-quant tensors and llama-shaped models.

The value distributions follow the benchmark description of the decode path:

* Q4_K super-blocks (144 B): fp16 ``d`` and ``dmin`` ~ |N(0, 0.002)|, 12 uniform
  scale bytes, 128 uniform quant bytes.
* Q5_K super-blocks (176 B, the reference's layout): as Q4_K plus 32 uniform
  high-bit bytes.
* Q6_K super-blocks (210 B): 128 B ``ql`` + 64 B ``qh`` uniform, 16 int8 scales
  uniform in [-32, 31], fp16 ``d`` ~ |N(0, 0.0005)|.
* Norm weights: fp32 1 + N(0, 0.02).

Subnormal fp16 scales are kept on purpose: the reference decodes them at half
their IEEE value (engine/src/ops.c:65-78) and the GPU path must match that.
"""
from __future__ import annotations

import dataclasses
import hashlib

import numpy as np

QK = 256
Q4K_BYTES = 144
Q5K_BYTES = 176
Q6K_BYTES = 210
T_F32, T_F16, T_Q4K, T_Q5K, T_Q6K = 0, 1, 12, 13, 14
BLOCK_BYTES = {T_Q4K: Q4K_BYTES, T_Q5K: Q5K_BYTES, T_Q6K: Q6K_BYTES}


def q4k_blocks(rng: np.random.Generator, n_blocks: int, d_sigma: float = 0.002) -> np.ndarray:
    """n_blocks Q4_K super-blocks as a (n_blocks, 144) uint8 array."""
    b = rng.integers(0, 256, size=(n_blocks, Q4K_BYTES), dtype=np.uint8)
    d = np.abs(rng.normal(0.0, d_sigma, size=(n_blocks, 2))).astype(np.float16)
    b[:, 0:4] = d.view(np.uint8).reshape(n_blocks, 4)
    return b


def q6k_blocks(rng: np.random.Generator, n_blocks: int, d_sigma: float = 0.0005) -> np.ndarray:
    """n_blocks Q6_K super-blocks as a (n_blocks, 210) uint8 array."""
    b = rng.integers(0, 256, size=(n_blocks, Q6K_BYTES), dtype=np.uint8)
    sc = rng.integers(-32, 32, size=(n_blocks, 16), dtype=np.int8)
    b[:, 192:208] = sc.view(np.uint8)
    d = np.abs(rng.normal(0.0, d_sigma, size=(n_blocks, 1))).astype(np.float16)
    b[:, 208:210] = d.view(np.uint8).reshape(n_blocks, 2)
    return b


def q5k_blocks(rng: np.random.Generator, n_blocks: int, d_sigma: float = 0.002) -> np.ndarray:
    """n_blocks Q5_K super-blocks (the reference's 176-byte layout
    {u16 d, u16 dmin, u8 scales[12], u8 qh[32], u8 qs[128]}) as a
    (n_blocks, 176) uint8 array; d and dmin as for Q4_K."""
    b = rng.integers(0, 256, size=(n_blocks, Q5K_BYTES), dtype=np.uint8)
    d = np.abs(rng.normal(0.0, d_sigma, size=(n_blocks, 2))).astype(np.float16)
    b[:, 0:4] = d.view(np.uint8).reshape(n_blocks, 4)
    return b


# rms of the dequantised weight per unit of d_sigma: Q4_K d * sc * (q - 7.5)
# with sc uniform 0..63 (rms 36.4) and q uniform 0..15 (std 4.6); Q5_K with q
# 0..31 (std 9.2); Q6_K sc * (q - 32), both uniform over 64 values (rms 18.5).
_GAIN = {T_Q4K: 36.4 * 4.6, T_Q5K: 36.4 * 9.2, T_Q6K: 18.5 * 18.5}


def _center(b: np.ndarray, qtype: int) -> None:
    """Q4_K / Q5_K blocks in place: mins = scales and dmin = d * (qmax / 2), so
    every sub-block dequantises to d * sc * (q - qmax / 2), zero-mean."""
    if qtype == T_Q6K:
        return
    sc = b[:, 4:16]
    sc[:, 4:8] = sc[:, 0:4]
    lo = sc[:, 8:12] & 0xF
    sc[:, 8:12] = lo | (lo << 4)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    half = 7.5 if qtype == T_Q4K else 15.5
    b[:, 2:4] = (d * half).astype(np.float16).view(np.uint8).reshape(-1, 2)


def quant_matrix(rng: np.random.Generator, qtype: int, rows: int, cols: int,
                 conditioned: bool = False) -> np.ndarray:
    """A rows x cols matrix in GGUF row-major block layout (flat uint8).

    conditioned: zero-mean weights of rms 1/sqrt(cols) (a unit-gain map, as
    trained weights are), instead of the benchmark distributions whose
    activations grow into the thousands across layers."""
    assert cols % QK == 0
    nb = rows * (cols // QK)
    gen = {T_Q4K: q4k_blocks, T_Q5K: q5k_blocks, T_Q6K: q6k_blocks}[qtype]
    if not conditioned:
        return gen(rng, nb).reshape(-1)
    blocks = gen(rng, nb, d_sigma=1.0 / (_GAIN[qtype] * np.sqrt(cols)))
    _center(blocks, qtype)
    return blocks.reshape(-1)


def norm_weight(rng: np.random.Generator, n: int) -> np.ndarray:
    return (1.0 + rng.normal(0.0, 0.02, size=n)).astype(np.float32)


@dataclasses.dataclass
class ModelShape:
    name: str
    n_layers: int
    n_embd: int
    n_heads: int
    n_kv_heads: int
    n_ff: int
    n_vocab: int
    # quant types per tensor (Q4_K_M mix: attn_v, ffn_down, output in Q6_K)
    t_q: int = T_Q4K
    t_k: int = T_Q4K
    t_v: int = T_Q6K
    t_o: int = T_Q4K
    t_gate: int = T_Q4K
    t_up: int = T_Q4K
    t_down: int = T_Q6K
    t_embd: int = T_Q4K
    t_out: int = T_Q6K
    hd: int = 0  # head dimension when n_heads * head_dim != n_embd (a tensor-parallel rank)

    @property
    def head_dim(self) -> int:
        return self.hd or self.n_embd // self.n_heads


SHAPES = {
    # TinyLlama-1.1B shape
    "tinyllama": ModelShape("tinyllama-1.1b-shape", 22, 2048, 32, 4, 5632, 32000),
    # Llama-3.1-8B shape
    "llama8b": ModelShape("llama-3.1-8b-shape", 32, 4096, 32, 8, 14336, 128256),
    # Llama-3.3-70B shape
    "llama70b": ModelShape("llama-3.3-70b-shape", 80, 8192, 64, 8, 28672, 128256),
    # small shapes for fast tests
    "tiny": ModelShape("tiny", 2, 256, 4, 2, 512, 1000),
    "small": ModelShape("small", 3, 512, 8, 2, 1536, 2048),
    # a Q4/Q5/Q6 mix (as in the reference's 70B Q4_K_M file): Q5_K keys, gate/up,
    # down and output head
    "mix5": ModelShape("mix5", 2, 512, 8, 2, 1536, 2048, t_k=T_Q5K, t_gate=T_Q5K, t_up=T_Q5K,
                       t_down=T_Q5K, t_out=T_Q5K),
}


@dataclasses.dataclass
class LayerWeights:
    attn_norm: np.ndarray
    wq: np.ndarray
    wk: np.ndarray
    wv: np.ndarray
    wo: np.ndarray
    ffn_norm: np.ndarray
    wg: np.ndarray
    wu: np.ndarray
    wd: np.ndarray


@dataclasses.dataclass
class Model:
    shape: ModelShape
    layers: list
    tok_embd: np.ndarray
    output_norm: np.ndarray
    output: np.ndarray

    def digest(self) -> str:
        h = hashlib.sha256()
        for L in self.layers:
            for a in dataclasses.astuple(L):
                h.update(np.ascontiguousarray(a).tobytes())
        for a in (self.tok_embd, self.output_norm, self.output):
            h.update(np.ascontiguousarray(a).tobytes())
        return h.hexdigest()


def make_layer(rng: np.random.Generator, s: ModelShape, conditioned: bool = False) -> LayerWeights:
    D, hd = s.n_embd, s.head_dim

    def qm(t, rows, cols):
        return quant_matrix(rng, t, rows, cols, conditioned)

    return LayerWeights(
        attn_norm=norm_weight(rng, D),
        wq=qm(s.t_q, s.n_heads * hd, D),
        wk=qm(s.t_k, s.n_kv_heads * hd, D),
        wv=qm(s.t_v, s.n_kv_heads * hd, D),
        wo=qm(s.t_o, D, s.n_heads * hd),
        ffn_norm=norm_weight(rng, D),
        wg=qm(s.t_gate, s.n_ff, D),
        wu=qm(s.t_up, s.n_ff, D),
        wd=qm(s.t_down, D, s.n_ff),
    )


def make_model(shape: ModelShape | str, seed: int = 0, n_layers: int | None = None,
               conditioned: bool = False) -> Model:
    """A seeded model of `shape`; conditioned: unit-gain zero-mean weights
    (quant_matrix), so activations and attention scores stay of order one."""
    s = SHAPES[shape] if isinstance(shape, str) else shape
    if n_layers is not None:
        s = dataclasses.replace(s, n_layers=n_layers)
    rng = np.random.default_rng(seed)
    layers = [make_layer(rng, s, conditioned) for _ in range(s.n_layers)]
    # embedding rows of rms ~1 (a 1-column gain), output head of unit gain
    tok = (quant_matrix(rng, s.t_embd, s.n_vocab, s.n_embd, False) if not conditioned else
           _embedding(rng, s.t_embd, s.n_vocab, s.n_embd))
    onorm = norm_weight(rng, s.n_embd)
    out = quant_matrix(rng, s.t_out, s.n_vocab, s.n_embd, conditioned)
    return Model(s, layers, tok, onorm, out)


def _embedding(rng: np.random.Generator, qtype: int, rows: int, cols: int) -> np.ndarray:
    gen = {T_Q4K: q4k_blocks, T_Q5K: q5k_blocks, T_Q6K: q6k_blocks}[qtype]
    blocks = gen(rng, rows * (cols // QK), d_sigma=1.0 / _GAIN[qtype])
    _center(blocks, qtype)
    return blocks.reshape(-1)


def layer_bytes(s: ModelShape) -> int:
    """Bytes of one layer's nine tensors packed at 32-byte alignment
    (engine/src/model_loader.c:181-201)."""
    D, hd = s.n_embd, s.head_dim

    def qb(t, r, c):
        return r * (c // QK) * BLOCK_BYTES[t]

    sizes = [4 * D, qb(s.t_q, s.n_heads * hd, D), qb(s.t_k, s.n_kv_heads * hd, D),
             qb(s.t_v, s.n_kv_heads * hd, D), qb(s.t_o, D, s.n_heads * hd), 4 * D,
             qb(s.t_gate, s.n_ff, D), qb(s.t_up, s.n_ff, D), qb(s.t_down, D, s.n_ff)]
    off = 0
    for sz in sizes:
        off = (off + 31) & ~31
        off += sz
    return off


def token_bytes(s: ModelShape) -> int:
    """Algorithmic weight bytes streamed per decoded token: every layer, the
    output head, and one embedding row."""
    head = s.n_vocab * (s.n_embd // QK) * BLOCK_BYTES[s.t_out]
    embd_row = (s.n_embd // QK) * BLOCK_BYTES[s.t_embd]
    return s.n_layers * layer_bytes(s) + head + embd_row


def kv_bytes_per_pos(s: ModelShape) -> int:
    """Q8_0 K+V bytes read per cached position per token (36-byte blocks)."""
    return s.n_layers * 2 * (s.n_kv_heads * s.head_dim // 32) * 36
