"""Tensor-parallel layout and weight sharding (host side).

Layout for `world` ranks (a Megatron-style split): Wq/Wk/Wv and gate/up are cut
by output rows, Wo and down by input columns, KV heads stay local to a rank;
one all-reduce after the O projection and one after down.

The output head is split by vocabulary rows in equal slices when n_vocab
divides by `world` (each rank takes the first maximum of its slice and the
pairs are merged in rank order), else replicated.  Embedding and norms are
replicated.

Query head h reads KV head h % n_kv (engine/src/ops.c:421), so a rank that
owns KV heads [kv_lo, kv_hi) owns the query heads whose h % n_kv falls there;
they are stored in the order (group g, KV head j) -> local head g*kvp + j, for
which the local `h % kvp` mapping is again right.  Wo columns of those heads
must be whole 256-element blocks: when one KV head per rank would leave
128-wide column groups (e.g. 8 KV heads, head_dim 128, 8 ranks), ranks are
paired into attention groups of A ranks that share the heads and split the
O projection's output rows instead (each computes D/A rows; the other rows
are zero in its partial sum).
"""
from __future__ import annotations

import dataclasses

import numpy as np

from .synth import BLOCK_BYTES, QK, LayerWeights, Model, ModelShape


@dataclasses.dataclass
class RankLayout:
    rank: int
    world: int
    group_size: int          # ranks sharing the same attention heads (A)
    kv_lo: int
    kv_hi: int
    q_heads: list            # global query heads in local order
    o_lo: int                # rows of the O projection this rank computes
    o_hi: int
    f_lo: int                # FFN columns (gate/up rows, down columns)
    f_hi: int
    v_lo: int                # output-head rows (vocabulary slice)
    v_hi: int


def layout(s: ModelShape, rank: int, world: int) -> RankLayout:
    hd = s.head_dim
    if world < 1 or s.n_ff % QK or s.n_ff // QK < world:
        raise ValueError(f"n_ff {s.n_ff} does not split into {world} ranks of whole blocks")
    for A in (a for a in range(1, world + 1) if world % a == 0):
        if (s.n_kv_heads * A) % world or s.n_embd % A:
            continue
        kvp = s.n_kv_heads * A // world
        # Wo column groups of whole 256-element blocks (all heads: one range)
        if (kvp * hd) % QK == 0 or (kvp == s.n_kv_heads and (s.n_heads * hd) % QK == 0):
            break
    else:
        raise ValueError(f"{s.n_kv_heads} KV heads of dim {hd} have no block-aligned split over {world} ranks")
    g, a = rank // A, rank % A
    kv_lo, kv_hi = g * kvp, (g + 1) * kvp
    G = s.n_heads // s.n_kv_heads
    q_heads = [gg * s.n_kv_heads + kv_lo + j for gg in range(G) for j in range(kvp)]
    rows = s.n_embd // A
    # FFN columns in whole 256-blocks, as even as the block count allows
    fb = s.n_ff // QK
    f_lo = (rank * fb // world) * QK
    f_hi = ((rank + 1) * fb // world) * QK
    if s.n_vocab % world == 0:
        vw = s.n_vocab // world
        v_lo, v_hi = rank * vw, (rank + 1) * vw
    else:
        v_lo, v_hi = 0, s.n_vocab
    return RankLayout(rank, world, A, kv_lo, kv_hi, q_heads, a * rows, (a + 1) * rows,
                      f_lo, f_hi, v_lo, v_hi)


def local_shape(s: ModelShape, lay: RankLayout) -> ModelShape:
    kvp = lay.kv_hi - lay.kv_lo
    return dataclasses.replace(s, n_heads=len(lay.q_heads), n_kv_heads=kvp, n_ff=lay.f_hi - lay.f_lo,
                               hd=s.head_dim)


def _rows(w: np.ndarray, t: int, n_rows: int, cols: int, sel) -> np.ndarray:
    rb = (cols // QK) * BLOCK_BYTES[t]
    m = w.reshape(n_rows, rb)
    return np.ascontiguousarray(m[sel]).reshape(-1)


def _cols(w: np.ndarray, t: int, n_rows: int, cols: int, col_ranges) -> np.ndarray:
    """Whole 256-column blocks [c0, c1) of every row, ranges concatenated."""
    bb = BLOCK_BYTES[t]
    m = w.reshape(n_rows, (cols // QK) * bb)
    parts = []
    for c0, c1 in col_ranges:
        assert c0 % QK == 0 and c1 % QK == 0
        parts.append(m[:, (c0 // QK) * bb:(c1 // QK) * bb])
    return np.ascontiguousarray(np.concatenate(parts, axis=1)).reshape(-1)


def _merge(ranges):
    out = []
    for a, b in ranges:
        if out and out[-1][1] == a:
            out[-1] = (out[-1][0], b)
        else:
            out.append((a, b))
    return out


def shard_layer(L: LayerWeights, s: ModelShape, lay: RankLayout) -> LayerWeights:
    hd, D = s.head_dim, s.n_embd
    qrows = np.concatenate([np.arange(h * hd, (h + 1) * hd) for h in lay.q_heads])
    kvrows = np.arange(lay.kv_lo * hd, lay.kv_hi * hd)
    frows = np.arange(lay.f_lo, lay.f_hi)
    kvp = lay.kv_hi - lay.kv_lo
    G = s.n_heads // s.n_kv_heads
    ocols = _merge([((gg * s.n_kv_heads + lay.kv_lo) * hd, (gg * s.n_kv_heads + lay.kv_lo + kvp) * hd)
                    for gg in range(G)])
    wo_rows = _rows(L.wo, s.t_o, D, s.n_heads * hd, np.arange(lay.o_lo, lay.o_hi))
    return LayerWeights(
        attn_norm=L.attn_norm.copy(),
        wq=_rows(L.wq, s.t_q, s.n_heads * hd, D, qrows),
        wk=_rows(L.wk, s.t_k, s.n_kv_heads * hd, D, kvrows),
        wv=_rows(L.wv, s.t_v, s.n_kv_heads * hd, D, kvrows),
        wo=_cols(wo_rows, s.t_o, lay.o_hi - lay.o_lo, s.n_heads * hd, ocols),
        ffn_norm=L.ffn_norm.copy(),
        wg=_rows(L.wg, s.t_gate, s.n_ff, D, frows),
        wu=_rows(L.wu, s.t_up, s.n_ff, D, frows),
        wd=_cols(L.wd, s.t_down, D, s.n_ff, [(lay.f_lo, lay.f_hi)]),
    )


def shard_model(model: Model, rank: int, world: int) -> tuple[Model, RankLayout]:
    """This rank's model: sharded layers and output-head rows; embedding and
    norms replicated.  The local shape keeps the full n_vocab (the embedding
    table is whole); the output matrix has v_hi - v_lo rows."""
    s = model.shape
    lay = layout(s, rank, world)
    layers = [shard_layer(L, s, lay) for L in model.layers]
    out = _rows(model.output, s.t_out, s.n_vocab, s.n_embd, np.arange(lay.v_lo, lay.v_hi))
    return Model(local_shape(s, lay), layers, model.tok_embd, model.output_norm, out), lay


def rank_token_bytes(s: ModelShape, lay: RankLayout) -> tuple[int, int]:
    """Algorithmic bytes one rank streams per decoded token: (weights of its
    shard incl. norms, output-head rows and one embedding row; Q8_0 K+V bytes
    per cached position of its KV heads)."""
    loc = local_shape(s, lay)
    D, hd = s.n_embd, s.head_dim

    def qb(t, r, c):
        return r * (c // QK) * BLOCK_BYTES[t]

    qd, kvd = loc.n_heads * hd, loc.n_kv_heads * hd
    layer = (8 * D + qb(s.t_q, qd, D) + qb(s.t_k, kvd, D) + qb(s.t_v, kvd, D)
             + qb(s.t_o, lay.o_hi - lay.o_lo, qd) + qb(s.t_gate, loc.n_ff, D) + qb(s.t_up, loc.n_ff, D)
             + qb(s.t_down, D, loc.n_ff))
    w = s.n_layers * layer + qb(s.t_out, lay.v_hi - lay.v_lo, D) + (D // QK) * BLOCK_BYTES[s.t_embd]
    kv = s.n_layers * 2 * (kvd // 32) * 36
    return w, kv
