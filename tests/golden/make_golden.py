"""Generates tests/golden/*.npz from the REFERENCE implementation itself.

The reference's C sources are compiled unmodified into oracle/_ref/libshkref.so
(``make -C oracle ref``, which reads them where oracle/Makefile's REF points).  This script
feeds seeded inputs through the reference entry points (op_matmul_q4_k,
op_matmul_q5_k, op_matmul_q6_k, op_rmsnorm, op_rope, q8_quantize_vec, op_attention, op_embed,
forward_layer_view) and stores inputs and outputs.  The committed fixtures
pin the oracle restatement (tests/test_oracle.py) on machines where the
reference sources are absent.

Usage: python tests/golden/make_golden.py [fixture names]   (default: all)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle_py import Reference, build  # noqa: E402
from shukuchi_b200 import synth  # noqa: E402


def subnormal_scales(blocks: np.ndarray, qtype: int, rng, frac=0.5) -> None:
    """Force a fraction of the fp16 scales to subnormal values (exercise the
    reference's subnormal decoding)."""
    n = blocks.shape[0]
    pick = rng.random(n) < frac
    sub = rng.integers(1, 0x400, size=n).astype(np.uint16)
    if qtype in (synth.T_Q4K, synth.T_Q5K):
        v = blocks[:, 0:2].copy().view(np.uint16).reshape(-1)
        v[pick] = sub[pick]
        blocks[:, 0:2] = v.view(np.uint8).reshape(n, 2)
        v2 = blocks[:, 2:4].copy().view(np.uint16).reshape(-1)
        v2[pick] = sub[::-1][pick]
        blocks[:, 2:4] = v2.view(np.uint8).reshape(n, 2)
    else:
        v = blocks[:, 208:210].copy().view(np.uint16).reshape(-1)
        v[pick] = sub[pick]
        blocks[:, 208:210] = v.view(np.uint8).reshape(n, 2)


def gemv_case(ref, rng, qtype, m, k):
    nb = m * (k // 256)
    blocks = {synth.T_Q4K: synth.q4k_blocks, synth.T_Q5K: synth.q5k_blocks,
              synth.T_Q6K: synth.q6k_blocks}[qtype](rng, nb)
    subnormal_scales(blocks, qtype, rng)
    w = blocks.reshape(-1)
    x = rng.normal(0.0, 1.0, size=k).astype(np.float32)
    y = ref.matvec(qtype, w, x, m, k)
    return dict(w=w, x=x, y=y, m=np.uint32(m), k=np.uint32(k))


def tiny_generate(ref, model, prompt, n_decode):
    """engine_generate's loop (engine/src/engine.c:343-495) on the reference
    forward_layer_view, lm_head through op_matmul_q6_k, first-index argmax."""
    s = model.shape
    h, step = ref.forward_layer_fn(model, max_seq=len(prompt) + n_decode + 1)
    try:
        pos = 0
        for t in prompt:
            hid = ref.embed(model.tok_embd, s.t_embd, int(t), s.n_embd)
            for layer in range(s.n_layers):
                step(layer, pos, hid)
            pos += 1
        toks, logits = [], []
        for _ in range(n_decode):
            lg = ref.matvec(s.t_out, model.output, hid, s.n_vocab, s.n_embd)
            nxt = int(np.argmax(lg))  # numpy argmax also returns the first maximum
            toks.append(nxt)
            logits.append(lg)
            hid = ref.embed(model.tok_embd, s.t_embd, nxt, s.n_embd)
            for layer in range(s.n_layers):
                step(layer, pos, hid)
            pos += 1
        return np.array(toks, np.uint32), np.stack(logits)
    finally:
        ref.L.ref_engine_free(h)


def main(only: list[str] | None = None) -> None:
    build(ref=True)
    ref = Reference()
    rng = np.random.default_rng(1234)
    out = {}
    out["gemv_q4k"] = gemv_case(ref, rng, synth.T_Q4K, 16, 512)
    out["gemv_q6k"] = gemv_case(ref, rng, synth.T_Q6K, 16, 512)
    # Q8_0: random, an all-zero block (scale 1), exact .5 ties, a saturating block
    x = rng.normal(0, 1, size=4 * 32).astype(np.float32)
    x[32:64] = 0.0
    x[64:96] = (np.arange(32, dtype=np.float32) - 16.0) * 0.5 + 0.25
    x[96] = 1e30
    out["q8"] = dict(x=x, blocks=ref.q8_quantize(x))
    w = (1.0 + rng.normal(0, 0.02, 512)).astype(np.float32)
    xr = rng.normal(0, 3, 512).astype(np.float32)
    out["rmsnorm"] = dict(x=xr, w=w, y=ref.rmsnorm(xr, w))
    qk = rng.normal(0, 1, 4 * 64).astype(np.float32)
    out["rope"] = dict(x=qk, y=ref.rope(qk, 4, 64, 37, 10000.0), n_heads=np.uint32(4),
                       head_dim=np.uint32(64), pos=np.uint32(37))
    H, KV, hd, seq = 8, 2, 64, 20
    q = rng.normal(0, 1, H * hd).astype(np.float32)
    k = rng.normal(0, 1, seq * KV * hd).astype(np.float32)
    v = rng.normal(0, 1, seq * KV * hd).astype(np.float32)
    sc = np.float32(1.0 / np.sqrt(hd))
    out["attention"] = dict(q=q, k=k, v=v, out=ref.attention(q, k, v, H, KV, hd, seq, sc),
                            dims=np.array([H, KV, hd, seq], np.uint32))
    table = synth.q4k_blocks(rng, 10 * 2)
    subnormal_scales(table, synth.T_Q4K, rng)
    table = table.reshape(-1)
    out["embed"] = dict(table=table, token=np.uint32(7), out=ref.embed(table, 12, 7, 512))
    model = synth.make_model("tiny", seed=7)
    prompt = np.array([3, 141, 59, 265], np.uint32)
    toks, logits = tiny_generate(ref, model, prompt, 6)
    out["tiny_model"] = dict(seed=np.uint32(7), digest=np.frombuffer(model.digest().encode(), np.uint8),
                             prompt=prompt, tokens=toks, logits=logits)
    # Q5_K (engine/src/ops.c:144-165, 316-359) from its own stream, so adding it
    # left the fixtures above unchanged
    out["gemv_q5k"] = gemv_case(ref, np.random.default_rng(1235), synth.T_Q5K, 16, 512)
    for name, d in out.items():
        if only and name not in only:
            continue
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
        print("wrote", name)


if __name__ == "__main__":
    main(sys.argv[1:] or None)
