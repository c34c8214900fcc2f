/*
 * oracle.h -- CPU restatement of Shukuchi's batch-1 decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the oracle that the CUDA path
 * (libshk_cuda.so) is compared against.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / reference leg may load it.  The product path
 * never calls into it and has no CPU fallback.
 *
 * Every function restates the algorithm of the reference C engine
 * (JimmyLi-Network/Shukuchi, engine/src/*.c) with the same floating-point
 * expression order, so that with the same compiler flags (-O2, no FMA
 * contraction) its outputs are bit-identical to the reference's.  That claim
 * is pinned by tests/test_oracle.py against golden vectors produced by the
 * reference itself (tests/golden/make_golden.py, oracle/_ref/).
 */
#ifndef SHK_ORACLE_H
#define SHK_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK 256
#define ORC_Q4K_BYTES 144
#define ORC_Q5K_BYTES 176
#define ORC_Q6K_BYTES 210
#define ORC_Q8_BYTES 36 /* {float scale; int8 q[32]} */

/* ggml type ids as stored in GGUF tensor infos */
#define ORC_T_F32 0
#define ORC_T_F16 1
#define ORC_T_Q4K 12
#define ORC_T_Q5K 13
#define ORC_T_Q6K 14

void orc_set_threads(int n);

float orc_half_to_float(uint16_t h);
void orc_dequant_q4k(const void *blocks, float *y, uint32_t k);
void orc_dequant_q5k(const void *blocks, float *y, uint32_t k);
void orc_dequant_q6k(const void *blocks, float *y, uint32_t k);
int orc_matvec(uint32_t dtype, const void *w, const float *x, float *y,
               uint32_t m, uint32_t k);
int orc_rmsnorm(const float *x, const float *w, float *y, uint32_t d);
int orc_rope(float *qk, uint32_t n_heads, uint32_t head_dim, uint32_t pos,
             float theta);
void orc_q8_quantize(const float *x, uint32_t n, void *out_blocks);
void orc_q8_dequantize(const void *in_blocks, uint32_t n, float *out);
int orc_attention(const float *q, const float *k, const float *v, float *out,
                  uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                  uint32_t seq_len, float scale);
void orc_swiglu(const float *gate, const float *up, float *h, uint32_t n);
int orc_embed(const void *table, uint32_t dtype, uint32_t token, float *out,
              uint32_t n_embd);
uint32_t orc_argmax(const float *x, uint32_t n);

/* Q8_0 KV store in the reference's block layout. */
typedef struct orc_kv orc_kv;
orc_kv *orc_kv_create(uint32_t n_layers, uint32_t n_kv_heads, uint32_t head_dim,
                      uint32_t block_size, uint32_t max_seq_len);
void orc_kv_destroy(orc_kv *c);
int orc_kv_append(orc_kv *c, uint32_t layer, uint32_t pos, const float *k,
                  const float *v);
int orc_kv_read_range(orc_kv *c, uint32_t layer, uint32_t start, uint32_t end,
                      float *k_out, float *v_out);
/* raw 36-byte blocks of one token: which = 0 for K, 1 for V */
const void *orc_kv_token_blocks(orc_kv *c, uint32_t layer, uint32_t pos,
                                int which);
void orc_kv_clear(orc_kv *c);
uint32_t orc_kv_seq_len(orc_kv *c, uint32_t layer);

typedef struct orc_layer {
    const float *attn_norm;
    const float *ffn_norm;
    const void *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    uint32_t tq, tk, tv, to, tg, tu, td;
} orc_layer;

typedef struct orc_model {
    uint32_t n_layers, n_embd, n_heads, n_kv_heads, head_dim, n_ff, n_vocab;
    float rope_theta;
    const orc_layer *layers;
    const void *tok_embd;
    uint32_t tok_embd_type;
    const void *output;
    uint32_t output_type;
} orc_model;

int orc_forward_layer(const orc_model *m, orc_kv *kv, uint32_t layer,
                      uint32_t pos, float *hidden);
/* Runs n_prompt prompt tokens then n_decode greedy tokens.  out_tokens gets
 * n_decode ids; out_logits (nullable) gets n_decode x n_vocab floats. */
int orc_generate(const orc_model *m, orc_kv *kv, const uint32_t *prompt,
                 uint32_t n_prompt, uint32_t n_decode, uint32_t *out_tokens,
                 float *out_logits);

#ifdef __cplusplus
}
#endif
#endif
