/*
 * shk_cuda.h -- C ABI of the B200 (sm_100a) decode path for the Shukuchi engine.
 *
 * This library replaces the reference's Apple Metal backend
 * (engine/include/metal_ops.h:5-26) and adds device-side versions of the ops
 * (engine/include/ops.h:9-38), the Q8_0 KV cache (engine/include/kv_cache.h:5-37)
 * and the per-layer forward (engine/src/engine.c:76-229), so the C engine keeps
 * its model/layer API and CLI while all math runs as hand-written CUDA kernels.
 *
 * Conventions
 *  - Plain C types only.  Pointers named *_dev are device pointers; *_host are
 *    host pointers.  `stream` is a cudaStream_t passed as void* (NULL = the
 *    context's compute stream).
 *  - Every call returns an int status: 0 ok, negative SHK_E* on error.  There is
 *    NO CPU fallback: an error is returned to the caller.
 *  - Device-side waits are bounded; a wait that runs out records SHK_ETIMEOUT
 *    in the context's error word (shk_cuda_check).
 *  - One compute thread per context; shk_cuda_layer_stage may be called from a
 *    separate loader thread (it uses the context's own copy stream).
 *  - Weight tensors are in GGUF block layout: Q4_K (ggml type 12, 144-byte
 *    super-blocks) and Q6_K (type 14, 210-byte super-blocks), rows of k/256
 *    blocks.  Device weight pointers must be 16-byte aligned.
 */
#ifndef SHK_CUDA_H
#define SHK_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum shk_status {
    SHK_OK = 0,
    SHK_EINVAL = -1,       /* bad argument / shape */
    SHK_ENOMEM = -2,       /* device or pinned allocation failed */
    SHK_ECUDA = -3,        /* CUDA runtime error */
    SHK_EUNSUPPORTED = -4, /* dtype or shape not handled (e.g. Q5_K) */
    SHK_ETIMEOUT = -5,     /* a bounded device wait ran out */
    SHK_ENODEV = -6,       /* no usable CUDA device */
    SHK_ENCCL = -7,        /* collective failure */
    SHK_EDEVICE = -8       /* kernel reported an error (bad position/token) */
};

typedef struct shk_ctx shk_ctx;     /* device, streams, error word, counters */
typedef struct shk_kv shk_kv;       /* Q8_0 KV cache in HBM */
typedef struct shk_model shk_model; /* dims, scratch, captured decode step */

struct shk_cuda_config {
    int device;     /* CUDA ordinal; -1 = current device */
    uint32_t flags; /* SHK_CUDA_FLAG_*; 0 = defaults */
};
/* Run whole-token decode (shk_cuda_token_step / shk_cuda_decode_steps) in the
 * persistent decode kernel (one cooperative launch per call, grid-wide
 * barriers between phases) instead of captured graphs of per-projection
 * kernels.  Both give the same results within fp32 rounding. */
#define SHK_CUDA_FLAG_PERSISTENT 2u
/* Capture the decode-step graphs without programmatic dependent launch
 * (each kernel then starts only after its predecessor has finished). */
#define SHK_CUDA_FLAG_NO_PDL 4u

/* ---- context: replaces metal_ops_init/metal_ops_shutdown/metal_available/
 *      metal_ops_report (engine/include/metal_ops.h:5-6, 24-25) ---- */
shk_ctx *shk_cuda_init(const struct shk_cuda_config *cfg);
void shk_cuda_shutdown(shk_ctx *ctx);
int shk_cuda_available(void);
void shk_cuda_report(shk_ctx *ctx);
/* Synchronises the compute stream and returns SHK_ETIMEOUT / SHK_EDEVICE if a
 * kernel recorded a device-side error since the last call (which clears it). */
int shk_cuda_check(shk_ctx *ctx);
const char *shk_cuda_strerror(int status);
void *shk_cuda_stream(shk_ctx *ctx);       /* compute stream (cudaStream_t) */
int shk_cuda_num_sms(shk_ctx *ctx);

/* ---- memory helpers for the engine and loader ---- */
int shk_cuda_dev_alloc(shk_ctx *ctx, size_t bytes, void **out_dev);
int shk_cuda_dev_free(shk_ctx *ctx, void *p_dev);
int shk_cuda_host_alloc(shk_ctx *ctx, size_t bytes, void **out_host); /* pinned */
int shk_cuda_host_free(shk_ctx *ctx, void *p_host);
int shk_cuda_memcpy_h2d(shk_ctx *ctx, void *dst_dev, const void *src_host, size_t bytes, void *stream);
int shk_cuda_memcpy_d2h(shk_ctx *ctx, void *dst_host, const void *src_dev, size_t bytes, void *stream);
int shk_cuda_sync(shk_ctx *ctx, void *stream);

/* ---- dequantise-matvec: replaces metal_matmul_q4k_vec / metal_matmul_q6k_vec
 *      (engine/include/metal_ops.h:7-23) as called from op_matmul_q4_k /
 *      op_matmul_q6_k (engine/src/ops.c:266-314, 361-404).
 *      y[r] = sum_k dequant(W[r,k]) * x[k], W m x k, k % 256 == 0.  Async. ---- */
int shk_cuda_matmul_q4k_vec(shk_ctx *ctx, const void *w_dev, const float *x_dev, float *y_dev,
                            uint32_t m, uint32_t k, void *stream);
int shk_cuda_matmul_q6k_vec(shk_ctx *ctx, const void *w_dev, const float *x_dev, float *y_dev,
                            uint32_t m, uint32_t k, void *stream);
/* replaces metal_matmul_q5k_vec (engine/include/metal_ops.h:5-26) as called
 * from op_matmul_q5_k (engine/src/ops.c:316-359).  W is in the reference's
 * 176-byte Q5_K block layout {u16 d, u16 dmin, u8 scales[12], u8 qh[32],
 * u8 qs[128]}, element i of a block = low nibble (i even) / high nibble (i odd)
 * of qs[i/2] plus bit i%8 of qh[i/8] as the fifth bit (dequantize_row_q5_k,
 * :144-165), rows dense; w_dev and x_dev 16-byte aligned.  Async. */
int shk_cuda_matmul_q5k_vec(shk_ctx *ctx, const void *w_dev, const float *x_dev, float *y_dev,
                            uint32_t m, uint32_t k, void *stream);

/* ---- Q6_K weight layout in HBM.  No counterpart in the reference (its
 *      weights stay in the GGUF layout in host memory).  The staged GEMV reads
 *      Q6_K rows in a planar layout: the same 210 * k/256 bytes of a row
 *      regrouped as [ql of every block][qh][scales][d], each plane 16-byte
 *      aligned, with the 16-byte chunks of a block rotated by the block index
 *      (ql chunk c of block b at 128 b + 16 ((c + b) & 7), qh chunk c at
 *      128 nb + 64 b + 16 ((c + (b >> 1)) & 3), scales at 192 nb + 16 b, d at
 *      208 nb + 2 b).  Weights registered with a model as Q6_K must be in this
 *      layout and carry dtype SHK_DTYPE_Q6_K_PLANAR (output head: GGUF Q6_K is
 *      also accepted, on the plain-load kernel). ---- */
#define SHK_DTYPE_Q6_K_PLANAR 0x10Eu
/* Converts `rows` Q6_K rows of k elements, row_stride bytes apart (0 = 210 *
 * k/256; must be a multiple of 16 and at most 227 KB), in place: to the
 * planar layout (to_planar != 0) or back to GGUF blocks.  Async on stream. */
int shk_cuda_q6k_repack(shk_ctx *ctx, void *w_dev, uint32_t rows, uint32_t k, uint32_t row_stride,
                        int to_planar, void *stream);
/* ---- Row-tiled weight layout for the tensor-core matvec.  No counterpart in
 *      the reference (its weights stay GGUF blocks in host memory, read by
 *      op_matmul_q4_k / op_matmul_q6_k, engine/src/ops.c:266-314, 361-404).
 *      A matrix of `rows` rows and nb = k/256 super-blocks becomes ceil(rows/16)
 *      row tiles; tile (row tile t, block b) holds block b of rows 16t..16t+15
 *      (rows past `rows` are zero) at byte (t * nb + b) * tile_bytes, tile_bytes
 *      = 16 * 144 (Q4_K) or 16 * 210 (Q6_K).  Inside a tile the GGUF bytes are
 *      only moved, into the order the tensor-core fragments read them:
 *        Q4_K: [0,256) the 16 rows' 16-byte block headers (d, dmin, scales);
 *              [256,2304) [chunk j<4][lane<32][16]: row g = lane/4 quant bytes
 *              32j + 8(lane%4) .. +7, then row g+8's.
 *        Q6_K: [0,3072) [half n<2][lane<32][48]: row g ql bytes 64n + 8t..+7,
 *              ql 64n+32+8t..+7, qh 32n+8t..+7 (t = lane%4), then row g+8's;
 *              [3072,3328) int8 scales[16] per row; [3328,3360) fp16 d per row.
 *      Weights registered as SHK_DTYPE_Q4_K_TILED / SHK_DTYPE_Q6_K_TILED run on
 *      the tensor-core matvec (mma.sync int8 over fixed-point x limbs). ---- */
#define SHK_DTYPE_Q4_K_TILED 0x20Cu
#define SHK_DTYPE_Q6_K_TILED 0x20Eu
/* Bytes of the tiled form of a rows x k matrix of dtype 12/14 (or a tiled
 * dtype); 0 for other dtypes or k not a multiple of 256. */
size_t shk_cuda_tiled_bytes(uint32_t dtype, uint32_t rows, uint32_t k);
/* GGUF rows (dtype 12 or 14, src_row_stride bytes apart, 0 = dense) -> the
 * tiled layout at dst_dev (shk_cuda_tiled_bytes bytes, 16-byte aligned, not
 * overlapping src).  Async on stream. */
int shk_cuda_tile(shk_ctx *ctx, uint32_t dtype, const void *src_dev, uint32_t src_row_stride, uint32_t rows,
                  uint32_t k, void *dst_dev, void *stream);
/* ---- batched prefill matmul on the tensor cores.  No counterpart in the
 *      reference, which feeds prompt tokens one at a time
 *      (engine/src/engine.c:306-501); this is the contraction those n_tokens
 *      op_matmul_q4_k / op_matmul_q6_k calls (engine/src/ops.c:266-314,
 *      361-404) add up to: y[t][r] = sum_k W[r][k] * x[t][k] for t <
 *      n_tokens, x fp32 [n_tokens][k], y fp32 [n_tokens][m].  Weights are
 *      dequantised to f16 tiles, each token row of x is scaled by a power of
 *      two (largest magnitude to [2^14, 2^15)) and rounded to f16, and the
 *      product runs f16 x f16 -> fp32 on tcgen05.mma (accumulators in TMEM),
 *      the scale put back exactly: results carry the f16 rounding of the
 *      inputs (2^-11 relative each).  dtype 12 (Q4_K) or
 *      SHK_DTYPE_Q6_K_PLANAR; row_stride 0 = dense rows.  Async on stream. ---- */
int shk_cuda_prefill_matmul(shk_ctx *ctx, uint32_t dtype, const void *w_dev, uint32_t row_stride,
                            const float *x_dev, float *y_dev, uint32_t m, uint32_t k, uint32_t n_tokens,
                            void *stream);
/* dequantise-matvec by dtype: 12 (Q4_K), 13 (Q5_K), 14 (GGUF Q6_K),
 * SHK_DTYPE_Q6_K_PLANAR, SHK_DTYPE_Q4_K_TILED or SHK_DTYPE_Q6_K_TILED;
 * row_stride 0 = dense rows (ignored for tiled weights; Q5_K rows must be
 * dense). */
int shk_cuda_matvec(shk_ctx *ctx, uint32_t dtype, const void *w_dev, uint32_t row_stride,
                    const float *x_dev, float *y_dev, uint32_t m, uint32_t k, void *stream);
/* Same contract as metal_matmul_q{4,6}k_vec: HOST weights/x/y, synchronous
 * (copies in, computes, copies out).  For callers that keep the reference's
 * host-resident layer buffers unchanged. */
int shk_cuda_matmul_q4k_vec_host(shk_ctx *ctx, const void *w_host, const float *x_host,
                                 float *y_host, uint32_t m, uint32_t k);
int shk_cuda_matmul_q6k_vec_host(shk_ctx *ctx, const void *w_host, const float *x_host,
                                 float *y_host, uint32_t m, uint32_t k);
int shk_cuda_matmul_q5k_vec_host(shk_ctx *ctx, const void *w_host, const float *x_host,
                                 float *y_host, uint32_t m, uint32_t k);

/* ---- op-level glue on device (engine/include/ops.h:9-38) ---- */
/* op_rmsnorm, n = 1 (engine/src/ops.c:195-214) */
int shk_cuda_rmsnorm(shk_ctx *ctx, const float *x_dev, const float *w_dev, float *y_dev,
                     uint32_t d, void *stream);
/* op_rope (engine/src/ops.c:216-238); in place */
int shk_cuda_rope(shk_ctx *ctx, float *qk_dev, uint32_t n_heads, uint32_t head_dim, uint32_t pos,
                  float rope_theta, void *stream);
/* SwiGLU of op_mlp_swiglu (engine/src/ops.c:491-496) */
int shk_cuda_swiglu(shk_ctx *ctx, const float *gate_dev, const float *up_dev, float *h_dev,
                    uint32_t n, void *stream);
/* op_embed for one token, Q4_K (12) or F16 (1) table (engine/src/ops.c:533-577) */
int shk_cuda_embed(shk_ctx *ctx, const void *table_dev, uint32_t dtype, uint32_t n_vocab,
                   uint32_t token, float *out_dev, uint32_t n_embd, void *stream);
/* first-index argmax (engine/src/engine.c:424-431); result to host.
 * n must be 1..0xFFFFFFFE (SHK_ARGMAX_NOALLOC_MAX_N below); else SHK_EINVAL. */
int shk_cuda_argmax(shk_ctx *ctx, const float *x_dev, uint32_t n, uint32_t *out_host);

/* ---- Q8_0 KV cache in HBM (engine/include/kv_cache.h:11-37).  Quantisation
 *      is bit-identical to q8_quantize_vec (engine/src/kv_cache.c:28-55). ---- */
struct shk_kv_config {
    uint32_t n_layers;
    uint32_t n_kv_heads;
    uint32_t head_dim; /* 64 or 128 */
    uint32_t block_size; /* kept for API parity; storage is per position */
    uint32_t max_seq_len; /* not capped at 2048 */
};
shk_kv *shk_cuda_kv_create(shk_ctx *ctx, const struct shk_kv_config *cfg);
void shk_cuda_kv_destroy(shk_kv *kv);
/* kv_cache_append (engine/src/kv_cache.c:130-155); k/v: n_kv*head_dim fp32 */
int shk_cuda_kv_append(shk_kv *kv, uint32_t layer, uint32_t pos, const float *k_dev,
                       const float *v_dev, void *stream);
/* kv_cache_append for positions start..start+n-1 in one launch, as the
 * reference's prefill loop appends them one by one (engine/src/engine.c:352-380
 * via forward_layer_view :133); k/v: n rows of n_kv*head_dim fp32 */
int shk_cuda_kv_append_range(shk_kv *kv, uint32_t layer, uint32_t start, uint32_t n,
                             const float *k_dev, const float *v_dev, void *stream);
/* kv_cache_read_range (engine/src/kv_cache.c:175-199): fp32 [pos][n_kv*hd] */
int shk_cuda_kv_read_range(shk_kv *kv, uint32_t layer, uint32_t start, uint32_t end,
                           float *k_dev, float *v_dev, void *stream);
/* raw 36-byte {float scale; int8 q[32]} blocks, reference order
 * [pos][n_kv*hd/32] -- for byte-exact comparisons */
int shk_cuda_kv_read_blocks(shk_kv *kv, uint32_t layer, uint32_t start, uint32_t end,
                            void *k_dev, void *v_dev, void *stream);
/* kv_cache_read_range + op_attention over positions [0, seq_len) fused on the
 * Q8_0 cache (engine/src/engine.c:137-158, engine/src/ops.c:406-461).  If
 * k_new_dev/v_new_dev are non-NULL they are first appended at seq_len-1. */
int shk_cuda_kv_attend(shk_kv *kv, uint32_t layer, const float *q_dev, const float *k_new_dev,
                       const float *v_new_dev, float *out_dev, uint32_t n_heads, uint32_t seq_len,
                       float scale, void *stream);
/* shk_cuda_kv_attend for n_seq sequences in one launch -- the KV
 * microbenchmark's batch of decode streams (no counterpart in the reference,
 * which decodes one sequence): sequence z appends to and attends cache layer
 * layer0 + z with q / out rows at z * n_heads * hd floats and k_new / v_new
 * rows at z * n_kv * hd; every sequence at seq_len.  Scratch for the split
 * partials grows on the first call of a larger n_seq (make that call outside
 * graph capture). */
int shk_cuda_kv_attend_batch(shk_kv *kv, uint32_t layer0, uint32_t n_seq, const float *q_dev,
                             const float *k_new_dev, const float *v_new_dev, float *out_dev,
                             uint32_t n_heads, uint32_t seq_len, float scale, void *stream);
/* kv_cache_clear / kv_cache_get_seq_len (engine/src/kv_cache.c:230-248) */
void shk_cuda_kv_clear(shk_kv *kv);
uint32_t shk_cuda_kv_seq_len(shk_kv *kv, uint32_t layer);

/* ---- model: per-layer forward, embed, lm_head+argmax, captured decode step ---- */
struct shk_model_desc {            /* struct model_info (model_loader.h:66-74) + resident */
    uint32_t n_layers, n_embd, n_heads, n_kv_heads, head_dim, n_ff, n_vocab;
    float rope_theta;              /* 0 -> 10000, as engine/src/engine.c:86 */
    const void *tok_embd_dev;      /* token_embd, resident */
    uint32_t tok_embd_dtype;
    const void *output_dev;        /* output (lm_head), resident */
    uint32_t output_dtype;
};
struct shk_layer_desc {            /* struct layer_view (model_loader.h:28-56), DEVICE pointers */
    const float *attn_norm, *ffn_norm;
    const void *attn_q, *attn_k, *attn_v, *attn_o, *ffn_gate, *ffn_up, *ffn_down;
    uint32_t attn_q_dtype, attn_k_dtype, attn_v_dtype, attn_o_dtype;
    uint32_t ffn_gate_dtype, ffn_up_dtype, ffn_down_dtype;
    uint32_t row_stride_v, row_stride_down; /* 0 = dense rows; else padded row bytes */
};
shk_model *shk_cuda_model_create(shk_ctx *ctx, const struct shk_model_desc *desc, shk_kv *kv);
void shk_cuda_model_destroy(shk_model *m);
/* Registers device weights of a layer for the captured whole-token step. */
int shk_cuda_model_set_layer(shk_model *m, uint32_t layer, const struct shk_layer_desc *lv);
/* forward_layer_view (engine/src/engine.c:76-229) on device-resident weights:
 * hidden_dev (n_embd fp32) is updated in place; K/V appended at pos. */
int shk_cuda_forward_layer(shk_model *m, const struct shk_layer_desc *lv, uint32_t layer,
                           uint32_t pos, float *hidden_dev, void *stream);
/* op_embed(token) into the model's hidden state */
int shk_cuda_model_embed(shk_model *m, uint32_t token, void *stream);
/* lm_head on the raw residual (no final norm, engine/src/engine.c:403-422) and
 * first-index argmax.  logits_host may be NULL. */
int shk_cuda_model_lm_head(shk_model *m, uint32_t *token_host, float *logits_host, void *stream);
float *shk_cuda_model_hidden(shk_model *m); /* device pointer to hidden[n_embd] */
/* One whole token through embed -> all layers (-> lm_head -> argmax when
 * want_next) as one captured CUDA graph.  token and pos come from the host;
 * the next token (and logits if logits_host != NULL) are copied back.  All
 * layers must be registered with shk_cuda_model_set_layer. */
int shk_cuda_token_step(shk_model *m, uint32_t token, uint32_t pos, int want_next,
                        uint32_t *next_host, float *logits_host);
/* Device-only decode steps: token and position stay on the device (argmax
 * feeds the next embed, position auto-increments).  Used for throughput. */
int shk_cuda_decode_steps(shk_model *m, uint32_t first_token, uint32_t first_pos, uint32_t n_steps,
                          void *stream);
int shk_cuda_model_token(shk_model *m, uint32_t *token_host); /* last argmax */
/* Batched prompt prefill: tokens[0..n) (host) at positions pos0.. run through
 * every layer as T = n rows at a time -- the projections on the tensor-core
 * matmul (shk_cuda_prefill_matmul: f16 operands, fp32 accumulation), RMSNorm,
 * RoPE, SwiGLU and residuals row-batched, the n K/V rows appended to the
 * Q8_0 cache in one launch per layer and every row's causal attention over
 * [0, pos0 + row] -- then the output head on the last row: its argmax to
 * *next_host (and its logits to logits_host when non-NULL).  The reference
 * feeds the prompt one token at a time (engine/src/engine.c:343-394); this is
 * the same computation with f16 rounding of the matmul inputs, so logits
 * differ from the token-by-token path by that rounding.  Weights must be
 * Q4_K or planar Q6_K (else SHK_EUNSUPPORTED: feed the prompt through
 * shk_cuda_token_step); single GPU. */
int shk_cuda_prefill(shk_model *m, const uint32_t *tokens_host, uint32_t n, uint32_t pos0,
                     uint32_t *next_host, float *logits_host, void *stream);
/* Timeline of the persistent decode kernel, for profiling (no counterpart in
 * the reference, whose CPU loop has no phases).  shk_cuda_model_trace_enable
 * (m, n) makes the following token_step / decode_steps launches record, on
 * CTA 0, %globaltimer (ns) at the start and at the arrival at / departure from
 * the grid barrier after each of the first n phases (n = 0 turns it off).
 * shk_cuda_model_trace_read copies up to cap values of the last launch
 * ([start, arrive_0, leave_0, arrive_1, ...]) and returns how many it wrote, or
 * a negative status.  Phases per token: embed, 5 per layer (QKV, attention, O,
 * gate/up, down), lm_head, argmax. */
int shk_cuda_model_trace_enable(shk_model *m, uint32_t n_phases);
int shk_cuda_model_trace_read(shk_model *m, uint64_t *out_host, uint32_t cap);
/* Profiling hook: enqueue one part of a registered layer's step at the device
 * position of the last step (part 0 RMSNorm+QKV+RoPE GEMV, 1 append+attention,
 * 2 O-proj+residual, 3 RMSNorm+gate/up+SwiGLU, 4 down+residual; 5 = lm_head
 * GEMV, layer ignored).  Returns the algorithmic bytes of that launch's
 * weights in *bytes_out (nullable). */
int shk_cuda_model_launch_part(shk_model *m, uint32_t layer, uint32_t part, void *stream,
                               uint64_t *bytes_out);

/* ---- layer streaming: pinned staging -> HBM on the context's copy stream
 *      (replaces the host-only prefetch ring, engine/src/prefetch.c:39-280) ---- */
/* Queue an async H2D copy of a staged layer blob into dst_dev and record the
 * completion event of `slot`.  Callable from the loader thread. */
int shk_cuda_layer_stage(shk_ctx *ctx, uint32_t slot, void *dst_dev, const void *pinned_src,
                         size_t bytes);
/* Strided variant: rows of src_row_bytes copied to rows of dst_row_bytes
 * (pads Q6_K rows to 16-byte multiples). */
int shk_cuda_layer_stage_rows(shk_ctx *ctx, uint32_t slot, void *dst_dev, size_t dst_row_bytes,
                              const void *pinned_src, size_t src_row_bytes, size_t rows);
/* General strided copy: `rows` runs of `width` bytes, src_pitch apart in the
 * pinned blob, to dst_pitch apart in HBM -- a tensor-parallel rank's column
 * shard of a matrix (its block range of every row) or its row range.  No
 * counterpart in the reference (it has no tensor parallelism). */
int shk_cuda_layer_stage_2d(shk_ctx *ctx, uint32_t slot, void *dst_dev, size_t dst_pitch,
                            const void *pinned_src, size_t src_pitch, size_t width, size_t rows);
/* Converts Q6_K rows just staged into dst_dev (rows x k elements, row_stride
 * bytes apart, 0 = dense) to the planar layout, in place, on the copy stream
 * after the slot's copies; the slot's commit covers it.  Callable from the
 * loader thread.  No counterpart in the reference. */
int shk_cuda_layer_stage_q6k_planar(shk_ctx *ctx, uint32_t slot, void *dst_dev, uint32_t rows, uint32_t k,
                                    uint32_t row_stride);
/* Marks the end of a slot's staging sequence (records its event). */
int shk_cuda_layer_commit(shk_ctx *ctx, uint32_t slot);
/* 1 if the slot's copies completed, 0 if still in flight (wait = 0), or block
 * until complete (wait != 0). */
int shk_cuda_layer_ready(shk_ctx *ctx, uint32_t slot, int wait);
/* Make `stream` wait (on the device) for the slot's copies. */
int shk_cuda_layer_wait(shk_ctx *ctx, uint32_t slot, void *stream);
/* Device-slot reuse (prefetcher_release, engine/src/prefetch.c:262-280): the
 * next staging into `slot` first waits, on the copy stream, for the work
 * queued on `stream` so far -- the kernels that read the slot's old layer. */
int shk_cuda_layer_release(shk_ctx *ctx, uint32_t slot, void *stream);

/* ---- failure detection.  No counterpart in the reference (its only device
 *      path is synchronous Metal).  Every device wait in this library is
 *      bounded; on expiry the kernel records a timeout and returns, and the
 *      next status check reports SHK_ETIMEOUT.  This launches one wait that
 *      nothing satisfies (an mbarrier that never completes) with a budget of
 *      budget_us microseconds (at most 1 s): it returns SHK_ETIMEOUT and the
 *      context stays usable. ---- */
int shk_cuda_selftest_wait_timeout(shk_ctx *ctx, uint32_t budget_us);

/* ---- tensor parallelism over the GPUs of one node: NCCL all-reduce over
 *      NVLink after the O and down projections (layout: Wq/Wk/Wv/
 *      gate/up split by output rows, Wo/down by input columns, KV heads local
 *      to a rank).  No counterpart in the reference (single device). ---- */
#define SHK_TP_ID_BYTES 128
/* Rank 0 creates the communicator id (returns its size); the caller passes
 * it to every rank, which then calls shk_cuda_tp_init before creating its
 * model.  NCCL is loaded at first use (libnccl.so.2). */
int shk_cuda_tp_unique_id(void *out, size_t cap);
int shk_cuda_tp_init(shk_ctx *ctx, int rank, int world, const void *id);
/* Ranks in the context's NCCL communicator (ncclCommCount): world after
 * shk_cuda_tp_init, 1 without one; negative on error.  No counterpart in the
 * reference (which has no tensor parallelism). */
int shk_cuda_tp_comm_size(shk_ctx *ctx);
/* This rank computes rows [o_lo, o_hi) of the O projection (its attn_o
 * weights have o_hi - o_lo rows; ranks that share attention heads split the
 * rows) and rows [v_lo, v_hi) of the output head (its output weights have
 * v_hi - v_lo rows).  The head is either replicated (0, n_vocab) or split in
 * equal slices in rank order (v_lo = rank * n_vocab / world); a split head's
 * argmax is merged over the ranks, and a logits copy to the host gathers the
 * slices first, so every rank must ask for logits on the same steps.
 * Default: all rows.  Call after shk_cuda_tp_init and before
 * shk_cuda_model_set_layer. */
int shk_cuda_model_set_tp_rows(shk_model *m, uint32_t o_lo, uint32_t o_hi, uint32_t v_lo, uint32_t v_hi);

/* Tensor-parallel all-reduce over NVLink peer memory instead of NCCL: the O
 * and down GEMVs send their partial output rows straight into every rank's
 * exchange buffer (plain peer stores) and raise a per-rank flag; the next
 * GEMV waits for the flags (bounded), adds the residual and the partials in
 * rank order and proceeds -- no collective kernel between them.  Setup, after
 * shk_cuda_model_set_tp_rows and before shk_cuda_model_set_layer: every rank
 * exports its buffer's IPC handle (64 bytes, returned size), the caller
 * gathers them in rank order and every rank imports the set together with
 * every rank's O rows (o_ranges: world x {o_lo, o_hi}).  The ranks must run
 * on separate GPUs of one node, one process per GPU (CUDA IPC).  NCCL is
 * still used for the vocabulary-split argmax.  No counterpart in the
 * reference. */
int shk_cuda_model_tp_p2p_export(shk_model *m, void *handle_out, size_t cap);
int shk_cuda_model_tp_p2p_import(shk_model *m, const void *handles, const uint32_t *o_ranges);

/* Tensor-parallel all-reduce over NVLink peer memory with the flags in the
 * data words, replacing the NCCL all-reduce after O and down: every rank
 * stores its partial row as 8-byte {value, step} words into every rank's
 * exchange buffer, then sums the ranks' rows from its own buffer in rank
 * order once each word carries the current step (bounded waits).  One small
 * kernel per all-reduce, inside the captured decode step.  Setup, after
 * shk_cuda_model_set_tp_rows and before the first token step: every rank
 * exports its buffer's IPC handle (64 bytes), the caller gathers them in rank
 * order and every rank imports the set.  One process per GPU of one node.  No
 * counterpart in the reference (which has no tensor parallelism). */
int shk_cuda_model_tp_ll_export(shk_model *m, void *handle_out, size_t cap);
int shk_cuda_model_tp_ll_import(shk_model *m, const void *handles);

/* ---- argmax without any device allocation.  No counterpart in the reference:
 *      it exists for callers that cannot call cudaMalloc (a sampler inside a
 *      host runtime that has already reserved the device's memory in its own
 *      pool, or code that holds only device pointers and a stream, no shk_ctx).
 *
 * Writes the first index of the maximum of x_dev[0..n) to *out_dev (device
 * memory), on `stream` (a cudaStream_t; NULL = the legacy default stream), on
 * the CURRENT device.  Same result as shk_cuda_argmax.  Asynchronous: read
 * *out_dev after the stream has been synchronised.
 *  - Scratch is a fixed 2304-byte array in the library's device image (block
 *    partials + merge ticket); every GPU that loads the library holds it until
 *    the process exits.  No cudaMalloc / cudaFree is called.
 *  - The first call in each CUDA context (one per device for runtime-API
 *    callers; a new one after cudaDeviceReset or under a caller's own driver
 *    context) looks up the array's device address in that context (set-up
 *    under a lock, cached by the context's unique id); make that first call
 *    before any stream capture.
 *  - All calls on a device share the array: calls whose kernels overlap on the
 *    GPU (e.g. on two streams at once) race and give wrong results.
 *  - n must be 1..SHK_ARGMAX_NOALLOC_MAX_N; larger or zero n returns
 *    SHK_EINVAL without launching anything. ---- */
#define SHK_ARGMAX_NOALLOC_MAX_N 0xFFFFFFFEu
int shk_cuda_argmax_noalloc(const float *x_dev, uint32_t n, uint32_t *out_dev, void *stream);

#ifdef __cplusplus
}
#endif
#endif
