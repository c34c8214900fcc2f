/* engine.h -- the Shukuchi engine API (engine/include/engine.h of the
 * reference: same functions, same structs) running its decode on the B200
 * path of libshk_cuda.so.
 *
 * Model files are GGUF (llama architecture, Q4_K / Q5_K / Q6_K weights, F32
 * norms).
 * Layer weights reach HBM through the streaming loader: a loader thread
 * pread()s each layer's contiguous span into pinned host staging (depth
 * `prefetch_depth`, 2 or 3 buffers) and queues cudaMemcpyAsync copies into
 * device memory on the context's copy stream; the engine thread makes its
 * compute stream wait on the copy events (no host polling).
 *
 * Options that the reference's config struct has no room for come from the
 * environment:
 *   SHUKUCHI_DEVICE        CUDA ordinal (default 0)
 *   SHUKUCHI_HBM_RESIDENT  1 (default): every layer is staged once into a
 *                          permanent device buffer and decode runs as one
 *                          captured graph per token; 0: layers stream through
 *                          prefetch_depth device slots on every token, as the
 *                          reference streams them from disk
 *   SHUKUCHI_MAX_SEQ       KV-cache capacity in positions (default 2048)
 *   SHUKUCHI_TP            1 (default), 2, 4 or 8: tensor parallel over GPUs
 *                          SHUKUCHI_DEVICE.. +TP-1, one context and thread per
 *                          rank, NCCL between them; Wq/Wk/Wv and gate/up split
 *                          by output rows, Wo and down by input columns, KV
 *                          heads local to a rank, the output head by vocabulary
 *                          rows; resident mode only (each layer is read once
 *                          and every rank copies its slices).  engine_cancel
 *                          takes effect at the end of a generation here
 *   SHUKUCHI_PREFILL       prompts of this many tokens or more (default 0 =
 *                          never) run as one batched prefill on the tensor
 *                          cores (shk_cuda_prefill: f16 matmul inputs, which
 *                          move the logits by up to ~3e-2 of their std on the
 *                          synthetic test models, above the decode path's
 *                          1e-2; greedy ids stay identical in the tests)
 *                          instead of a decode step per token; single GPU,
 *                          HBM-resident mode, Q4_K / Q6_K weights
 *   SHUKUCHI_DEBUG         set and not "0": per-layer quant types and, for
 *                          the first prompt token, the embedding's and layer
 *                          0's intermediate statistics on stdout, as the
 *                          reference prints them (engine/src/engine.c:23-51)
 */
#ifndef SHK_ENGINE_H
#define SHK_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct engine_handle engine_handle_t;

typedef void (*token_callback)(uint32_t token_id, const char *text, void *user);

struct engine_config { /* engine/include/engine.h:12-19 */
    uint32_t n_threads;
    uint32_t batch_size;
    uint32_t prefetch_depth; /* 2 or 3 */
    uint32_t kv_block_size;
    uint32_t kv_quant; /* 0 = Q8_0 (the only one implemented) */
    int use_mmap;
};

struct streaming_stats { /* engine/include/model_loader.h:82-91 */
    uint64_t layer_loads;
    uint64_t layer_bytes_read;
    size_t max_layer_size;
    size_t peak_buffer_usage;
    size_t peak_rss;
    uint32_t max_concurrent_buffers;
    uint32_t prefetch_hits;
    uint32_t prefetch_misses;
};

engine_handle_t *engine_open(const char *model_path, const struct engine_config *cfg);
int engine_set_prompt(engine_handle_t *h, const char *prompt);
int engine_generate(engine_handle_t *h, uint32_t max_tokens);
int engine_generate_stream(engine_handle_t *h, uint32_t max_tokens, token_callback cb, void *user);
const char *engine_get_output(engine_handle_t *h);
const uint32_t *engine_get_tokens(engine_handle_t *h, size_t *n_tokens);
void engine_cancel(engine_handle_t *h);
void engine_close(engine_handle_t *h);
int engine_get_streaming_stats(engine_handle_t *h, struct streaming_stats *out);

/* Additions (no counterpart in the reference API): token ids in, ids and the
 * logits of every generated token out (n_decode x n_vocab floats, may be
 * NULL), for parity checks against the reference's CPU path. */
int engine_generate_ids(engine_handle_t *h, const uint32_t *prompt, uint32_t n_prompt,
                        uint32_t n_decode, uint32_t *out_ids, float *out_logits);
uint32_t engine_vocab_size(engine_handle_t *h);
/* The GPU backend's counters on stderr (matvec calls, layer forwards, token
 * steps, staged copies and bytes): the CLI's closing report, as the
 * reference's main prints metal_ops_report() (engine/src/main.c:106). */
void engine_report(engine_handle_t *h);
/* The tensor-parallel split of rank `rank` of `world` (no GPU needed):
 * shape = {n_embd, n_heads, n_kv_heads, head_dim, n_ff, n_vocab}; out = {A
 * (ranks sharing attention heads), kv_lo, kv_hi, o_lo, o_hi (O-projection
 * output rows), f_lo, f_hi (FFN columns), v_lo, v_hi (output-head rows)}.
 * 0 on success, -1 when the shape has no block-aligned split. */
int engine_tp_layout(const uint32_t shape[6], uint32_t rank, uint32_t world, uint32_t out[9]);
/* The prompt tokenizer alone (no GPU needed): the ids of `text` under a GGUF
 * file's vocabulary, at most cap of them; returns the count or -1. */
int engine_tokenize_file(const char *model_path, const char *text, uint32_t *out, uint32_t cap);
/* Parses a model file's header only (no GPU needed): layers, width, heads,
 * KV heads, FFN width, vocabulary, largest layer span.  0 on success. */
int engine_inspect(const char *model_path, uint32_t out[6], uint64_t *max_layer_bytes);

#ifdef __cplusplus
}
#endif
#endif
