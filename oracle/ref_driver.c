/*
 * ref_driver.c -- thin C entry points around the UNMODIFIED reference engine,
 * built into oracle/_ref/libshkref.so by oracle/Makefile straight from the
 * reference sources.  Test and baseline infrastructure only: it lets the tests
 * pin the oracle restatement against the reference itself and lets bench.py
 * time the reference CPU path.  Nothing in the product links it.
 *
 * engine.c and kv_cache.c are included (not linked) so that the static
 * forward_layer_view (engine/src/engine.c:76), the engine_handle struct and
 * q8_quantize_vec (engine/src/kv_cache.c:28) are reachable.
 */
#include "engine.c"
#include "kv_cache.c"

#include <time.h>

int ref_matmul(uint32_t dtype, const void *w, const float *x, float *y,
               uint32_t m, uint32_t k) {
    if (dtype == 12) return op_matmul_q4_k(NULL, w, x, y, m, k);
    if (dtype == 13) return op_matmul_q5_k(NULL, w, x, y, m, k);
    if (dtype == 14) return op_matmul_q6_k(NULL, w, x, y, m, k);
    return -1;
}

int ref_rmsnorm(const float *x, const float *w, float *y, uint32_t d) {
    return op_rmsnorm(NULL, x, w, y, 1, d);
}

int ref_rope(float *qk, uint32_t n_heads, uint32_t head_dim, uint32_t pos, float theta) {
    return op_rope(NULL, qk, n_heads, head_dim, pos, theta);
}

int ref_attention(const float *q, const float *k, const float *v, float *out,
                  uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t seq, float scale) {
    return op_attention(NULL, q, k, v, out, n_heads, n_kv, hd, seq, scale, NULL);
}

int ref_softmax(float *x, uint32_t n) { return op_softmax(NULL, x, n); }

int ref_embed(const void *table, uint32_t dtype, uint32_t tok, float *out, uint32_t n_embd) {
    return op_embed(NULL, table, dtype, &tok, out, 1, n_embd);
}

int ref_mlp_swiglu(const float *x, const void *wg, const void *wu, const void *wd,
                   float *y, uint32_t d_in, uint32_t d_ff) {
    return op_mlp_swiglu(NULL, x, wg, wu, wd, y, 1, d_in, d_ff);
}

void ref_q8_quantize(const float *x, uint32_t n, void *out) {
    q8_quantize_vec(x, n, (struct q8_block *)out);
}

/* Reference KV cache, exposed with raw block access for byte comparisons. */
void *ref_kv_create(uint32_t n_layers, uint32_t n_kv, uint32_t hd, uint32_t block, uint32_t max_seq) {
    struct kv_cache_config c = {n_layers, n_kv, hd, block, max_seq, KV_Q8_0};
    return kv_cache_create(&c);
}
void ref_kv_destroy(void *c) { kv_cache_destroy((kv_cache_t *)c); }
int ref_kv_append(void *c, uint32_t layer, uint32_t pos, const float *k, const float *v) {
    return kv_cache_append((kv_cache_t *)c, layer, pos, k, v);
}
int ref_kv_read_range(void *c, uint32_t layer, uint32_t s, uint32_t e, float *k, float *v) {
    return kv_cache_read_range((kv_cache_t *)c, layer, s, e, k, v);
}
const void *ref_kv_token_blocks(void *cv, uint32_t layer, uint32_t pos, int which) {
    kv_cache_t *c = (kv_cache_t *)cv;
    struct kv_block *blk = &c->blocks[layer * c->n_blocks + pos / c->cfg.block_size];
    struct q8_block *base = which ? blk->v : blk->k;
    return base + (pos % c->cfg.block_size) * c->q8_blocks_per_token;
}

/* An engine handle without a GGUF file: dims + a KV cache, for driving
 * forward_layer_view on weights that live in caller memory. */
void *ref_engine_new(uint32_t n_layers, uint32_t n_embd, uint32_t n_heads,
                     uint32_t n_kv, uint32_t max_seq) {
    struct engine_handle *h = calloc(1, sizeof(*h));
    if (!h) return NULL;
    h->info.n_layers = n_layers;
    h->info.n_embd = n_embd;
    h->info.n_heads = n_heads;
    h->info.n_kv_heads = n_kv;
    h->info.head_dim = n_embd / n_heads;
    h->info.rope_theta = 0.0f; /* as model_get_info leaves it */
    struct kv_cache_config c = {n_layers, n_kv, h->info.head_dim, 32, max_seq, KV_Q8_0};
    h->kv = kv_cache_create(&c);
    if (!h->kv) { free(h); return NULL; }
    return h;
}
void ref_engine_free(void *hv) {
    struct engine_handle *h = hv;
    if (!h) return;
    kv_cache_destroy(h->kv);
    free(h);
}
void *ref_engine_kv(void *hv) { return ((struct engine_handle *)hv)->kv; }

/* ptrs/types/sizes in layer_view order: attn_norm, q, k, v, o, ffn_norm,
 * gate, up, down */
int ref_forward_layer(void *hv, const void *const *ptrs, const uint32_t *types,
                      const uint64_t *sizes, uint32_t layer, uint32_t pos, float *hidden) {
    struct layer_view lv;
    memset(&lv, 0, sizeof(lv));
    lv.layer_id = layer;
    lv.attn_norm = ptrs[0]; lv.attn_q = ptrs[1]; lv.attn_k = ptrs[2];
    lv.attn_v = ptrs[3]; lv.attn_o = ptrs[4]; lv.ffn_norm = ptrs[5];
    lv.ffn_gate = ptrs[6]; lv.ffn_up = ptrs[7]; lv.ffn_down = ptrs[8];
    lv.attn_norm_dtype = types[0]; lv.attn_q_dtype = types[1]; lv.attn_k_dtype = types[2];
    lv.attn_v_dtype = types[3]; lv.attn_o_dtype = types[4]; lv.ffn_norm_dtype = types[5];
    lv.ffn_gate_dtype = types[6]; lv.ffn_up_dtype = types[7]; lv.ffn_down_dtype = types[8];
    lv.attn_q_size = sizes[1]; lv.attn_k_size = sizes[2]; lv.attn_v_size = sizes[3];
    lv.attn_o_size = sizes[4]; lv.ffn_gate_size = sizes[6]; lv.ffn_up_size = sizes[7];
    lv.ffn_down_size = sizes[8];
    return forward_layer_view((struct engine_handle *)hv, &lv, layer, pos, hidden);
}

/* Opens a GGUF through the reference loader + prefetcher and runs token ids
 * (bypassing the text tokenizer) through the same loop as engine_generate
 * (engine/src/engine.c:343-495), capturing logits.  stats_out (nullable)
 * receives the streaming_stats fields as 8 uint64. */
static int ref_run_layers(engine_handle_t *h, uint32_t pos, float *hidden) {
    uint32_t n_layers = h->info.n_layers;
    prefetch_request_t *req0 = prefetcher_request(h->prefetch, 0);
    prefetch_request_t *req1 = (n_layers > 1) ? prefetcher_request(h->prefetch, 1) : NULL;
    if (!req0) return -1;
    for (uint32_t l = 0; l < n_layers; ++l) {
        prefetch_request_t *next_req = NULL;
        if (l + 2 < n_layers) next_req = prefetcher_request(h->prefetch, l + 2);
        struct layer_buffer *buf = prefetcher_wait(req0);
        if (!buf) return -1;
        int rc = forward_layer_view(h, &buf->view, l, pos, hidden);
        prefetcher_release(h->prefetch, buf);
        if (rc != 0) return -1;
        req0 = req1;
        req1 = next_req;
        if (l + 1 < n_layers && !req0) return -1;
    }
    return 0;
}

int ref_generate_file(const char *path, uint32_t depth, const uint32_t *prompt,
                      uint32_t n_prompt, uint32_t n_decode, uint32_t *out_ids,
                      float *out_logits, uint64_t *stats_out) {
    struct engine_config cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.prefetch_depth = depth;
    cfg.kv_block_size = 32;
    engine_handle_t *h = engine_open(path, &cfg);
    if (!h) return -1;
    int rc = -1;
    struct resident_tensors res;
    uint32_t n_vocab = 0;
    float *hidden = NULL, *logits = NULL;
    if (model_get_resident(h->model, &res) || model_get_vocab_size(h->model, &n_vocab) || !h->prefetch)
        goto out;
    uint32_t D = h->info.n_embd, pos = 0;
    hidden = calloc(D, 4);
    logits = malloc((size_t)n_vocab * 4);
    if (!hidden || !logits) goto out;
    for (uint32_t i = 0; i < n_prompt; ++i, ++pos) {
        uint32_t tok = prompt[i];
        if (op_embed(NULL, res.token_embd, res.token_embd_dtype, &tok, hidden, 1, D)) goto out;
        if (ref_run_layers(h, pos, hidden)) goto out;
    }
    for (uint32_t t = 0; t < n_decode; ++t, ++pos) {
        if (matmul_quant(res.lm_head_dtype, res.lm_head, hidden, logits, n_vocab, D)) goto out;
        uint32_t next = 0;
        float mx = logits[0];
        for (uint32_t i = 1; i < n_vocab; ++i)
            if (logits[i] > mx) { mx = logits[i]; next = i; }
        if (out_ids) out_ids[t] = next;
        if (out_logits) memcpy(out_logits + (size_t)t * n_vocab, logits, (size_t)n_vocab * 4);
        if (op_embed(NULL, res.token_embd, res.token_embd_dtype, &next, hidden, 1, D)) goto out;
        if (ref_run_layers(h, pos, hidden)) goto out;
    }
    if (stats_out) {
        struct streaming_stats st;
        if (engine_get_streaming_stats(h, &st) == 0) {
            stats_out[0] = st.layer_loads; stats_out[1] = st.layer_bytes_read;
            stats_out[2] = st.max_layer_size; stats_out[3] = st.peak_buffer_usage;
            stats_out[4] = st.peak_rss; stats_out[5] = st.max_concurrent_buffers;
            stats_out[6] = st.prefetch_hits; stats_out[7] = st.prefetch_misses;
        }
    }
    rc = 0;
out:
    free(hidden);
    free(logits);
    engine_close(h);
    return rc;
}

double ref_now(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

/* model_tokenize (engine/src/model_loader.c:441-518) on a GGUF file's
 * vocabulary: the ids (BOS first when the file names one), at most cap of
 * them; returns the count or -1. */
int ref_tokenize(const char *path, const char *text, uint32_t *out, uint32_t cap) {
    struct model_config mcfg;
    memset(&mcfg, 0, sizeof(mcfg));
    mcfg.prefer_gguf = 1;
    model_handle_t *m = model_open(path, &mcfg);
    if (!m) return -1;
    uint32_t *ids = NULL, n = 0;
    int rc = model_tokenize(m, text, &ids, &n);
    if (!rc) {
        for (uint32_t i = 0; i < n && i < cap; ++i) out[i] = ids[i];
        rc = (int)n;
    }
    free(ids);
    model_close(m);
    return rc;
}
