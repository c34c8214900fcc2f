/* engine.c -- GGUF llama model, layer-streaming loader and token loop over
 * libshk_cuda (see engine.h).
 *
 * Reference behaviour kept (engine/src/engine.c:306-501): the prompt is fed
 * token by token; each generated token is the first-index argmax of the
 * logits of the previous position (no final norm, rope theta 10000), is
 * printed as "<id>text", and is itself run through all layers.  An empty
 * prompt decodes from token 1.  Prompt text is tokenised by greedy longest
 * match over the vocabulary after mapping whitespace to U+2581, with the BOS
 * id first when the file names one (engine/src/model_loader.c:441-513).
 */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "engine.h"

#include <errno.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/resource.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../include/shk_cuda.h"
#include "gguf.h"
#include "lstr.h"

enum { TN_ATTN_NORM, TN_Q, TN_K, TN_V, TN_O, TN_FFN_NORM, TN_GATE, TN_UP, TN_DOWN, TN_COUNT };
static const char *const k_suffix[TN_COUNT] = {
    "attn_norm.weight", "attn_q.weight",   "attn_k.weight", "attn_v.weight",   "attn_output.weight",
    "ffn_norm.weight",  "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};

struct tensor_loc {
    uint64_t off, size;  /* file offset (absolute), bytes */
    uint32_t type;
    uint64_t rows, row_bytes;
    uint64_t dev_off;    /* offset in the layer's device buffer (256-aligned) */
    uint64_t dev_row;    /* padded device row bytes, 0 = dense copy */
};

struct layer_map {
    struct tensor_loc t[TN_COUNT];
    uint64_t span_off, span_len; /* contiguous file range holding the nine tensors */
    uint64_t dev_bytes;
};

struct tp_layout { /* one rank's slices (tensor parallelism, see below) */
    uint32_t A, kv_lo, kv_hi, o_lo, o_hi, f_lo, f_hi, v_lo, v_hi;
};

struct tp_rank {
    uint32_t rank;
    struct tp_layout lay;
    shk_ctx *ctx;
    shk_kv *kv;
    shk_model *m;
    void *d_embd, *d_out;
    void **d_buf;              /* one per layer (resident) */
    struct shk_layer_desc *ld; /* per layer */
    /* a generation's inputs and results (rank threads) */
    const uint32_t *prompt;
    uint32_t n_prompt, n_decode;
    int want_logits; /* rank 0 copies logits: every rank gathers on the same steps */
    float *lg;       /* n_vocab floats of scratch for those copies */
    int rc;
};

struct engine_handle {
    struct gguf_file g;
    struct engine_config cfg;
    uint32_t n_layers, n_embd, n_heads, n_kv, head_dim, n_ff, n_vocab;
    char **vocab;
    uint32_t *vocab_slot; /* open-addressing index: string -> lowest id (tokenizer) */
    uint32_t vocab_cap, vocab_maxlen;
    int has_bos;
    uint32_t bos;
    struct layer_map *lm;
    uint64_t max_span, max_dev;
    uint32_t depth;
    int resident;
    uint32_t max_seq;

    shk_ctx *ctx;
    shk_kv *kv;
    shk_model *m;
    void *d_embd, *d_out;
    void **d_buf;   /* resident: one per layer; ring: one per slot */
    uint32_t n_buf;
    void **pinned;  /* depth staging buffers of max_span bytes */

    pthread_t thr;
    int thr_started;
    pthread_mutex_t mu;
    pthread_cond_t cv;
    uint64_t n_req;        /* requests to stage: resident n_layers; ring: per generation */
    uint64_t req_staged;   /* requests whose copies are queued */
    uint64_t req_consumed; /* requests the engine has finished enqueuing work for */
    int stop, loader_err;
    struct streaming_stats st;
    int registered;

    /* tensor parallelism (SHUKUCHI_TP = world > 1): one GPU and context per
     * rank; ranks[0] is also ctx/kv/m above */
    uint32_t tp;
    struct tp_rank *ranks;
    int tp_broken;

    char *prompt;
    uint32_t *out_ids;
    size_t n_out, cap_out;
    char *text;
    size_t text_len, text_cap;
    volatile int cancel;
    uint32_t pos;      /* next KV position */
    uint64_t ring_next; /* ring mode: next loader request to consume */
};

static void *tp_rank_main(void *arg);

/* A model file: GGUF, or the LSTR container (engine/lstr.h) by its magic. */
static int model_file_open(const char *path, struct gguf_file *g) {
    return lstr_is(path) ? lstr_open(path, g) : gguf_open(path, g);
}

static int env_int(const char *name, int def) {
    const char *v = getenv(name);
    if (!v || !*v) return def;
    return (int)strtol(v, NULL, 10);
}

static uint64_t al256(uint64_t x) { return (x + 255) & ~(uint64_t)255; }

/* ------------------------------- debug ---------------------------------- */
/* SHUKUCHI_DEBUG (set and not "0"), engine/src/engine.c:23-51: the quant
 * types of every layer a token runs through, and for the first prompt token
 * the embedding and layer 0's intermediates (min / max / mean / NaN / inf),
 * computed through the op-level calls in the reference's op order. */

static int debug_enabled(void) {
    const char *e = getenv("SHUKUCHI_DEBUG");
    return e && e[0] && strcmp(e, "0") != 0;
}

static void debug_stats(const char *name, const float *x, uint32_t n) {
    if (!x || !n) {
        printf("[DEBUG] %s: empty\n", name);
        return;
    }
    float lo = x[0], hi = x[0], sum = 0.0f;
    int nan = 0, inf = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const float v = x[i];
        nan |= isnan(v) ? 1 : 0;
        inf |= isinf(v) ? 1 : 0;
        if (v < lo) lo = v;
        if (v > hi) hi = v;
        sum += v;
    }
    printf("[DEBUG] %s: min=%.4f max=%.4f mean=%.4f nan=%d inf=%d\n", name, lo, hi, sum / (float)n, nan, inf);
}

static int debug_dev(shk_ctx *c, const char *name, const float *dev, uint32_t n, float *host) {
    if (shk_cuda_memcpy_d2h(c, host, dev, (size_t)n * 4, NULL) != SHK_OK || shk_cuda_sync(c, NULL) != SHK_OK)
        return -1;
    debug_stats(name, host, n);
    return 0;
}

/* the file's ggml types, as the reference prints its layer view's (not the
 * device layouts they were converted to) */
static void debug_dtypes(const struct engine_handle *h, uint32_t l) {
    const struct tensor_loc *t = h->lm[l].t;
    printf("[DEBUG] dtypes: q=%u k=%u v=%u o=%u gate=%u up=%u down=%u\n", t[TN_Q].type, t[TN_K].type,
           t[TN_V].type, t[TN_O].type, t[TN_GATE].type, t[TN_UP].type, t[TN_DOWN].type);
}

/* ------------------------------ model map ------------------------------- */

/* The tokenizer's vocabulary and BOS id (engine/src/model_loader.c:107-111). */
static void map_vocab(struct engine_handle *h) {
    struct gguf_file *g = &h->g;
    const struct gguf_value *tok = gguf_get(g, "tokenizer.ggml.tokens");
    if (tok && tok->type == GGUF_ARRAY && tok->arr_type == GGUF_STRING && tok->arr_n) {
        h->vocab = tok->arr_str;
        h->n_vocab = (uint32_t)tok->arr_n;
    }
    const struct gguf_value *bos = gguf_get(g, "tokenizer.ggml.bos_token_id");
    if (bos && bos->type == GGUF_U32) {
        h->has_bos = 1;
        h->bos = (uint32_t)bos->u;
    }
}

static int map_model(struct engine_handle *h) {
    struct gguf_file *g = &h->g;
    h->n_layers = (uint32_t)gguf_get_uint(g, "llama.block_count", 0);
    h->n_embd = (uint32_t)gguf_get_uint(g, "llama.embedding_length", 0);
    h->n_heads = (uint32_t)gguf_get_uint(g, "llama.attention.head_count", 0);
    h->n_kv = (uint32_t)gguf_get_uint(g, "llama.attention.head_count_kv", h->n_heads);
    if (!h->n_layers || !h->n_embd || !h->n_heads || !h->n_kv || h->n_embd % h->n_heads) return -1;
    h->head_dim = h->n_embd / h->n_heads;
    map_vocab(h);
    const struct gguf_tensor_info *out = gguf_find_tensor(g, "output.weight");
    const struct gguf_tensor_info *emb = gguf_find_tensor(g, "token_embd.weight");
    if (!out || !emb || out->n_dims != 2 || emb->n_dims != 2) return -1;
    if (!h->n_vocab) h->n_vocab = (uint32_t)out->dims[1];
    if (out->dims[1] != h->n_vocab || out->dims[0] != h->n_embd) return -1;
    /* every tensor must lie inside the file: a truncated file is rejected
     * here instead of by a short read in the middle of a generation */
    struct stat sb;
    if (fstat(g->fd, &sb) != 0) return -1;
    for (uint64_t i = 0; i < g->n_tensors; ++i)
        if (g->tensors[i].offset + g->tensors[i].size > (uint64_t)sb.st_size) return -1;
    h->lm = (struct layer_map *)calloc(h->n_layers, sizeof(struct layer_map));
    if (!h->lm) return -1;
    char name[96];
    for (uint32_t l = 0; l < h->n_layers; ++l) {
        struct layer_map *L = &h->lm[l];
        uint64_t lo = UINT64_MAX, hi = 0, dev = 0;
        for (int t = 0; t < TN_COUNT; ++t) {
            snprintf(name, sizeof(name), "blk.%u.%s", l, k_suffix[t]);
            const struct gguf_tensor_info *ti = gguf_find_tensor(g, name);
            if (!ti || !ti->size) return -1;
            struct tensor_loc *tl = &L->t[t];
            tl->off = ti->offset;
            tl->size = ti->size;
            tl->type = ti->type;
            tl->rows = ti->n_dims == 2 ? ti->dims[1] : 1;
            tl->row_bytes = ti->size / tl->rows;
            const int norm = t == TN_ATTN_NORM || t == TN_FFN_NORM;
            if (norm && ti->type != 0) return -1; /* F32 norm weights */
            if (!norm && ti->type != 12 && ti->type != 13 && ti->type != 14) return -1; /* Q4_K / Q5_K / Q6_K */
            tl->dev_row = 0;
            if (!norm && tl->row_bytes % 16) {
                /* Q6_K rows of a width that is not a multiple of 2048: pad to
                 * 16 bytes so every row starts where a bulk copy can read it;
                 * only attn_v and ffn_down carry a row stride */
                if (t != TN_V && t != TN_DOWN) return -1;
                tl->dev_row = (tl->row_bytes + 15) & ~(uint64_t)15;
            }
            tl->dev_off = dev;
            dev = al256(dev + (tl->dev_row ? tl->dev_row * tl->rows : tl->size));
            if (tl->off < lo) lo = tl->off;
            if (tl->off + tl->size > hi) hi = tl->off + tl->size;
        }
        L->span_off = lo;
        L->span_len = hi - lo;
        L->dev_bytes = dev;
        if (L->span_len > h->max_span) h->max_span = L->span_len;
        if (L->dev_bytes > h->max_dev) h->max_dev = L->dev_bytes;
        if (l == 0) h->n_ff = (uint32_t)L->t[TN_GATE].rows;
    }
    return 0;
}

static int pread_all(int fd, void *dst, uint64_t len, uint64_t off) {
    uint8_t *d = (uint8_t *)dst;
    while (len) {
        ssize_t n = pread(fd, d, len > (1u << 30) ? (1u << 30) : len, (off_t)off);
        if (n < 0 && errno == EINTR) continue;
        if (n <= 0) return -1;
        d += n;
        off += (uint64_t)n;
        len -= (uint64_t)n;
    }
    return 0;
}

/* A span read by several threads at once (SHUKUCHI_IO_THREADS, default 4):
 * one thread's pread from the page cache into pinned memory copies at
 * ~7 GB/s, below what the H2D link takes. */
struct pread_job {
    int fd, rc;
    uint8_t *dst;
    uint64_t len, off;
};
static void *pread_main(void *arg) {
    struct pread_job *j = (struct pread_job *)arg;
    j->rc = pread_all(j->fd, j->dst, j->len, j->off);
    return NULL;
}
static int pread_span(int fd, void *dst, uint64_t len, uint64_t off) {
    int nt = env_int("SHUKUCHI_IO_THREADS", 4);
    if (nt > 16) nt = 16;
    if (nt <= 1 || len < (16u << 20)) return pread_all(fd, dst, len, off);
    struct pread_job jobs[16];
    pthread_t th[16];
    int started[16];
    const uint64_t piece = ((len + (uint64_t)nt - 1) / (uint64_t)nt + 4095) & ~(uint64_t)4095;
    int n = 0, rc = 0;
    for (uint64_t o = 0; o < len && n < nt; o += piece, ++n) {
        jobs[n] = (struct pread_job){fd, 0, (uint8_t *)dst + o, (len - o < piece ? len - o : piece), off + o};
        started[n] = pthread_create(&th[n], NULL, pread_main, &jobs[n]) == 0;
        if (!started[n]) jobs[n].rc = pread_all(fd, jobs[n].dst, jobs[n].len, jobs[n].off); /* here instead */
    }
    for (int i = 0; i < n; ++i) {
        if (started[i]) pthread_join(th[i], NULL);
        rc |= jobs[i].rc;
    }
    return rc ? -1 : 0;
}

static int upload_tensor(struct engine_handle *h, const struct gguf_tensor_info *ti, void **dev) {
    void *host = NULL;
    if (shk_cuda_host_alloc(h->ctx, ti->size, &host) != SHK_OK) return -1;
    int rc = pread_all(h->g.fd, host, ti->size, ti->offset);
    if (!rc) rc = shk_cuda_dev_alloc(h->ctx, ti->size, dev) == SHK_OK ? 0 : -1;
    if (!rc) rc = shk_cuda_memcpy_h2d(h->ctx, *dev, host, ti->size, NULL) == SHK_OK ? 0 : -1;
    if (!rc) rc = shk_cuda_sync(h->ctx, NULL) == SHK_OK ? 0 : -1; /* before the staging is freed */
    shk_cuda_host_free(h->ctx, host);
    return rc;
}

static void layer_desc(struct engine_handle *h, uint32_t l, const uint8_t *base, struct shk_layer_desc *d) {
    const struct layer_map *L = &h->lm[l];
    memset(d, 0, sizeof(*d));
    d->attn_norm = (const float *)(base + L->t[TN_ATTN_NORM].dev_off);
    d->ffn_norm = (const float *)(base + L->t[TN_FFN_NORM].dev_off);
    d->attn_q = base + L->t[TN_Q].dev_off;
    d->attn_k = base + L->t[TN_K].dev_off;
    d->attn_v = base + L->t[TN_V].dev_off;
    d->attn_o = base + L->t[TN_O].dev_off;
    d->ffn_gate = base + L->t[TN_GATE].dev_off;
    d->ffn_up = base + L->t[TN_UP].dev_off;
    d->ffn_down = base + L->t[TN_DOWN].dev_off;
    /* Q6_K tensors were converted to the planar layout while staging */
#define DT(i) (L->t[i].type == 14 ? SHK_DTYPE_Q6_K_PLANAR : L->t[i].type)
    d->attn_q_dtype = DT(TN_Q);
    d->attn_k_dtype = DT(TN_K);
    d->attn_v_dtype = DT(TN_V);
    d->attn_o_dtype = DT(TN_O);
    d->ffn_gate_dtype = DT(TN_GATE);
    d->ffn_up_dtype = DT(TN_UP);
    d->ffn_down_dtype = DT(TN_DOWN);
#undef DT
    d->row_stride_v = (uint32_t)L->t[TN_V].dev_row;
    d->row_stride_down = (uint32_t)L->t[TN_DOWN].dev_row;
}

/* Layer 0 at position 0 for SHUKUCHI_DEBUG: engine/src/engine.c:105-221's
 * op order (RMSNorm, Q/K/V matvecs, RoPE, Q8_0 append and read-back,
 * attention, O, residual, RMSNorm, gate/up, SwiGLU, down, residual) on
 * scratch buffers and a one-position scratch KV cache, so the real pass that
 * follows is untouched.  `hidden` is the embedded token (device). */
static int debug_layer0(struct engine_handle *h, const struct shk_layer_desc *d, const float *hidden) {
    shk_ctx *c = h->ctx;
    const uint32_t D = h->n_embd, hd = h->head_dim, qd = h->n_heads * hd, kvd = h->n_kv * hd, F = h->n_ff;
    const uint32_t big = (D > F ? D : F) > qd ? (D > F ? D : F) : qd;
    float *host = (float *)malloc((size_t)big * 4), *hres = (float *)malloc((size_t)D * 4);
    float *buf[12] = {0};
    enum { NRM, Q, K, V, KC, VC, ATT, PRJ, HID, G, U, HM };
    const uint32_t sz[12] = {D, qd, kvd, kvd, kvd, kvd, qd, D, D, F, F, F};
    struct shk_kv_config kc = {1, h->n_kv, hd, 32, 8};
    shk_kv *kv = shk_cuda_kv_create(c, &kc);
    int rc = (!host || !hres || !kv) ? -1 : 0;
    for (int i = 0; !rc && i < 12; ++i) rc = shk_cuda_dev_alloc(c, (size_t)sz[i] * 4, (void **)&buf[i]) != SHK_OK;
#define OK(x) (!rc && (rc = ((x) != SHK_OK)) == 0)
#define DUMP(name, i, n) (!rc && (rc = debug_dev(c, name, buf[i], n, host)) == 0)
    OK(shk_cuda_rmsnorm(c, hidden, d->attn_norm, buf[NRM], D, NULL));
    DUMP("attn_norm", NRM, D);
    OK(shk_cuda_matvec(c, d->attn_q_dtype, d->attn_q, 0, buf[NRM], buf[Q], qd, D, NULL));
    DUMP("Q", Q, qd);
    OK(shk_cuda_matvec(c, d->attn_k_dtype, d->attn_k, 0, buf[NRM], buf[K], kvd, D, NULL));
    DUMP("K", K, kvd);
    OK(shk_cuda_matvec(c, d->attn_v_dtype, d->attn_v, d->row_stride_v, buf[NRM], buf[V], kvd, D, NULL));
    DUMP("V", V, kvd);
    OK(shk_cuda_rope(c, buf[Q], h->n_heads, hd, 0, 10000.0f, NULL));
    OK(shk_cuda_rope(c, buf[K], h->n_kv, hd, 0, 10000.0f, NULL));
    DUMP("Q_rope", Q, qd);
    DUMP("K_rope", K, kvd);
    OK(shk_cuda_kv_append(kv, 0, 0, buf[K], buf[V], NULL));
    OK(shk_cuda_kv_read_range(kv, 0, 0, 1, buf[KC], buf[VC], NULL));
    DUMP("K_cache", KC, kvd);
    DUMP("V_cache", VC, kvd);
    OK(shk_cuda_kv_attend(kv, 0, buf[Q], NULL, NULL, buf[ATT], h->n_heads, 1, 1.0f / sqrtf((float)hd), NULL));
    DUMP("attn_out", ATT, qd);
    OK(shk_cuda_matvec(c, d->attn_o_dtype, d->attn_o, 0, buf[ATT], buf[PRJ], D, qd, NULL));
    DUMP("attn_proj", PRJ, D);
    /* residual on the host: hidden + attn_proj */
    OK(shk_cuda_memcpy_d2h(c, hres, hidden, (size_t)D * 4, NULL));
    OK(shk_cuda_sync(c, NULL));
    for (uint32_t i = 0; !rc && i < D; ++i) hres[i] += host[i];
    if (!rc) debug_stats("hidden_after_attn", hres, D);
    OK(shk_cuda_memcpy_h2d(c, buf[HID], hres, (size_t)D * 4, NULL));
    OK(shk_cuda_rmsnorm(c, buf[HID], d->ffn_norm, buf[NRM], D, NULL));
    DUMP("ffn_norm", NRM, D);
    OK(shk_cuda_matvec(c, d->ffn_gate_dtype, d->ffn_gate, 0, buf[NRM], buf[G], F, D, NULL));
    OK(shk_cuda_matvec(c, d->ffn_up_dtype, d->ffn_up, 0, buf[NRM], buf[U], F, D, NULL));
    OK(shk_cuda_swiglu(c, buf[G], buf[U], buf[HM], F, NULL));
    OK(shk_cuda_matvec(c, d->ffn_down_dtype, d->ffn_down, d->row_stride_down, buf[HM], buf[PRJ], D, F, NULL));
    DUMP("mlp_out", PRJ, D);
    for (uint32_t i = 0; !rc && i < D; ++i) hres[i] += host[i];
    if (!rc) debug_stats("hidden_after_mlp", hres, D);
    OK(shk_cuda_check(c));
#undef OK
#undef DUMP
    for (int i = 0; i < 12; ++i)
        if (buf[i]) shk_cuda_dev_free(c, buf[i]);
    if (kv) shk_cuda_kv_destroy(kv);
    free(host);
    free(hres);
    return rc ? -1 : 0;
}

/* ------------------------------- loader --------------------------------- */
/* Request k stages layer k % n_layers through pinned buffer / event slot
 * k % depth.  Resident mode: requests 0..n_layers-1 into each layer's own
 * device buffer, once.  Ring mode: an endless sequence into device slot
 * k % depth, at most `depth` requests ahead of the engine (the slot's previous
 * layer must have been consumed; the copies also wait on the device for the
 * kernels that read it, via shk_cuda_layer_release). */

static void *loader_main(void *arg) {
    struct engine_handle *h = (struct engine_handle *)arg;
    for (uint64_t k = 0;; ++k) {
        pthread_mutex_lock(&h->mu);
        while (!h->stop && (k >= h->n_req || (!h->resident && k >= h->req_consumed + h->depth)))
            pthread_cond_wait(&h->cv, &h->mu);
        const int stop = h->stop;
        pthread_mutex_unlock(&h->mu);
        if (stop) break;
        const uint32_t l = (uint32_t)(k % h->n_layers), s = (uint32_t)(k % h->depth);
        const struct layer_map *L = &h->lm[l];
        int rc = shk_cuda_layer_ready(h->ctx, s, 1) < 0; /* the staging buffer's last copies landed */
        uint8_t *pin = (uint8_t *)h->pinned[s];
        if (!rc) rc = pread_span(h->g.fd, pin, L->span_len, L->span_off);
        uint8_t *dst = (uint8_t *)h->d_buf[h->resident ? l : s];
        for (int t = 0; !rc && t < TN_COUNT; ++t) {
            const struct tensor_loc *tl = &L->t[t];
            const uint8_t *src = pin + (tl->off - L->span_off);
            if (tl->dev_row)
                rc = shk_cuda_layer_stage_rows(h->ctx, s, dst + tl->dev_off, tl->dev_row, src, tl->row_bytes,
                                               tl->rows) != SHK_OK;
            else
                rc = shk_cuda_layer_stage(h->ctx, s, dst + tl->dev_off, src, tl->size) != SHK_OK;
            if (!rc && tl->type == 14) /* Q6_K: the GEMV reads the planar layout */
                rc = shk_cuda_layer_stage_q6k_planar(h->ctx, s, dst + tl->dev_off, (uint32_t)tl->rows,
                                                     (uint32_t)(tl->row_bytes / 210 * 256),
                                                     (uint32_t)(tl->dev_row ? tl->dev_row : tl->row_bytes)) != SHK_OK;
        }
        if (!rc) rc = shk_cuda_layer_commit(h->ctx, s) != SHK_OK;
        pthread_mutex_lock(&h->mu);
        if (rc) {
            h->loader_err = 1;
        } else {
            h->req_staged = k + 1;
            h->st.layer_loads++;
            h->st.layer_bytes_read += L->span_len;
        }
        pthread_cond_broadcast(&h->cv);
        pthread_mutex_unlock(&h->mu);
        if (rc) break;
    }
    return NULL;
}

/* Engine side: wait until request k is queued, count a prefetch hit when its
 * copies have already landed, and make the compute stream wait for them. */
static int acquire(struct engine_handle *h, uint64_t k) {
    pthread_mutex_lock(&h->mu);
    while (h->req_staged <= k && !h->loader_err) pthread_cond_wait(&h->cv, &h->mu);
    const int err = h->loader_err && h->req_staged <= k;
    pthread_mutex_unlock(&h->mu);
    if (err) return -1;
    const uint32_t s = (uint32_t)(k % h->depth);
    const int ready = shk_cuda_layer_ready(h->ctx, s, 0);
    if (ready < 0) return -1;
    if (ready) h->st.prefetch_hits++;
    else h->st.prefetch_misses++;
    return shk_cuda_layer_wait(h->ctx, s, NULL) == SHK_OK ? 0 : -1;
}

static void consume(struct engine_handle *h, uint64_t k) {
    if (!h->resident) shk_cuda_layer_release(h->ctx, (uint32_t)(k % h->depth), NULL);
    pthread_mutex_lock(&h->mu);
    if (k + 1 > h->req_consumed) h->req_consumed = k + 1;
    pthread_cond_broadcast(&h->cv);
    pthread_mutex_unlock(&h->mu);
}

/* Resident mode: all layers staged and registered for the captured step. */
static int register_layers(struct engine_handle *h) {
    if (h->registered) {
        h->st.prefetch_hits += h->n_layers; /* resident: every layer is already in HBM */
        return 0;
    }
    for (uint32_t l = 0; l < h->n_layers; ++l) {
        if (acquire(h, l)) return -1;
        struct shk_layer_desc d;
        layer_desc(h, l, (const uint8_t *)h->d_buf[l], &d);
        if (shk_cuda_model_set_layer(h->m, l, &d) != SHK_OK) return -1;
        consume(h, l);
    }
    if (shk_cuda_sync(h->ctx, NULL) != SHK_OK) return -1;
    h->registered = 1;
    return 0;
}

/* ------------------------------ tokenizer ------------------------------- */
/* Greedy longest match (engine/src/model_loader.c:483-513 scans the whole
 * vocabulary for every position: O(V * len)).  Here the vocabulary is hashed
 * once; at each position the candidate lengths are tried from the longest
 * vocabulary string down, so the first hit is the longest match, and among
 * equal strings the index keeps the lowest id -- the reference's choice
 * (strictly longer matches replace, ties keep the first). */

static uint64_t str_hash(const char *p, size_t n) {
    uint64_t x = 1469598103934665603ull; /* FNV-1a */
    for (size_t i = 0; i < n; ++i) x = (x ^ (uint8_t)p[i]) * 1099511628211ull;
    return x;
}

static int vocab_index_build(struct engine_handle *h) {
    if (!h->vocab || !h->n_vocab) return 0;
    uint32_t cap = 1;
    while (cap < 2u * h->n_vocab) cap <<= 1;
    h->vocab_slot = (uint32_t *)malloc((size_t)cap * sizeof(uint32_t));
    if (!h->vocab_slot) return -1;
    memset(h->vocab_slot, 0xFF, (size_t)cap * sizeof(uint32_t));
    h->vocab_cap = cap;
    for (uint32_t t = 0; t < h->n_vocab; ++t) {
        const char *v = h->vocab[t];
        const size_t n = strlen(v);
        if (!n) continue;
        if (n > h->vocab_maxlen) h->vocab_maxlen = (uint32_t)n;
        for (uint32_t i = (uint32_t)str_hash(v, n) & (cap - 1);; i = (i + 1) & (cap - 1)) {
            const uint32_t id = h->vocab_slot[i];
            if (id == UINT32_MAX) {
                h->vocab_slot[i] = t;
                break;
            }
            if (strlen(h->vocab[id]) == n && memcmp(h->vocab[id], v, n) == 0) break; /* keep the first */
        }
    }
    return 0;
}

static uint32_t vocab_find(const struct engine_handle *h, const char *p, size_t n) {
    for (uint32_t i = (uint32_t)str_hash(p, n) & (h->vocab_cap - 1);; i = (i + 1) & (h->vocab_cap - 1)) {
        const uint32_t id = h->vocab_slot[i];
        if (id == UINT32_MAX) return UINT32_MAX;
        const char *v = h->vocab[id];
        if (strncmp(v, p, n) == 0 && v[n] == '\0') return id;
    }
}

static int tokenize(struct engine_handle *h, const char *text, uint32_t **out, uint32_t *n_out) {
    *out = NULL;
    *n_out = 0;
    const size_t len = text ? strlen(text) : 0;
    char *norm = (char *)malloc(3 * len + 1);
    /* one id per normalised byte at most (unknown bytes), plus BOS */
    uint32_t *ids = (uint32_t *)malloc((3 * len + 2) * sizeof(uint32_t));
    if (!norm || !ids) {
        free(norm);
        free(ids);
        return -1;
    }
    size_t nl = 0;
    for (size_t i = 0; i < len; ++i) {
        const char c = text[i];
        if (c == ' ' || c == '\n' || c == '\t' || c == '\r') { /* U+2581 */
            norm[nl++] = (char)0xE2;
            norm[nl++] = (char)0x96;
            norm[nl++] = (char)0x81;
        } else {
            norm[nl++] = c;
        }
    }
    uint32_t n = 0;
    if (h->has_bos) ids[n++] = h->bos;
    for (size_t i = 0; i < nl;) {
        size_t best = 0;
        uint32_t best_id = 0;
        if (h->vocab_slot) {
            size_t len = nl - i < h->vocab_maxlen ? nl - i : h->vocab_maxlen;
            for (; len > 0; --len) {
                const uint32_t id = vocab_find(h, norm + i, len);
                if (id != UINT32_MAX) {
                    best = len;
                    best_id = id;
                    break;
                }
            }
        }
        if (!best) best = 1; /* unknown byte: token 0 */
        ids[n++] = best_id;
        i += best;
    }
    free(norm);
    *out = ids;
    *n_out = n;
    return 0;
}

static int emit(struct engine_handle *h, uint32_t id, token_callback cb, void *user, int print) {
    if (h->n_out == h->cap_out) {
        const size_t cap = h->cap_out ? 2 * h->cap_out : 64;
        uint32_t *p = (uint32_t *)realloc(h->out_ids, cap * sizeof(uint32_t));
        if (!p) return -1;
        h->out_ids = p;
        h->cap_out = cap;
    }
    h->out_ids[h->n_out++] = id;
    const char *s = (h->vocab && id < h->n_vocab) ? h->vocab[id] : "";
    char piece[64];
    snprintf(piece, sizeof(piece), "<%u>", id);
    const size_t need = h->text_len + strlen(piece) + strlen(s) + 1;
    if (need > h->text_cap) {
        const size_t cap = need * 2;
        char *t = (char *)realloc(h->text, cap);
        if (!t) return -1;
        h->text = t;
        h->text_cap = cap;
    }
    h->text_len += (size_t)sprintf(h->text + h->text_len, "%s%s", piece, s);
    if (cb) cb(id, s, user);
    if (print) {
        printf("%s%s", piece, s);
        fflush(stdout);
    }
    return 0;
}

static void note_rss(struct engine_handle *h) {
    struct rusage ru;
    if (getrusage(RUSAGE_SELF, &ru) == 0 && (size_t)ru.ru_maxrss * 1024u > h->st.peak_rss)
        h->st.peak_rss = (size_t)ru.ru_maxrss * 1024u;
}

/* One token through all layers at h->pos; with want_next the lm_head argmax
 * is returned in *next (and the logits copied to `logits` when given). */
static int step(struct engine_handle *h, uint32_t tok, int want_next, uint32_t *next, float *logits) {
    if (h->pos >= h->max_seq) return -1;
    const int dbg = debug_enabled() && h->tp <= 1; /* the dumps run the unsharded layer */
    if (h->resident) {
        if (register_layers(h)) return -1;
        if (dbg) {
            if (h->pos == 0) { /* the embedded first token and layer 0's intermediates */
                if (shk_cuda_model_embed(h->m, tok, NULL) != SHK_OK) return -1;
                float *emb = (float *)malloc((size_t)h->n_embd * 4);
                const int r = !emb || debug_dev(h->ctx, "embed", shk_cuda_model_hidden(h->m), h->n_embd, emb);
                free(emb);
                if (r) return -1;
            }
            for (uint32_t l = 0; l < h->n_layers; ++l) { /* each layer's line, layer 0's stats after its own */
                debug_dtypes(h, l);
                if (l == 0 && h->pos == 0) {
                    struct shk_layer_desc d0;
                    layer_desc(h, 0, (const uint8_t *)h->d_buf[0], &d0);
                    if (debug_layer0(h, &d0, shk_cuda_model_hidden(h->m))) return -1;
                }
            }
        }
        const int e = shk_cuda_token_step(h->m, tok, h->pos, want_next, next, logits);
        if (e != SHK_OK) {
            fprintf(stderr, "engine: position %u: token step failed (%d)\n", h->pos, e);
            return -1;
        }
    } else {
        if (shk_cuda_model_embed(h->m, tok, NULL) != SHK_OK) return -1;
        float *hidden = shk_cuda_model_hidden(h->m);
        if (dbg && h->pos == 0) {
            float *emb = (float *)malloc((size_t)h->n_embd * 4);
            const int r = !emb || debug_dev(h->ctx, "embed", hidden, h->n_embd, emb);
            free(emb);
            if (r) return -1;
        }
        for (uint32_t l = 0; l < h->n_layers; ++l) {
            const uint64_t k = h->ring_next++; /* k % n_layers == l: passes run whole */
            if (acquire(h, k)) return -1;
            struct shk_layer_desc d;
            layer_desc(h, l, (const uint8_t *)h->d_buf[k % h->depth], &d);
            if (dbg) {
                debug_dtypes(h, l);
                if (l == 0 && h->pos == 0 && debug_layer0(h, &d, hidden)) return -1;
            }
            if (shk_cuda_forward_layer(h->m, &d, l, h->pos, hidden, NULL) != SHK_OK) return -1;
            consume(h, k);
        }
        if (want_next && shk_cuda_model_lm_head(h->m, next, logits, NULL) != SHK_OK) return -1;
        if (!want_next && shk_cuda_check(h->ctx) != SHK_OK) return -1;
    }
    h->pos++;
    return 0;
}

/* engine/src/engine.c:306-501 token schedule. */
static int generate(struct engine_handle *h, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_decode,
                    token_callback cb, void *user, int print, float *logits_out) {
    static const uint32_t k_default = 1;
    if (!n_prompt) {
        prompt = &k_default;
        n_prompt = 1;
    }
    h->n_out = 0;
    h->text_len = 0;
    if (h->text) h->text[0] = '\0';
    h->cancel = 0;
    h->pos = 0; /* each generation starts a new sequence */
    shk_cuda_kv_clear(h->kv);
    if (!h->resident) {
        /* the ring streams exactly the passes this generation runs, like the
         * reference's per-token requests: one per layer per prompt token and
         * per generated token */
        pthread_mutex_lock(&h->mu);
        h->n_req = h->ring_next + (uint64_t)(n_prompt + n_decode) * h->n_layers;
        pthread_cond_broadcast(&h->cv);
        pthread_mutex_unlock(&h->mu);
    }
    for (uint32_t i = 0; i < n_prompt; ++i)
        if (prompt[i] >= h->n_vocab) return -1;
    /* tensor parallel: ranks 1.. run the same steps on their own threads */
    pthread_t th[8];
    uint32_t started = 0;
    if (h->tp > 1) {
        if (h->tp_broken) return -1;
        for (uint32_t ri = 1; ri < h->tp; ++ri) {
            struct tp_rank *r = &h->ranks[ri];
            r->prompt = prompt;
            r->n_prompt = n_prompt;
            r->n_decode = n_decode;
            r->want_logits = logits_out != NULL;
            if (r->want_logits && !r->lg && !(r->lg = (float *)malloc((size_t)h->n_vocab * 4))) break;
            if (pthread_create(&th[ri], NULL, tp_rank_main, r) != 0) break;
            started = ri;
        }
        if (started + 1 != h->tp) {
            h->tp_broken = 1; /* the started ranks wait for rank 0 in their collectives */
            return -1;
        }
    }
    int rc = 0;
    uint32_t next = 0, first = 0;
    /* prompts of SHUKUCHI_PREFILL tokens or more (0, the default: never):
     * one batched prefill on the tensor cores instead of a step per token
     * (single GPU, HBM-resident, Q4_K / Q6_K weights; else the token loop
     * below).  Off by default: its f16 matmul inputs move the logits away
     * from the reference's by more than the decode path's tolerance. */
    const int pf_min = env_int("SHUKUCHI_PREFILL", 0);
    if (pf_min > 0 && n_prompt >= (uint32_t)pf_min && h->resident && h->tp <= 1 && !debug_enabled() &&
        !register_layers(h)) {
        const int r = shk_cuda_prefill(h->m, prompt, n_prompt, 0, &next, logits_out, NULL);
        if (r == SHK_OK) {
            h->pos = n_prompt;
            first = n_prompt;
        } else if (r != SHK_EUNSUPPORTED) {
            rc = -1;
        }
    }
    for (uint32_t i = first; i < n_prompt && !rc; ++i) {
        const int last = i + 1 == n_prompt;
        rc = step(h, prompt[i], last, &next, last ? logits_out : NULL);
    }
    /* cancellation ends a generation between tokens; tensor-parallel ranks
     * run every step in lockstep, so there it takes effect at the end */
    for (uint32_t j = 0; j < n_decode && !rc && (h->tp > 1 || !h->cancel); ++j) {
        rc = emit(h, next, cb, user, print);
        const int want = j + 1 < n_decode;
        float *lg = (want && logits_out) ? logits_out + (size_t)(j + 1) * h->n_vocab : NULL;
        uint32_t nx = 0;
        if (!rc) rc = step(h, next, want, &nx, lg);
        if (want) next = nx;
        note_rss(h);
    }
    if (h->tp > 1) {
        if (rc) {
            h->tp_broken = 1; /* ranks left blocked in a collective: the handle is unusable */
            return -1;
        }
        for (uint32_t ri = 1; ri < h->tp; ++ri) {
            pthread_join(th[ri], NULL);
            rc |= h->ranks[ri].rc;
        }
    }
    if (rc) return -1;
    if (print) printf("\n");
    return 0;
}

/* ------------------------- tensor parallelism ---------------------------- */
/* SHUKUCHI_TP = 2, 4 or 8 (resident mode): one GPU (SHUKUCHI_DEVICE + r),
 * context and thread per rank, an NCCL communicator across them.  The split
 * is the Megatron-style one, and the same as the Python side's
 * shukuchi_b200/tp.py: Wq/Wk/Wv and gate/up are cut by output rows, Wo and
 * down by input columns in whole 256-element blocks, KV heads stay local to a
 * rank.  Query head h reads KV head h % n_kv (engine/src/ops.c:423), so a rank
 * owning KV heads [kv_lo, kv_hi) owns the query heads whose h % n_kv falls
 * there, stored in the order (group g, KV head j).  When one KV head per rank
 * would leave Wo column groups that are not whole blocks, A ranks share the
 * heads and split the O projection's output rows.  The output head is split
 * by vocabulary rows when n_vocab divides by the world (argmax merged over
 * the ranks on the device), else replicated.  Each layer's span is read once
 * into pinned staging and every rank copies its slices out of it with
 * strided copies on its own copy stream. */

int engine_tp_layout(const uint32_t shape[6], uint32_t rank, uint32_t world, uint32_t out[9]) {
    const uint32_t D = shape[0], H = shape[1], KV = shape[2], hd = shape[3], F = shape[4], V = shape[5];
    if (!world || rank >= world || !KV || !H || H % KV || F % 256 || F / 256 < world) return -1;
    uint32_t A = 0, kvp = 0;
    for (uint32_t a = 1; a <= world && !A; ++a) {
        if (world % a || (KV * a) % world || D % a) continue;
        kvp = KV * a / world;
        if ((kvp * hd) % 256 == 0 || (kvp == KV && (H * hd) % 256 == 0)) A = a;
    }
    if (!A) return -1;
    const uint32_t g = rank / A, ar = rank % A, rows = D / A, fb = F / 256;
    out[0] = A;
    out[1] = g * kvp;
    out[2] = (g + 1) * kvp;
    out[3] = ar * rows;
    out[4] = (ar + 1) * rows;
    out[5] = (uint32_t)((uint64_t)rank * fb / world) * 256;
    out[6] = (uint32_t)((uint64_t)(rank + 1) * fb / world) * 256;
    out[7] = V % world == 0 ? rank * (V / world) : 0;
    out[8] = V % world == 0 ? (rank + 1) * (V / world) : V;
    return 0;
}

static uint64_t blk_bytes(uint32_t type) { return type == 12 ? 144 : type == 13 ? 176 : type == 14 ? 210 : 0; }

struct piece {             /* one strided copy out of the layer's pinned span */
    uint64_t src_off;      /* from the tensor's first byte */
    uint64_t src_pitch, width, rows;
    uint64_t dst_off;      /* from the shard's first byte */
};
struct shard {
    uint64_t rows, cols, pitch; /* shard rows, elements per row, bytes between rows */
    int padded;                 /* pitch > dense row bytes (Q6_K V / down) */
    uint32_t np;
    struct piece p[8];
};

/* Rank `lay`'s slice of tensor t of layer l. */
static int tp_shard(const struct engine_handle *h, const struct tensor_loc *tl, int t, const struct tp_layout *lay,
                    struct shard *sh) {
    const uint64_t hd = h->head_dim, KV = h->n_kv, G = h->n_heads / h->n_kv, kvp = lay->kv_hi - lay->kv_lo;
    const uint64_t rb = tl->row_bytes, bb = blk_bytes(tl->type);
    memset(sh, 0, sizeof(*sh));
    if (t == TN_ATTN_NORM || t == TN_FFN_NORM) {
        sh->rows = 1;
        sh->cols = tl->size / 4;
        sh->pitch = tl->size;
        sh->np = 1;
        sh->p[0] = (struct piece){0, tl->size, tl->size, 1, 0};
        return 0;
    }
    if (!bb || rb % bb) return -1;
    const uint64_t full_cols = rb / bb * 256;
    uint64_t width = rb;
    switch (t) {
    case TN_Q:
        sh->rows = G * kvp * hd;
        sh->cols = full_cols;
        if (G > 8) return -1;
        for (uint64_t g = 0; g < G; ++g)
            sh->p[sh->np++] = (struct piece){(g * KV + lay->kv_lo) * hd * rb, rb, rb, kvp * hd, g * kvp * hd};
        break;
    case TN_K:
    case TN_V:
        sh->rows = kvp * hd;
        sh->cols = full_cols;
        sh->p[sh->np++] = (struct piece){lay->kv_lo * hd * rb, rb, rb, kvp * hd, 0};
        break;
    case TN_O: {
        sh->rows = lay->o_hi - lay->o_lo;
        /* column ranges of this rank's heads, merged where adjacent */
        uint64_t c0[8], c1[8], n = 0;
        if (G > 8) return -1;
        for (uint64_t g = 0; g < G; ++g) {
            const uint64_t a = (g * KV + lay->kv_lo) * hd, b = a + kvp * hd;
            if (n && c1[n - 1] == a)
                c1[n - 1] = b;
            else {
                c0[n] = a;
                c1[n] = b;
                ++n;
            }
        }
        width = 0;
        for (uint64_t i = 0; i < n; ++i) {
            if (c0[i] % 256 || c1[i] % 256) return -1;
            const uint64_t w = (c1[i] - c0[i]) / 256 * bb;
            sh->p[sh->np++] = (struct piece){lay->o_lo * rb + c0[i] / 256 * bb, rb, w, sh->rows, width};
            width += w;
        }
        sh->cols = width / bb * 256;
        break;
    }
    case TN_GATE:
    case TN_UP:
        sh->rows = lay->f_hi - lay->f_lo;
        sh->cols = full_cols;
        sh->p[sh->np++] = (struct piece){lay->f_lo * rb, rb, rb, sh->rows, 0};
        break;
    case TN_DOWN:
        sh->rows = tl->rows;
        width = (lay->f_hi - lay->f_lo) / 256 * bb;
        sh->cols = lay->f_hi - lay->f_lo;
        sh->p[sh->np++] = (struct piece){lay->f_lo / 256 * bb, rb, width, sh->rows, 0};
        break;
    default:
        return -1;
    }
    sh->pitch = width;
    if (width % 16) {
        /* Q6_K rows whose width is not a 16-byte multiple: padded rows, as the
         * single-GPU loader pads them; only V and down carry a row stride */
        if (t != TN_V && t != TN_DOWN) return -1;
        sh->pitch = (width + 15) & ~(uint64_t)15;
        sh->padded = 1;
    }
    /* destination offsets of row-packed pieces are in rows: scale to bytes */
    for (uint32_t i = 0; i < sh->np; ++i)
        if (t == TN_Q) sh->p[i].dst_off *= sh->pitch;
    return 0;
}

struct tp_init_job {
    struct engine_handle *h;
    struct tp_rank *r;
    const uint8_t *id;
    int rc;
};

/* Per-rank setup that joins the communicator (NCCL initialisation is
 * collective: every rank's call runs concurrently, one thread each). */
static void *tp_init_main(void *arg) {
    struct tp_init_job *j = (struct tp_init_job *)arg;
    struct engine_handle *h = j->h;
    struct tp_rank *r = j->r;
    j->rc = -1;
    if (shk_cuda_tp_init(r->ctx, (int)r->rank, (int)h->tp, j->id) != SHK_OK) return NULL;
    const uint32_t kvp = r->lay.kv_hi - r->lay.kv_lo;
    struct shk_kv_config kc = {h->n_layers, kvp, h->head_dim, 32, h->max_seq};
    r->kv = shk_cuda_kv_create(r->ctx, &kc);
    if (!r->kv) return NULL;
    j->rc = 0;
    return NULL;
}

/* Reads rows [r0, r0 + n) of a tensor into pinned memory and copies them to a
 * new device buffer of this rank (Q6_K rows converted to the planar layout
 * when they are 16-byte multiples). */
static int tp_upload_rows(struct engine_handle *h, struct tp_rank *r, const struct gguf_tensor_info *ti,
                          uint64_t r0, uint64_t n, void **dev, uint32_t *dtype) {
    const uint64_t rows = ti->n_dims == 2 ? ti->dims[1] : 1, rb = ti->size / rows, bytes = n * rb;
    void *host = NULL;
    if (shk_cuda_host_alloc(r->ctx, bytes, &host) != SHK_OK) return -1;
    int rc = pread_all(h->g.fd, host, bytes, ti->offset + r0 * rb);
    if (!rc) rc = shk_cuda_dev_alloc(r->ctx, bytes, dev) == SHK_OK ? 0 : -1;
    if (!rc) rc = shk_cuda_memcpy_h2d(r->ctx, *dev, host, bytes, NULL) == SHK_OK ? 0 : -1;
    if (!rc) rc = shk_cuda_sync(r->ctx, NULL) == SHK_OK ? 0 : -1;
    shk_cuda_host_free(r->ctx, host);
    *dtype = ti->type;
    if (!rc && ti->type == 14 && rb % 16 == 0) {
        rc = shk_cuda_q6k_repack(r->ctx, *dev, (uint32_t)n, (uint32_t)(rb / 210 * 256), 0, 1, NULL) == SHK_OK &&
                     shk_cuda_sync(r->ctx, NULL) == SHK_OK
                 ? 0
                 : -1;
        *dtype = SHK_DTYPE_Q6_K_PLANAR;
    }
    return rc;
}

/* Every layer: its span read once into pinned staging (two buffers
 * alternating), each rank's slices copied into the rank's device buffer for
 * the layer (Q6_K shards converted to the planar layout there) and
 * registered with the rank's model. */
static int tp_stage_layers(struct engine_handle *h) {
    for (uint32_t l = 0; l < h->n_layers; ++l) {
        const struct layer_map *L = &h->lm[l];
        const uint32_t s = l % 2;
        for (uint32_t ri = 0; ri < h->tp; ++ri) /* the pinned buffer's previous copies landed */
            if (shk_cuda_layer_ready(h->ranks[ri].ctx, s, 1) < 0) return -1;
        uint8_t *pin = (uint8_t *)h->pinned[s];
        if (pread_span(h->g.fd, pin, L->span_len, L->span_off)) return -1;
        h->st.layer_loads++;
        h->st.layer_bytes_read += L->span_len;
        for (uint32_t ri = 0; ri < h->tp; ++ri) {
            struct tp_rank *r = &h->ranks[ri];
            struct shard sh[TN_COUNT];
            uint64_t off[TN_COUNT], dev = 0;
            for (int t = 0; t < TN_COUNT; ++t) {
                if (tp_shard(h, &L->t[t], t, &r->lay, &sh[t])) return -1;
                off[t] = dev;
                dev = al256(dev + sh[t].pitch * sh[t].rows);
            }
            if (shk_cuda_dev_alloc(r->ctx, dev, &r->d_buf[l]) != SHK_OK) return -1;
            uint8_t *base = (uint8_t *)r->d_buf[l];
            for (int t = 0; t < TN_COUNT; ++t) {
                const struct tensor_loc *tl = &L->t[t];
                const uint8_t *src = pin + (tl->off - L->span_off);
                for (uint32_t i = 0; i < sh[t].np; ++i) {
                    const struct piece *pc = &sh[t].p[i];
                    if (shk_cuda_layer_stage_2d(r->ctx, s, base + off[t] + pc->dst_off, sh[t].pitch,
                                                src + pc->src_off, pc->src_pitch, pc->width, pc->rows) != SHK_OK)
                        return -1;
                }
                if (tl->type == 14 &&
                    shk_cuda_layer_stage_q6k_planar(r->ctx, s, base + off[t], (uint32_t)sh[t].rows,
                                                    (uint32_t)sh[t].cols,
                                                    (uint32_t)(sh[t].padded ? sh[t].pitch : 0)) != SHK_OK)
                    return -1;
            }
            if (shk_cuda_layer_commit(r->ctx, s) != SHK_OK) return -1;
            struct shk_layer_desc *d = &r->ld[l];
            memset(d, 0, sizeof(*d));
            d->attn_norm = (const float *)(base + off[TN_ATTN_NORM]);
            d->ffn_norm = (const float *)(base + off[TN_FFN_NORM]);
            d->attn_q = base + off[TN_Q];
            d->attn_k = base + off[TN_K];
            d->attn_v = base + off[TN_V];
            d->attn_o = base + off[TN_O];
            d->ffn_gate = base + off[TN_GATE];
            d->ffn_up = base + off[TN_UP];
            d->ffn_down = base + off[TN_DOWN];
#define DT(i) (L->t[i].type == 14 ? SHK_DTYPE_Q6_K_PLANAR : L->t[i].type)
            d->attn_q_dtype = DT(TN_Q);
            d->attn_k_dtype = DT(TN_K);
            d->attn_v_dtype = DT(TN_V);
            d->attn_o_dtype = DT(TN_O);
            d->ffn_gate_dtype = DT(TN_GATE);
            d->ffn_up_dtype = DT(TN_UP);
            d->ffn_down_dtype = DT(TN_DOWN);
#undef DT
            d->row_stride_v = sh[TN_V].padded ? (uint32_t)sh[TN_V].pitch : 0;
            d->row_stride_down = sh[TN_DOWN].padded ? (uint32_t)sh[TN_DOWN].pitch : 0;
        }
    }
    for (uint32_t ri = 0; ri < h->tp; ++ri) {
        struct tp_rank *r = &h->ranks[ri];
        for (uint32_t s = 0; s < 2; ++s)
            if (shk_cuda_layer_ready(r->ctx, s, 1) < 0 || shk_cuda_layer_wait(r->ctx, s, NULL) != SHK_OK) return -1;
        for (uint32_t l = 0; l < h->n_layers; ++l)
            if (shk_cuda_model_set_layer(r->m, l, &r->ld[l]) != SHK_OK) return -1;
        if (shk_cuda_sync(r->ctx, NULL) != SHK_OK) return -1;
    }
    h->registered = 1;
    return 0;
}

static int tp_open(struct engine_handle *h) {
    if (!h->resident) return -1; /* tensor parallel runs from HBM-resident shards */
    const int base = env_int("SHUKUCHI_DEVICE", 0);
    h->ranks = (struct tp_rank *)calloc(h->tp, sizeof(struct tp_rank));
    if (!h->ranks) return -1;
    const uint32_t shape[6] = {h->n_embd, h->n_heads, h->n_kv, h->head_dim, h->n_ff, h->n_vocab};
    for (uint32_t ri = 0; ri < h->tp; ++ri) {
        struct tp_rank *r = &h->ranks[ri];
        r->rank = ri;
        uint32_t o[9];
        if (engine_tp_layout(shape, ri, h->tp, o)) return -1;
        r->lay = (struct tp_layout){o[0], o[1], o[2], o[3], o[4], o[5], o[6], o[7], o[8]};
        struct shk_cuda_config cc = {base + (int)ri, 0};
        r->ctx = shk_cuda_init(&cc);
        r->d_buf = (void **)calloc(h->n_layers, sizeof(void *));
        r->ld = (struct shk_layer_desc *)calloc(h->n_layers, sizeof(struct shk_layer_desc));
        if (!r->ctx || !r->d_buf || !r->ld) return -1;
    }
    uint8_t id[SHK_TP_ID_BYTES];
    if (shk_cuda_tp_unique_id(id, sizeof(id)) <= 0) return -1;
    struct tp_init_job jobs[8];
    pthread_t th[8];
    if (h->tp > 8) return -1;
    for (uint32_t ri = 0; ri < h->tp; ++ri) {
        jobs[ri] = (struct tp_init_job){h, &h->ranks[ri], id, -1};
        if (pthread_create(&th[ri], NULL, tp_init_main, &jobs[ri]) != 0) {
            for (uint32_t j = 0; j < ri; ++j) pthread_join(th[j], NULL);
            return -1;
        }
    }
    int rc = 0;
    for (uint32_t ri = 0; ri < h->tp; ++ri) {
        pthread_join(th[ri], NULL);
        rc |= jobs[ri].rc;
    }
    if (rc) return -1;
    const struct gguf_tensor_info *emb = gguf_find_tensor(&h->g, "token_embd.weight");
    const struct gguf_tensor_info *out = gguf_find_tensor(&h->g, "output.weight");
    for (uint32_t ri = 0; ri < h->tp; ++ri) {
        struct tp_rank *r = &h->ranks[ri];
        uint32_t emb_t = 0, out_t = 0;
        if (tp_upload_rows(h, r, emb, 0, h->n_vocab, &r->d_embd, &emb_t)) return -1;
        if (emb_t != emb->type) return -1; /* the embedding table keeps its GGUF layout */
        if (tp_upload_rows(h, r, out, r->lay.v_lo, r->lay.v_hi - r->lay.v_lo, &r->d_out, &out_t)) return -1;
        const uint32_t kvp = r->lay.kv_hi - r->lay.kv_lo, G = h->n_heads / h->n_kv;
        struct shk_model_desc md = {h->n_layers, h->n_embd, G * kvp, kvp, h->head_dim,
                                    r->lay.f_hi - r->lay.f_lo, h->n_vocab, 10000.0f, r->d_embd, emb->type,
                                    r->d_out, out_t};
        r->m = shk_cuda_model_create(r->ctx, &md, r->kv);
        if (!r->m) return -1;
        if (shk_cuda_model_set_tp_rows(r->m, r->lay.o_lo, r->lay.o_hi, r->lay.v_lo, r->lay.v_hi) != SHK_OK)
            return -1;
    }
    /* rank 0 is the handle's own context (reports, the debug dumps' device) */
    h->ctx = h->ranks[0].ctx;
    h->kv = h->ranks[0].kv;
    h->m = h->ranks[0].m;
    h->pinned = (void **)calloc(2, sizeof(void *));
    if (!h->pinned) return -1;
    h->depth = 2;
    for (uint32_t i = 0; i < 2; ++i)
        if (shk_cuda_host_alloc(h->ctx, h->max_span, &h->pinned[i]) != SHK_OK) return -1;
    h->st.max_layer_size = (size_t)h->max_span;
    h->st.peak_buffer_usage = (size_t)h->max_span * 2;
    h->st.max_concurrent_buffers = 2;
    return tp_stage_layers(h);
}

static void tp_close(struct engine_handle *h) {
    for (uint32_t ri = 0; h->ranks && ri < h->tp; ++ri) {
        struct tp_rank *r = &h->ranks[ri];
        if (r->ctx) shk_cuda_sync(r->ctx, NULL);
        if (r->m) shk_cuda_model_destroy(r->m);
        if (r->kv) shk_cuda_kv_destroy(r->kv);
        if (r->ctx) {
            for (uint32_t l = 0; r->d_buf && l < h->n_layers; ++l)
                if (r->d_buf[l]) shk_cuda_dev_free(r->ctx, r->d_buf[l]);
            if (r->d_embd) shk_cuda_dev_free(r->ctx, r->d_embd);
            if (r->d_out) shk_cuda_dev_free(r->ctx, r->d_out);
        }
    }
    if (h->pinned && h->ranks && h->ranks[0].ctx)
        for (uint32_t i = 0; i < 2; ++i)
            if (h->pinned[i]) shk_cuda_host_free(h->ranks[0].ctx, h->pinned[i]);
    free(h->pinned);
    h->pinned = NULL;
    for (uint32_t ri = 0; h->ranks && ri < h->tp; ++ri) {
        struct tp_rank *r = &h->ranks[ri];
        if (r->ctx) shk_cuda_shutdown(r->ctx);
        free(r->d_buf);
        free(r->ld);
        free(r->lg);
    }
    free(h->ranks);
    h->ranks = NULL;
    h->ctx = NULL;
    h->kv = NULL;
    h->m = NULL;
}

/* A rank's token loop (ranks 1..world-1 on their own threads; rank 0 runs in
 * generate()): the same steps on every rank, in lockstep through the
 * collectives inside each step; every rank gets the same next token. */
static void *tp_rank_main(void *arg) {
    struct tp_rank *r = (struct tp_rank *)arg;
    r->rc = -1;
    shk_cuda_kv_clear(r->kv);
    uint32_t pos = 0, next = 0;
    for (uint32_t i = 0; i < r->n_prompt; ++i, ++pos) {
        const int last = i + 1 == r->n_prompt;
        float *lg = (last && r->want_logits) ? r->lg : NULL;
        const int e = shk_cuda_token_step(r->m, r->prompt[i], pos, last, &next, lg);
        if (e != SHK_OK) {
            fprintf(stderr, "engine: rank %u, prompt position %u: token step failed (%d)\n", r->rank, pos, e);
            return NULL;
        }
    }
    for (uint32_t j = 0; j < r->n_decode; ++j, ++pos) {
        const int want = j + 1 < r->n_decode;
        uint32_t nx = 0;
        float *lg = (want && r->want_logits) ? r->lg : NULL;
        const int e = shk_cuda_token_step(r->m, next, pos, want, &nx, lg);
        if (e != SHK_OK) {
            fprintf(stderr, "engine: rank %u, position %u: token step failed (%d)\n", r->rank, pos, e);
            return NULL;
        }
        if (want) next = nx;
    }
    r->rc = 0;
    return NULL;
}

/* ------------------------------- public --------------------------------- */

void engine_close(engine_handle_t *h) {
    if (!h) return;
    if (h->thr_started) {
        pthread_mutex_lock(&h->mu);
        h->stop = 1;
        pthread_cond_broadcast(&h->cv);
        pthread_mutex_unlock(&h->mu);
        pthread_join(h->thr, NULL);
    }
    if (h->ranks) {
        if (h->tp_broken) { /* rank threads may still hold the contexts: leave them */
            gguf_close(&h->g);
            return;
        }
        tp_close(h);
    }
    if (h->ctx) shk_cuda_sync(h->ctx, NULL);
    if (h->m) shk_cuda_model_destroy(h->m);
    if (h->kv) shk_cuda_kv_destroy(h->kv);
    if (h->ctx) {
        for (uint32_t i = 0; h->d_buf && i < h->n_buf; ++i)
            if (h->d_buf[i]) shk_cuda_dev_free(h->ctx, h->d_buf[i]);
        for (uint32_t i = 0; h->pinned && i < h->depth; ++i)
            if (h->pinned[i]) shk_cuda_host_free(h->ctx, h->pinned[i]);
        if (h->d_embd) shk_cuda_dev_free(h->ctx, h->d_embd);
        if (h->d_out) shk_cuda_dev_free(h->ctx, h->d_out);
        shk_cuda_shutdown(h->ctx);
    }
    free(h->d_buf);
    free(h->pinned);
    free(h->lm);
    free(h->vocab_slot);
    free(h->prompt);
    free(h->out_ids);
    free(h->text);
    pthread_mutex_destroy(&h->mu);
    pthread_cond_destroy(&h->cv);
    gguf_close(&h->g);
    free(h);
}

engine_handle_t *engine_open(const char *model_path, const struct engine_config *cfg) {
    if (!model_path) return NULL;
    struct engine_handle *h = (struct engine_handle *)calloc(1, sizeof(*h));
    if (!h) return NULL;
    h->g.fd = -1;
    pthread_mutex_init(&h->mu, NULL);
    pthread_cond_init(&h->cv, NULL);
    if (cfg) h->cfg = *cfg;
    h->depth = h->cfg.prefetch_depth ? h->cfg.prefetch_depth : 2;
    if (h->depth < 2) h->depth = 2;
    if (h->depth > 3) h->depth = 3;
    h->resident = env_int("SHUKUCHI_HBM_RESIDENT", 1) != 0;
    h->max_seq = (uint32_t)env_int("SHUKUCHI_MAX_SEQ", 2048);
    if (model_file_open(model_path, &h->g) || map_model(h) || vocab_index_build(h)) goto fail;
    h->tp = (uint32_t)env_int("SHUKUCHI_TP", 1);
    if (h->tp != 1 && h->tp != 2 && h->tp != 4 && h->tp != 8) goto fail;
    if (h->tp > 1) {
        if (tp_open(h)) goto fail;
        return h;
    }
    struct shk_cuda_config cc = {env_int("SHUKUCHI_DEVICE", 0), 0};
    h->ctx = shk_cuda_init(&cc);
    if (!h->ctx) goto fail;
    struct shk_kv_config kc = {h->n_layers, h->n_kv, h->head_dim, h->cfg.kv_block_size ? h->cfg.kv_block_size : 32,
                               h->max_seq};
    h->kv = shk_cuda_kv_create(h->ctx, &kc);
    if (!h->kv) goto fail;
    const struct gguf_tensor_info *emb = gguf_find_tensor(&h->g, "token_embd.weight");
    const struct gguf_tensor_info *out = gguf_find_tensor(&h->g, "output.weight");
    if (upload_tensor(h, emb, &h->d_embd) || upload_tensor(h, out, &h->d_out)) goto fail;
    uint32_t out_type = out->type;
    if (out_type == 14 && (out->size / out->dims[1]) % 16 == 0) { /* planar Q6_K head */
        if (shk_cuda_q6k_repack(h->ctx, h->d_out, (uint32_t)out->dims[1], h->n_embd, 0, 1, NULL) != SHK_OK ||
            shk_cuda_sync(h->ctx, NULL) != SHK_OK)
            goto fail;
        out_type = SHK_DTYPE_Q6_K_PLANAR;
    }
    struct shk_model_desc md = {h->n_layers, h->n_embd, h->n_heads, h->n_kv, h->head_dim, h->n_ff, h->n_vocab,
                                10000.0f /* engine/src/ops.c:223: the reference's fixed theta */,
                                h->d_embd, emb->type, h->d_out, out_type};
    h->m = shk_cuda_model_create(h->ctx, &md, h->kv);
    if (!h->m) goto fail;
    h->n_buf = h->resident ? h->n_layers : h->depth;
    h->d_buf = (void **)calloc(h->n_buf, sizeof(void *));
    h->pinned = (void **)calloc(h->depth, sizeof(void *));
    if (!h->d_buf || !h->pinned) goto fail;
    for (uint32_t i = 0; i < h->n_buf; ++i)
        if (shk_cuda_dev_alloc(h->ctx, h->max_dev, &h->d_buf[i]) != SHK_OK) goto fail;
    for (uint32_t i = 0; i < h->depth; ++i)
        if (shk_cuda_host_alloc(h->ctx, h->max_span, &h->pinned[i]) != SHK_OK) goto fail;
    h->st.max_layer_size = (size_t)h->max_span;
    h->st.peak_buffer_usage = (size_t)h->max_span * h->depth;
    h->st.max_concurrent_buffers = h->depth;
    h->n_req = h->resident ? h->n_layers : 0; /* ring: set per generation */
    if (pthread_create(&h->thr, NULL, loader_main, h) != 0) goto fail;
    h->thr_started = 1;
    return h;
fail:
    engine_close(h);
    return NULL;
}

int engine_set_prompt(engine_handle_t *h, const char *prompt) {
    if (!h) return -1;
    free(h->prompt);
    h->prompt = prompt ? strdup(prompt) : NULL;
    return (prompt && !h->prompt) ? -1 : 0;
}

static int generate_text(engine_handle_t *h, uint32_t max_tokens, token_callback cb, void *user, int print) {
    if (!h || max_tokens == 0) return -1;
    uint32_t *ids = NULL, n = 0;
    if (tokenize(h, h->prompt ? h->prompt : "", &ids, &n)) return -1;
    const int rc = generate(h, ids, n, max_tokens, cb, user, print, NULL);
    free(ids);
    return rc;
}

int engine_generate(engine_handle_t *h, uint32_t max_tokens) { return generate_text(h, max_tokens, NULL, NULL, 1); }

int engine_generate_stream(engine_handle_t *h, uint32_t max_tokens, token_callback cb, void *user) {
    return generate_text(h, max_tokens, cb, user, 0);
}

int engine_generate_ids(engine_handle_t *h, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_decode,
                        uint32_t *out_ids, float *out_logits) {
    if (!h || !n_decode || (n_prompt && !prompt)) return -1;
    const int rc = generate(h, prompt, n_prompt, n_decode, NULL, NULL, 0, out_logits);
    if (!rc && out_ids) memcpy(out_ids, h->out_ids, h->n_out * sizeof(uint32_t));
    return rc ? rc : (int)h->n_out;
}

const char *engine_get_output(engine_handle_t *h) { return (h && h->text) ? h->text : ""; }

const uint32_t *engine_get_tokens(engine_handle_t *h, size_t *n) {
    if (n) *n = h ? h->n_out : 0;
    return h ? h->out_ids : NULL;
}

void engine_cancel(engine_handle_t *h) {
    if (h) h->cancel = 1;
}

int engine_get_streaming_stats(engine_handle_t *h, struct streaming_stats *out) {
    if (!h || !out) return -1;
    note_rss(h);
    pthread_mutex_lock(&h->mu);
    *out = h->st;
    pthread_mutex_unlock(&h->mu);
    return 0;
}

uint32_t engine_vocab_size(engine_handle_t *h) { return h ? h->n_vocab : 0; }

void engine_report(engine_handle_t *h) {
    if (h && h->ctx) shk_cuda_report(h->ctx);
}

int engine_tokenize_file(const char *model_path, const char *text, uint32_t *out, uint32_t cap) {
    struct engine_handle *h = (struct engine_handle *)calloc(1, sizeof(*h));
    if (!h) return -1;
    h->g.fd = -1;
    int rc = model_file_open(model_path, &h->g);
    if (!rc) {
        map_vocab(h);
        rc = vocab_index_build(h);
    }
    uint32_t *ids = NULL, n = 0;
    if (!rc) rc = tokenize(h, text, &ids, &n);
    if (!rc) {
        for (uint32_t i = 0; i < n && i < cap; ++i) out[i] = ids[i];
        rc = (int)n;
    }
    free(ids);
    free(h->vocab_slot);
    gguf_close(&h->g);
    free(h);
    return rc;
}

int engine_inspect(const char *model_path, uint32_t out[6], uint64_t *max_layer_bytes) {
    struct engine_handle *h = (struct engine_handle *)calloc(1, sizeof(*h));
    if (!h) return -1;
    int rc = model_file_open(model_path, &h->g);
    if (!rc) rc = map_model(h);
    if (!rc) {
        out[0] = h->n_layers;
        out[1] = h->n_embd;
        out[2] = h->n_heads;
        out[3] = h->n_kv;
        out[4] = h->n_ff;
        out[5] = h->n_vocab;
        if (max_layer_bytes) *max_layer_bytes = h->max_span;
    }
    free(h->lm);
    gguf_close(&h->g);
    free(h);
    return rc;
}
