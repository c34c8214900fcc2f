/* lstr.c -- LSTR container reader (format in lstr.h) and XXH64.
 *
 * lstr_open fills the same file index the GGUF reader produces (struct
 * gguf_file: the llama.* metadata, the vocabulary, named tensors at absolute
 * file offsets), so the loader, the tokenizer and the model map are shared:
 * a layer's nine tensors sit in one aligned block, which the loader reads
 * with one pread into pinned staging.
 */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "lstr.h"

#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "gguf.h"

/* ---------------------------------- XXH64 ---------------------------------- */
/* The published XXH64 algorithm (Y. Collet, xxHash specification v0.1.1):
 * four 64-bit lanes over 32-byte stripes, then the tail in 8 / 4 / 1-byte
 * steps and the final avalanche. */
static const uint64_t P1 = 0x9E3779B185EBCA87ull, P2 = 0xC2B2AE3D27D4EB4Full, P3 = 0x165667B19E3779F9ull,
                      P4 = 0x85EBCA77C2B2AE63ull, P5 = 0x27D4EB2F165667C5ull;

static uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
static uint64_t rd64(const uint8_t *p) {
    uint64_t v;
    memcpy(&v, p, 8);
    return v;
}
static uint32_t rd32(const uint8_t *p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}
static uint64_t xround(uint64_t acc, uint64_t in) { return rotl64(acc + in * P2, 31) * P1; }
static uint64_t xmerge(uint64_t h, uint64_t v) { return (h ^ xround(0, v)) * P1 + P4; }

uint64_t lstr_xxh64(const void *data, uint64_t len, uint64_t seed) {
    const uint8_t *p = (const uint8_t *)data, *end = p + len;
    uint64_t h;
    if (len >= 32) {
        uint64_t v1 = seed + P1 + P2, v2 = seed + P2, v3 = seed, v4 = seed - P1;
        for (; p + 32 <= end; p += 32) {
            v1 = xround(v1, rd64(p));
            v2 = xround(v2, rd64(p + 8));
            v3 = xround(v3, rd64(p + 16));
            v4 = xround(v4, rd64(p + 24));
        }
        h = rotl64(v1, 1) + rotl64(v2, 7) + rotl64(v3, 12) + rotl64(v4, 18);
        h = xmerge(xmerge(xmerge(xmerge(h, v1), v2), v3), v4);
    } else {
        h = seed + P5;
    }
    h += len;
    for (; p + 8 <= end; p += 8) h = rotl64(h ^ xround(0, rd64(p)), 27) * P1 + P4;
    if (p + 4 <= end) {
        h = rotl64(h ^ ((uint64_t)rd32(p) * P1), 23) * P2 + P3;
        p += 4;
    }
    for (; p < end; ++p) h = rotl64(h ^ ((uint64_t)*p * P5), 11) * P1;
    h ^= h >> 33;
    h *= P2;
    h ^= h >> 29;
    h *= P3;
    h ^= h >> 32;
    return h;
}

uint32_t lstr_dtype_of_ggml(uint32_t t) {
    switch (t) {
        case 0: return LSTR_DTYPE_F32;
        case 1: return LSTR_DTYPE_F16;
        case 12: return LSTR_DTYPE_Q4_K;
        case 13: return LSTR_DTYPE_Q5_K;
        case 14: return LSTR_DTYPE_Q6_K;
        default: return 0;
    }
}

uint32_t lstr_ggml_of_dtype(uint32_t d) {
    switch (d) {
        case LSTR_DTYPE_F32: return 0;
        case LSTR_DTYPE_F16: return 1;
        case LSTR_DTYPE_Q4_K: return 12;
        case LSTR_DTYPE_Q5_K: return 13;
        case LSTR_DTYPE_Q6_K: return 14;
        default: return 0xFFFFFFFFu;
    }
}

/* --------------------------------- reader ---------------------------------- */

static int pread_full(int fd, void *dst, uint64_t len, uint64_t off) {
    uint8_t *d = (uint8_t *)dst;
    while (len) {
        const ssize_t n = pread(fd, d, len > (1u << 30) ? (1u << 30) : len, (off_t)off);
        if (n < 0 && errno == EINTR) continue;
        if (n <= 0) return -1;
        d += n;
        off += (uint64_t)n;
        len -= (uint64_t)n;
    }
    return 0;
}

static const char *const k_layer_suffix[9] = {
    "attn_norm.weight", "attn_q.weight",   "attn_k.weight", "attn_v.weight",   "attn_output.weight",
    "ffn_norm.weight",  "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight"};

static int add_u32(struct gguf_file *f, const char *key, uint32_t v) {
    const uint64_t i = f->n_kv++;
    f->keys[i] = strdup(key);
    f->vals[i].type = GGUF_U32;
    f->vals[i].u = v;
    return f->keys[i] ? 0 : -1;
}

/* A tensor's rows x row-elements from its dtype and byte size, as GGUF dims
 * (dims[0] = elements per row). */
static int add_tensor(struct gguf_file *f, const char *name, uint32_t ggml, uint64_t off, uint64_t size,
                      uint64_t row_elems) {
    struct gguf_tensor_info *ti = &f->tensors[f->n_tensors++];
    ti->name = strdup(name);
    if (!ti->name || ggml == 0xFFFFFFFFu) return -1;
    ti->type = ggml;
    ti->offset = off;
    ti->size = size;
    const uint64_t row_bytes = gguf_type_bytes(ggml, row_elems);
    if (!row_bytes || size % row_bytes) return -1;
    ti->n_dims = size == row_bytes ? 1 : 2;
    ti->dims[0] = row_elems;
    ti->dims[1] = size / row_bytes;
    return 0;
}

int lstr_is(const char *path) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return 0;
    uint32_t m = 0;
    const int ok = pread_full(fd, &m, 4, 0) == 0 && m == LSTR_MAGIC;
    close(fd);
    return ok;
}

int lstr_open(const char *path, struct gguf_file *f) {
    memset(f, 0, sizeof(*f));
    f->fd = open(path, O_RDONLY);
    if (f->fd < 0) return -1;
    struct lstr_header hd;
    uint8_t *res = NULL;
    struct lstr_layer_index_entry *idx = NULL;
    struct lstr_tensor_entry *tt = NULL;
    if (pread_full(f->fd, &hd, sizeof(hd), 0) || hd.magic != LSTR_MAGIC || hd.endian_tag != LSTR_ENDIAN_TAG ||
        hd.version != LSTR_VERSION || hd.header_size != LSTR_HEADER_SIZE || !hd.n_layers || !hd.n_embd ||
        !hd.n_heads || hd.n_layers > (1u << 16) || hd.index_size != (uint64_t)hd.n_layers * sizeof(*idx) ||
        hd.resident_size > (1ull << 34) || hd.resident_size < 8)
        goto fail;
    idx = (struct lstr_layer_index_entry *)malloc(hd.index_size);
    res = (uint8_t *)malloc(8 + 64 * sizeof(struct lstr_tensor_entry)); /* the section's table only */
    if (!idx || !res || pread_full(f->fd, idx, hd.index_size, hd.index_offset)) goto fail;
    /* the resident section's table and its small records (not the tensors) */
    uint32_t n_res = 0;
    if (pread_full(f->fd, res, 8, hd.resident_offset)) goto fail;
    memcpy(&n_res, res, 4);
    if (!n_res || n_res > 64 || 8 + (uint64_t)n_res * sizeof(struct lstr_tensor_entry) > hd.resident_size ||
        pread_full(f->fd, res + 8, (uint64_t)n_res * sizeof(struct lstr_tensor_entry), hd.resident_offset + 8))
        goto fail;
    const struct lstr_tensor_entry *re = (const struct lstr_tensor_entry *)(res + 8);
    f->keys = (char **)calloc(16, sizeof(char *));
    f->vals = (struct gguf_value *)calloc(16, sizeof(struct gguf_value));
    f->tensors = (struct gguf_tensor_info *)calloc((size_t)hd.n_layers * 9 + 3, sizeof(struct gguf_tensor_info));
    if (!f->keys || !f->vals || !f->tensors) goto fail;
    struct lstr_meta meta;
    memset(&meta, 0, sizeof(meta));
    int have_meta = 0, have_vocab = 0;
    for (uint32_t i = 0; i < n_res; ++i) {
        const struct lstr_tensor_entry *e = &re[i];
        if (e->offset + e->size > hd.resident_size) goto fail;
        const uint64_t abs = hd.resident_offset + e->offset;
        if (e->tensor_id == LSTR_ID_META) {
            if (e->size < sizeof(meta) || pread_full(f->fd, &meta, sizeof(meta), abs)) goto fail;
            have_meta = 1;
        } else if (e->tensor_id == LSTR_ID_VOCAB) {
            uint8_t *v = (uint8_t *)malloc(e->size);
            if (!v || pread_full(f->fd, v, e->size, abs)) {
                free(v);
                goto fail;
            }
            uint32_t n = 0;
            memcpy(&n, v, 4);
            const uint64_t k = f->n_kv++;
            f->keys[k] = strdup("tokenizer.ggml.tokens");
            struct gguf_value *gv = &f->vals[k];
            gv->type = GGUF_ARRAY;
            gv->arr_type = GGUF_STRING;
            gv->arr_n = n;
            gv->arr_str = (char **)calloc(n ? n : 1, sizeof(char *));
            int bad = !f->keys[k] || !gv->arr_str || n > (1u << 26);
            uint64_t o = 4;
            for (uint32_t t = 0; !bad && t < n; ++t) {
                uint32_t len = 0;
                if (o + 4 > e->size) { bad = 1; break; }
                memcpy(&len, v + o, 4);
                o += 4;
                if (o + len > e->size || !(gv->arr_str[t] = (char *)malloc((size_t)len + 1))) { bad = 1; break; }
                memcpy(gv->arr_str[t], v + o, len);
                gv->arr_str[t][len] = '\0';
                o += len;
            }
            free(v);
            if (bad) goto fail;
            have_vocab = 1;
        }
    }
    if (!have_meta || !have_vocab) goto fail;
    for (uint32_t i = 0; i < n_res; ++i) {
        const struct lstr_tensor_entry *e = &re[i];
        const char *name = e->tensor_id == LSTR_ID_TOKEN_EMBD   ? "token_embd.weight"
                           : e->tensor_id == LSTR_ID_OUTPUT_NORM ? "output_norm.weight"
                           : e->tensor_id == LSTR_ID_OUTPUT      ? "output.weight"
                                                                 : NULL;
        if (name && add_tensor(f, name, lstr_ggml_of_dtype(e->dtype), hd.resident_offset + e->offset, e->size,
                               hd.n_embd))
            goto fail;
    }
    if (add_u32(f, "llama.block_count", hd.n_layers) || add_u32(f, "llama.embedding_length", hd.n_embd) ||
        add_u32(f, "llama.attention.head_count", hd.n_heads) ||
        add_u32(f, "llama.attention.head_count_kv", hd.n_kv_heads) ||
        add_u32(f, "llama.feed_forward_length", meta.n_ff) ||
        (meta.has_bos && add_u32(f, "tokenizer.ggml.bos_token_id", meta.bos_id)))
        goto fail;
    /* layer blocks: each block's tensor table */
    char name[96];
    const uint32_t D = hd.n_embd, hdim = hd.reserved1 ? hd.reserved1 : hd.n_embd / hd.n_heads, F = meta.n_ff;
    const uint64_t row_elems[9] = {D, D, D, D, (uint64_t)hd.n_heads * hdim, D, D, D, F};
    tt = (struct lstr_tensor_entry *)malloc(9 * sizeof(*tt));
    if (!tt || !F) goto fail;
    for (uint32_t l = 0; l < hd.n_layers; ++l) {
        const struct lstr_layer_index_entry *e = &idx[l];
        if (e->layer_id != l || e->n_tensors != 9 || !e->tensor_table_offset ||
            e->tensor_table_offset + 9 * sizeof(*tt) > e->size ||
            pread_full(f->fd, tt, 9 * sizeof(*tt), e->offset + e->tensor_table_offset))
            goto fail;
        for (uint32_t t = 0; t < 9; ++t) {
            if (tt[t].tensor_id != t || tt[t].offset + tt[t].size > e->tensor_table_offset) goto fail;
            snprintf(name, sizeof(name), "blk.%u.%s", l, k_layer_suffix[t]);
            if (add_tensor(f, name, lstr_ggml_of_dtype(tt[t].dtype), e->offset + tt[t].offset, tt[t].size,
                           row_elems[t]))
                goto fail;
        }
    }
    f->version = 0;
    f->alignment = 256;
    free(idx);
    free(res);
    free(tt);
    return 0;
fail:
    free(idx);
    free(res);
    free(tt);
    gguf_close(f);
    return -1;
}

/* Verifies every layer block's checksum (LSTR_FLAG_HAS_CHECKSUMS): 0 when all
 * match or the file has none, -1 otherwise. */
int lstr_verify(const char *path) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return -1;
    struct lstr_header hd;
    int rc = pread_full(fd, &hd, sizeof(hd), 0) || hd.magic != LSTR_MAGIC ? -1 : 0;
    if (!rc && (hd.format_flags & LSTR_FLAG_HAS_CHECKSUMS)) {
        struct lstr_layer_index_entry e;
        for (uint32_t l = 0; !rc && l < hd.n_layers; ++l) {
            rc = pread_full(fd, &e, sizeof(e), hd.index_offset + (uint64_t)l * sizeof(e));
            uint8_t *b = rc ? NULL : (uint8_t *)malloc(e.size ? e.size : 1);
            if (!rc && (!b || pread_full(fd, b, e.size, e.offset) || lstr_xxh64(b, e.size, 0) != e.checksum))
                rc = -1;
            free(b);
        }
    }
    close(fd);
    return rc;
}
