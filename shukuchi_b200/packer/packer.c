/* packer.c -- GGUF -> LSTR container (format in engine/lstr.h).
 *
 * The reference declares this step (model_packer/src/packer.c:1-9, a stub
 * returning 0) and the container (include/lstr_format.h).  Here the packer
 * reads a llama GGUF file and writes: the 256-byte header, the layer index,
 * the resident section (vocabulary, metadata, token embedding, output norm,
 * output head) and one block per layer -- its nine tensors at 256-byte
 * offsets, then its tensor table -- each block starting on the configured
 * alignment, with an XXH64 of the block in the index when asked.
 */
#ifndef _GNU_SOURCE
#define _GNU_SOURCE
#endif
#include "packer.h"

#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "../engine/gguf.h"
#include "../engine/lstr.h"

static const char *const k_sfx[9] = {"attn_norm.weight", "attn_q.weight",   "attn_k.weight",
                                     "attn_v.weight",    "attn_output.weight", "ffn_norm.weight",
                                     "ffn_gate.weight",  "ffn_up.weight",   "ffn_down.weight"};

static uint64_t al(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

static int rd(int fd, void *dst, uint64_t len, uint64_t off) {
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

static int wr(int fd, const void *src, uint64_t len, uint64_t off) {
    const uint8_t *s = (const uint8_t *)src;
    while (len) {
        const ssize_t n = pwrite(fd, s, len > (1u << 30) ? (1u << 30) : len, (off_t)off);
        if (n < 0 && errno == EINTR) continue;
        if (n <= 0) return -1;
        s += n;
        off += (uint64_t)n;
        len -= (uint64_t)n;
    }
    return 0;
}

/* Copies a tensor's bytes from the GGUF file to `off` in the output. */
static int copy_tensor(int in, int out, const struct gguf_tensor_info *ti, uint64_t off, uint8_t *buf, uint64_t cap) {
    for (uint64_t done = 0; done < ti->size;) {
        const uint64_t n = ti->size - done < cap ? ti->size - done : cap;
        if (rd(in, buf, n, ti->offset + done) || wr(out, buf, n, off + done)) return -1;
        done += n;
    }
    return 0;
}

int packer_run(const char *input_path, const char *output_path, const struct packer_config *cfg) {
    if (!input_path || !output_path) return -1;
    const uint64_t align = cfg && cfg->alignment ? cfg->alignment : 4096;
    if (align < 256 || (align & (align - 1))) return -1;
    const int sums = cfg && cfg->write_checksums;
    struct gguf_file g;
    if (gguf_open(input_path, &g)) return -1;
    int rc = -1, out = -1;
    uint8_t *buf = NULL, *blk = NULL;
    struct lstr_layer_index_entry *idx = NULL;
    const uint32_t L = (uint32_t)gguf_get_uint(&g, "llama.block_count", 0);
    const uint32_t D = (uint32_t)gguf_get_uint(&g, "llama.embedding_length", 0);
    const uint32_t H = (uint32_t)gguf_get_uint(&g, "llama.attention.head_count", 0);
    const uint32_t KV = (uint32_t)gguf_get_uint(&g, "llama.attention.head_count_kv", H);
    const struct gguf_value *tok = gguf_get(&g, "tokenizer.ggml.tokens");
    const struct gguf_value *bos = gguf_get(&g, "tokenizer.ggml.bos_token_id");
    const struct gguf_tensor_info *emb = gguf_find_tensor(&g, "token_embd.weight");
    const struct gguf_tensor_info *onorm = gguf_find_tensor(&g, "output_norm.weight");
    const struct gguf_tensor_info *outw = gguf_find_tensor(&g, "output.weight");
    if (!L || !D || !H || !emb || !onorm || !outw || !tok || tok->type != GGUF_ARRAY ||
        tok->arr_type != GGUF_STRING || outw->n_dims != 2)
        goto done;
    const struct gguf_tensor_info *t[9];
    char name[96];
    uint64_t max_block = 0;
    idx = (struct lstr_layer_index_entry *)calloc(L, sizeof(*idx));
    if (!idx) goto done;
    for (uint32_t l = 0; l < L; ++l) {
        uint64_t o = 0;
        for (int i = 0; i < 9; ++i) {
            snprintf(name, sizeof(name), "blk.%u.%s", l, k_sfx[i]);
            if (!(t[i] = gguf_find_tensor(&g, name)) || !lstr_dtype_of_ggml(t[i]->type)) goto done;
            o = al(o, 256) + t[i]->size;
        }
        const uint64_t sz = al(o, 8) + 9 * sizeof(struct lstr_tensor_entry);
        if (sz > max_block) max_block = sz;
    }
    const struct gguf_tensor_info *gate0 = gguf_find_tensor(&g, "blk.0.ffn_gate.weight");
    /* resident records: vocabulary, metadata, token_embd, output_norm, output */
    uint64_t vocab_bytes = 4;
    for (uint64_t i = 0; i < tok->arr_n; ++i) vocab_bytes += 4 + strlen(tok->arr_str[i]);
    struct lstr_meta meta;
    memset(&meta, 0, sizeof(meta));
    meta.n_ff = gate0 && gate0->n_dims == 2 ? (uint32_t)gate0->dims[1] : 0;
    meta.has_bos = bos && bos->type == GGUF_U32;
    meta.bos_id = meta.has_bos ? (uint32_t)bos->u : 0;
    meta.token_embd_rows = emb->n_dims == 2 ? (uint32_t)emb->dims[1] : 1;
    meta.output_rows = (uint32_t)outw->dims[1];
    if (!meta.n_ff) goto done;
    struct lstr_tensor_entry re[5];
    const uint64_t res_off = al(LSTR_HEADER_SIZE + (uint64_t)L * sizeof(*idx), 256);
    uint64_t o = al(8 + sizeof(re), 256);
    const uint32_t ids[5] = {LSTR_ID_VOCAB, LSTR_ID_META, LSTR_ID_TOKEN_EMBD, LSTR_ID_OUTPUT_NORM, LSTR_ID_OUTPUT};
    const uint64_t sizes[5] = {vocab_bytes, sizeof(meta), emb->size, onorm->size, outw->size};
    const uint32_t dts[5] = {LSTR_DTYPE_BYTES, LSTR_DTYPE_BYTES, lstr_dtype_of_ggml(emb->type),
                             lstr_dtype_of_ggml(onorm->type), lstr_dtype_of_ggml(outw->type)};
    for (int i = 0; i < 5; ++i) {
        if (!dts[i]) goto done;
        re[i] = (struct lstr_tensor_entry){ids[i], dts[i], o, sizes[i]};
        o = al(o + sizes[i], 256);
    }
    const uint64_t res_size = o;
    out = open(output_path, O_CREAT | O_TRUNC | O_WRONLY, 0644);
    const uint64_t cap = 64ull << 20;
    buf = (uint8_t *)malloc(cap);
    blk = (uint8_t *)malloc(max_block ? max_block : 1);
    if (out < 0 || !buf || !blk) goto done;
    /* resident section */
    {
        uint32_t hdr2[2] = {5, 0};
        if (wr(out, hdr2, 8, res_off) || wr(out, re, sizeof(re), res_off + 8)) goto done;
        uint8_t *v = (uint8_t *)malloc(vocab_bytes);
        if (!v) goto done;
        uint32_t n = (uint32_t)tok->arr_n;
        memcpy(v, &n, 4);
        uint64_t p = 4;
        for (uint64_t i = 0; i < tok->arr_n; ++i) {
            const uint32_t len = (uint32_t)strlen(tok->arr_str[i]);
            memcpy(v + p, &len, 4);
            memcpy(v + p + 4, tok->arr_str[i], len);
            p += 4 + len;
        }
        const int e = wr(out, v, vocab_bytes, res_off + re[0].offset);
        free(v);
        if (e || wr(out, &meta, sizeof(meta), res_off + re[1].offset) ||
            copy_tensor(g.fd, out, emb, res_off + re[2].offset, buf, cap) ||
            copy_tensor(g.fd, out, onorm, res_off + re[3].offset, buf, cap) ||
            copy_tensor(g.fd, out, outw, res_off + re[4].offset, buf, cap))
            goto done;
    }
    /* layer blocks */
    uint64_t pos = al(res_off + res_size, align);
    const uint64_t layers_off = pos;
    for (uint32_t l = 0; l < L; ++l) {
        struct lstr_tensor_entry te[9];
        uint64_t bo = 0;
        memset(blk, 0, max_block);
        for (int i = 0; i < 9; ++i) {
            snprintf(name, sizeof(name), "blk.%u.%s", l, k_sfx[i]);
            t[i] = gguf_find_tensor(&g, name);
            bo = al(bo, 256);
            if (rd(g.fd, blk + bo, t[i]->size, t[i]->offset)) goto done;
            te[i] = (struct lstr_tensor_entry){(uint32_t)i, lstr_dtype_of_ggml(t[i]->type), bo, t[i]->size};
            bo += t[i]->size;
        }
        const uint64_t tt_off = al(bo, 8), size = tt_off + sizeof(te);
        memcpy(blk + tt_off, te, sizeof(te));
        idx[l] = (struct lstr_layer_index_entry){l, 9, pos, size, lstr_dtype_of_ggml(t[1]->type), (uint32_t)tt_off,
                                                 sums ? lstr_xxh64(blk, size, 0) : 0};
        if (wr(out, blk, size, pos)) goto done;
        pos = al(pos + size, align);
    }
    const uint64_t file_size = pos;
    if (ftruncate(out, (off_t)file_size)) goto done;
    if (wr(out, idx, (uint64_t)L * sizeof(*idx), LSTR_HEADER_SIZE)) goto done;
    struct lstr_header hd;
    memset(&hd, 0, sizeof(hd));
    hd.magic = LSTR_MAGIC;
    hd.endian_tag = LSTR_ENDIAN_TAG;
    hd.version = LSTR_VERSION;
    hd.header_size = LSTR_HEADER_SIZE;
    hd.min_loader_version = 1;
    hd.format_flags = LSTR_FLAG_HAS_TENSOR_TABLE | (sums ? LSTR_FLAG_HAS_CHECKSUMS : 0) |
                      (align == 4096 ? LSTR_FLAG_LAYER_ALIGN_4K : 0) |
                      (align == (2u << 20) ? LSTR_FLAG_LAYER_ALIGN_2M : 0);
    hd.n_layers = L;
    hd.n_vocab = (uint32_t)tok->arr_n;
    hd.n_embd = D;
    hd.n_heads = H;
    hd.n_kv_heads = KV;
    hd.ctx_size = (uint32_t)gguf_get_uint(&g, "llama.context_length", 0);
    hd.rope_type = 1;
    hd.rope_theta = (float)gguf_get_float(&g, "llama.rope.freq_base", 10000.0);
    hd.reserved0 = meta.n_ff;
    hd.reserved1 = D / H;
    hd.index_offset = LSTR_HEADER_SIZE;
    hd.index_size = (uint64_t)L * sizeof(*idx);
    hd.resident_offset = res_off;
    hd.resident_size = res_size;
    hd.layers_offset = layers_off;
    hd.file_size = file_size;
    const struct gguf_value *nm = gguf_get(&g, "general.name");
    snprintf(hd.model_name, sizeof(hd.model_name), "%s", nm && nm->type == GGUF_STRING && nm->s ? nm->s : "");
    snprintf(hd.build_tag, sizeof(hd.build_tag), "shukuchi-b200 packer");
    if (wr(out, &hd, sizeof(hd), 0)) goto done;
    rc = 0;
done:
    if (out >= 0 && close(out) && !rc) rc = -1;
    free(buf);
    free(blk);
    free(idx);
    gguf_close(&g);
    return rc;
}
