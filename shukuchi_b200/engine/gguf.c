/* gguf.c -- GGUF index: header, metadata, tensor table (see gguf.h). */
#include "gguf.h"

#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* Buffered sequential reader over the file's header region. */
struct rd {
    int fd;
    uint8_t buf[1 << 16];
    size_t len, pos;
    uint64_t file_pos; /* file offset of buf[0] */
    int err;
};

static int rd_fill(struct rd *r) {
    if (r->pos < r->len) return 0;
    r->file_pos += r->len;
    ssize_t n = pread(r->fd, r->buf, sizeof(r->buf), (off_t)r->file_pos);
    if (n <= 0) {
        r->err = 1;
        return -1;
    }
    r->len = (size_t)n;
    r->pos = 0;
    return 0;
}

static int rd_bytes(struct rd *r, void *dst, size_t n) {
    uint8_t *d = (uint8_t *)dst;
    while (n) {
        if (rd_fill(r)) return -1;
        size_t k = r->len - r->pos;
        if (k > n) k = n;
        memcpy(d, r->buf + r->pos, k);
        r->pos += k;
        d += k;
        n -= k;
    }
    return 0;
}

static uint64_t rd_u64(struct rd *r) { uint64_t v = 0; rd_bytes(r, &v, 8); return v; }
static uint32_t rd_u32(struct rd *r) { uint32_t v = 0; rd_bytes(r, &v, 4); return v; }

static char *rd_str(struct rd *r) {
    uint64_t n = rd_u64(r);
    if (r->err || n > (1u << 30)) {
        r->err = 1;
        return NULL;
    }
    char *s = (char *)malloc(n + 1);
    if (!s) {
        r->err = 1;
        return NULL;
    }
    if (rd_bytes(r, s, n)) {
        free(s);
        return NULL;
    }
    s[n] = '\0';
    return s;
}

static size_t scalar_size(uint32_t t) {
    switch (t) {
        case GGUF_U8: case GGUF_I8: case GGUF_BOOL: return 1;
        case GGUF_U16: case GGUF_I16: return 2;
        case GGUF_U32: case GGUF_I32: case GGUF_F32: return 4;
        case GGUF_U64: case GGUF_I64: case GGUF_F64: return 8;
        default: return 0;
    }
}

static void scalar_decode(uint32_t t, const uint8_t *p, struct gguf_value *v) {
    v->type = t;
    switch (t) {
        case GGUF_U8: case GGUF_BOOL: v->u = p[0]; break;
        case GGUF_I8: v->u = (uint64_t)(int64_t)(int8_t)p[0]; break;
        case GGUF_U16: { uint16_t x; memcpy(&x, p, 2); v->u = x; break; }
        case GGUF_I16: { int16_t x; memcpy(&x, p, 2); v->u = (uint64_t)(int64_t)x; break; }
        case GGUF_U32: { uint32_t x; memcpy(&x, p, 4); v->u = x; break; }
        case GGUF_I32: { int32_t x; memcpy(&x, p, 4); v->u = (uint64_t)(int64_t)x; break; }
        case GGUF_F32: { float x; memcpy(&x, p, 4); v->f = x; break; }
        case GGUF_U64: case GGUF_I64: memcpy(&v->u, p, 8); break;
        case GGUF_F64: memcpy(&v->f, p, 8); break;
        default: break;
    }
    if (t != GGUF_F32 && t != GGUF_F64) v->f = (double)(int64_t)v->u;
}

static int rd_value(struct rd *r, uint32_t t, struct gguf_value *v) {
    memset(v, 0, sizeof(*v));
    v->type = t;
    if (t == GGUF_STRING) {
        v->s = rd_str(r);
        return v->s ? 0 : -1;
    }
    if (t == GGUF_ARRAY) {
        v->arr_type = rd_u32(r);
        v->arr_n = rd_u64(r);
        if (r->err) return -1;
        if (v->arr_type == GGUF_STRING) {
            if (v->arr_n > (1u << 26)) return -1;
            v->arr_str = (char **)calloc(v->arr_n ? v->arr_n : 1, sizeof(char *));
            if (!v->arr_str) return -1;
            for (uint64_t i = 0; i < v->arr_n; ++i)
                if (!(v->arr_str[i] = rd_str(r))) return -1;
            return 0;
        }
        const size_t es = scalar_size(v->arr_type);
        if (!es) return -1;
        uint8_t tmp[8];
        for (uint64_t i = 0; i < v->arr_n; ++i)  /* numeric arrays are skipped */
            if (rd_bytes(r, tmp, es)) return -1;
        return 0;
    }
    const size_t es = scalar_size(t);
    uint8_t tmp[8];
    if (!es || rd_bytes(r, tmp, es)) return -1;
    scalar_decode(t, tmp, v);
    return 0;
}

uint64_t gguf_type_bytes(uint32_t t, uint64_t n) {
    switch (t) {
        case 0: return 4 * n;                      /* F32 */
        case 1: return 2 * n;                      /* F16 */
        case 12: return n % 256 ? 0 : n / 256 * 144; /* Q4_K */
        case 13: return n % 256 ? 0 : n / 256 * 176; /* Q5_K */
        case 14: return n % 256 ? 0 : n / 256 * 210; /* Q6_K */
        default: return 0;
    }
}

void gguf_close(struct gguf_file *f) {
    if (!f) return;
    for (uint64_t i = 0; f->keys && i < f->n_kv; ++i) {
        free(f->keys[i]);
        struct gguf_value *v = &f->vals[i];
        free((char *)v->s);
        if (v->arr_str) {
            for (uint64_t j = 0; j < v->arr_n; ++j) free(v->arr_str[j]);
            free(v->arr_str);
        }
    }
    free(f->keys);
    free(f->vals);
    for (uint64_t i = 0; f->tensors && i < f->n_tensors; ++i) free(f->tensors[i].name);
    free(f->tensors);
    if (f->fd >= 0) close(f->fd);
    memset(f, 0, sizeof(*f));
    f->fd = -1;
}

int gguf_open(const char *path, struct gguf_file *f) {
    memset(f, 0, sizeof(*f));
    f->fd = open(path, O_RDONLY);
    if (f->fd < 0) return -1;
    struct rd *r = (struct rd *)calloc(1, sizeof(struct rd));
    if (!r) goto fail;
    r->fd = f->fd;
    char magic[4];
    if (rd_bytes(r, magic, 4) || memcmp(magic, "GGUF", 4) != 0) goto fail;
    f->version = rd_u32(r);
    if (f->version < 2 || f->version > 3) goto fail;
    f->n_tensors = rd_u64(r);
    f->n_kv = rd_u64(r);
    if (r->err || f->n_tensors > (1u << 20) || f->n_kv > (1u << 20)) goto fail;
    f->keys = (char **)calloc(f->n_kv ? f->n_kv : 1, sizeof(char *));
    f->vals = (struct gguf_value *)calloc(f->n_kv ? f->n_kv : 1, sizeof(struct gguf_value));
    f->tensors = (struct gguf_tensor_info *)calloc(f->n_tensors ? f->n_tensors : 1,
                                                   sizeof(struct gguf_tensor_info));
    if (!f->keys || !f->vals || !f->tensors) goto fail;
    for (uint64_t i = 0; i < f->n_kv; ++i) {
        if (!(f->keys[i] = rd_str(r))) goto fail;
        const uint32_t t = rd_u32(r);
        if (r->err || rd_value(r, t, &f->vals[i])) goto fail;
    }
    f->alignment = (uint32_t)gguf_get_uint(f, "general.alignment", 32);
    if (f->alignment == 0 || (f->alignment & (f->alignment - 1))) goto fail;
    for (uint64_t i = 0; i < f->n_tensors; ++i) {
        struct gguf_tensor_info *ti = &f->tensors[i];
        if (!(ti->name = rd_str(r))) goto fail;
        ti->n_dims = rd_u32(r);
        if (ti->n_dims == 0 || ti->n_dims > 4) goto fail;
        uint64_t n = 1;
        for (uint32_t d = 0; d < ti->n_dims; ++d) n *= (ti->dims[d] = rd_u64(r));
        ti->type = rd_u32(r);
        ti->offset = rd_u64(r);
        if (r->err) goto fail;
        ti->size = gguf_type_bytes(ti->type, n);
    }
    const uint64_t hdr_end = r->file_pos + r->pos;
    f->data_offset = (hdr_end + f->alignment - 1) / f->alignment * f->alignment;
    for (uint64_t i = 0; i < f->n_tensors; ++i) f->tensors[i].offset += f->data_offset;
    free(r);
    return 0;
fail:
    free(r);
    gguf_close(f);
    return -1;
}

const struct gguf_value *gguf_get(const struct gguf_file *f, const char *key) {
    for (uint64_t i = 0; i < f->n_kv; ++i)
        if (strcmp(f->keys[i], key) == 0) return &f->vals[i];
    return NULL;
}

uint64_t gguf_get_uint(const struct gguf_file *f, const char *key, uint64_t def) {
    const struct gguf_value *v = gguf_get(f, key);
    if (!v || v->type == GGUF_STRING || v->type == GGUF_ARRAY || v->type == GGUF_F32 ||
        v->type == GGUF_F64)
        return def;
    return v->u;
}

double gguf_get_float(const struct gguf_file *f, const char *key, double def) {
    const struct gguf_value *v = gguf_get(f, key);
    if (!v || v->type == GGUF_STRING || v->type == GGUF_ARRAY) return def;
    return v->f;
}

const struct gguf_tensor_info *gguf_find_tensor(const struct gguf_file *f, const char *name) {
    for (uint64_t i = 0; i < f->n_tensors; ++i)
        if (strcmp(f->tensors[i].name, name) == 0) return &f->tensors[i];
    return NULL;
}
