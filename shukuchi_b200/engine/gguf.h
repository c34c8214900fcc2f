/* gguf.h -- GGUF (v2/v3) file index for the engine's loader.
 *
 * Parses the header, the metadata the llama loader needs and the tensor
 * table; tensor data stays in the file and is read later with pread into
 * pinned staging memory (see engine.c).  Mirrors what the reference's reader
 * exposes to its loader (engine/include/gguf_reader.h): key lookup, tensor
 * lookup by name, absolute data offsets.
 */
#ifndef SHK_GGUF_H
#define SHK_GGUF_H

#include <stddef.h>
#include <stdint.h>

enum gguf_type {
    GGUF_U8 = 0, GGUF_I8 = 1, GGUF_U16 = 2, GGUF_I16 = 3, GGUF_U32 = 4, GGUF_I32 = 5,
    GGUF_F32 = 6, GGUF_BOOL = 7, GGUF_STRING = 8, GGUF_ARRAY = 9, GGUF_U64 = 10,
    GGUF_I64 = 11, GGUF_F64 = 12
};

struct gguf_value {
    uint32_t type;      /* enum gguf_type */
    uint64_t u;         /* integer / bool value (sign-extended for signed types) */
    double f;           /* floating value */
    const char *s;      /* GGUF_STRING */
    uint32_t arr_type;  /* GGUF_ARRAY element type */
    uint64_t arr_n;     /* GGUF_ARRAY length */
    char **arr_str;     /* GGUF_ARRAY of strings (NULL otherwise) */
};

struct gguf_tensor_info {
    char *name;
    uint32_t n_dims;
    uint64_t dims[4];   /* dims[0] = elements per row */
    uint32_t type;      /* ggml type: 0 F32, 1 F16, 12 Q4_K, 13 Q5_K, 14 Q6_K */
    uint64_t offset;    /* absolute file offset of the data */
    uint64_t size;      /* bytes */
};

struct gguf_file {
    int fd;
    uint32_t version;
    uint64_t n_kv, n_tensors;
    char **keys;
    struct gguf_value *vals;
    struct gguf_tensor_info *tensors;
    uint64_t data_offset;
    uint32_t alignment;
};

/* 0 on success; the file stays open for pread. */
int gguf_open(const char *path, struct gguf_file *f);
void gguf_close(struct gguf_file *f);
const struct gguf_value *gguf_get(const struct gguf_file *f, const char *key);
/* integer metadata (any integer type); returns def when absent */
uint64_t gguf_get_uint(const struct gguf_file *f, const char *key, uint64_t def);
double gguf_get_float(const struct gguf_file *f, const char *key, double def);
const struct gguf_tensor_info *gguf_find_tensor(const struct gguf_file *f, const char *name);
/* bytes of a tensor of ggml type t with n elements (0 for unknown types) */
uint64_t gguf_type_bytes(uint32_t t, uint64_t n);

#endif
