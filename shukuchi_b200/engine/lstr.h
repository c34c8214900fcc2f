/* lstr.h -- the LSTR layer-streaming container (little-endian).
 *
 * The reference defines the format (include/lstr_format.h:1-79) -- a 256-byte
 * header, a layer index, a resident section and aligned layer blocks with
 * per-layer tensor tables -- but writes and reads none of it (its packer,
 * model_packer/src/packer.c, is an empty stub).  The structs below keep the
 * reference's field order and sizes, so a file is the reference's format; the
 * additions are spelled out here:
 *   - dtypes: the reference's F16 / F32 / Q8_0 / Q4_0 ids plus the K-quants
 *     under their ggml ids (Q4_K 12, Q5_K 13, Q6_K 14);
 *   - layer blocks: the nine tensors of a layer first, each at a 256-byte
 *     offset from the block base, tensor_id = its slot (attn_norm, attn_q,
 *     attn_k, attn_v, attn_output, ffn_norm, ffn_gate, ffn_up, ffn_down =
 *     0..8), then the block's tensor table (tensor_table_offset); blocks start
 *     on the container's alignment (4 KiB or 2 MiB flags) so one pread -- or an
 *     O_DIRECT read -- stages a layer;
 *   - resident section: a u32 entry count, a u32 zero, then lstr_tensor_entry
 *     records whose offsets are from the section start: the token embedding
 *     (tensor_id LSTR_ID_TOKEN_EMBD), output_norm, output, the vocabulary
 *     (LSTR_ID_VOCAB: u32 count, then per token a u32 length and the bytes)
 *     and a metadata record (LSTR_ID_META: struct lstr_meta);
 *   - header.reserved0 = n_ff, header.reserved1 = head_dim.
 * The reference's padding expression counts 11 four-byte fields where its
 * struct has 17 (its size assertion cannot hold as written); here the fields
 * keep their order, a reserved2 word aligns the 64-bit offsets and the
 * padding makes the header exactly 256 bytes.
 * Checksums (LSTR_FLAG_HAS_CHECKSUMS) are XXH64, seed 0, of each layer block
 * (its tensors and table, up to `size`).
 */
#ifndef SHK_LSTR_H
#define SHK_LSTR_H

#include <stdint.h>

#define LSTR_MAGIC 0x5254534cU /* "LSTR" */
#define LSTR_VERSION 1
#define LSTR_HEADER_SIZE 256
#define LSTR_ENDIAN_TAG 0x01020304U

enum lstr_format_flags {
    LSTR_FLAG_HAS_CHECKSUMS = 1u << 0,
    LSTR_FLAG_HAS_TENSOR_TABLE = 1u << 1,
    LSTR_FLAG_LAYER_ALIGN_4K = 1u << 2,
    LSTR_FLAG_LAYER_ALIGN_2M = 1u << 3,
};

enum lstr_dtype {
    LSTR_DTYPE_F16 = 1,
    LSTR_DTYPE_F32 = 2,
    LSTR_DTYPE_Q8_0 = 10,
    LSTR_DTYPE_Q4_0 = 11,
    LSTR_DTYPE_Q4_K = 12,
    LSTR_DTYPE_Q5_K = 13,
    LSTR_DTYPE_Q6_K = 14,
    LSTR_DTYPE_BYTES = 0xFF, /* resident records that are not tensors */
};

struct lstr_header {
    uint32_t magic, endian_tag, version, header_size, min_loader_version;
    uint32_t format_flags, n_layers, n_vocab, n_embd;
    uint32_t n_heads, n_kv_heads, ctx_size, rope_type;
    float rope_theta, rope_scale;
    uint32_t reserved0, reserved1;
    uint32_t reserved2; /* explicit: the 64-bit offsets start 8-byte aligned */
    uint64_t index_offset, index_size, resident_offset, resident_size;
    uint64_t layers_offset, file_size;
    char model_name[64];
    char build_tag[64];
    uint8_t padding[LSTR_HEADER_SIZE - 4 * 18 - 8 * 6 - 64 - 64];
};
_Static_assert(sizeof(struct lstr_header) == LSTR_HEADER_SIZE, "lstr_header size");

struct lstr_layer_index_entry {
    uint32_t layer_id, n_tensors;
    uint64_t offset, size;
    uint32_t dtype, tensor_table_offset;
    uint64_t checksum;
};
_Static_assert(sizeof(struct lstr_layer_index_entry) == 40, "lstr_layer_index_entry size");

struct lstr_tensor_entry {
    uint32_t tensor_id, dtype;
    uint64_t offset, size;
};
_Static_assert(sizeof(struct lstr_tensor_entry) == 24, "lstr_tensor_entry size");

enum { LSTR_ID_TOKEN_EMBD = 100, LSTR_ID_OUTPUT_NORM = 101, LSTR_ID_OUTPUT = 102,
       LSTR_ID_VOCAB = 200, LSTR_ID_META = 201 };

struct lstr_meta {       /* the LSTR_ID_META record */
    uint32_t n_ff;
    uint32_t has_bos, bos_id;
    uint32_t token_embd_rows, output_rows;
    uint32_t reserved[11];
};

struct gguf_file;
/* 1 when the file starts with the LSTR magic. */
int lstr_is(const char *path);
/* Opens a container as the loader's file index (the same struct the GGUF
 * reader fills: metadata keys, vocabulary, named tensors at absolute file
 * offsets); 0 on success. */
int lstr_open(const char *path, struct gguf_file *f);
/* 0 when every layer block matches its index checksum (or there are none). */
int lstr_verify(const char *path);
uint64_t lstr_xxh64(const void *data, uint64_t len, uint64_t seed);
/* ggml type -> lstr dtype and back (0 / LSTR_DTYPE_BYTES when unknown). */
uint32_t lstr_dtype_of_ggml(uint32_t ggml_type);
uint32_t lstr_ggml_of_dtype(uint32_t dtype);

#endif
