// mmv.cuh -- batch-1 Q4_K / Q6_K dequantise-matvec on the tensor cores
// (mma.sync int8) over row-tiled weights: host-side plan API.
//
// Reference semantics: op_matmul_q4_k / op_matmul_q6_k (engine/src/ops.c:266-314,
// 361-404): y[r] = sum_k dequant(W[r, k]) * x[k].
//
// Tiled weight layout in HBM (produced from GGUF rows by mmv_tile_launch): a
// matrix of m rows and nb = k/256 super-blocks is cut into ceil(m/16) row
// tiles; row tile t, block b is one tile of 16 rows x 256 elements at
// (t * nb + b) * tile_bytes, so a row tile's K range is contiguous.  Rows past
// m are zero.  Inside a tile the bytes of each lane's mma fragments are
// contiguous (see mmv_dev.cuh), the quants and scales are the GGUF bytes
// unchanged, only moved.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "gemv.cuh"

namespace shk {

constexpr int T_Q4K_TILED = 0x20C;
constexpr int T_Q6K_TILED = 0x20E;
constexpr uint32_t Q4T_BYTES = 16 * 144;  // 2304
constexpr uint32_t Q6T_BYTES = 16 * 210;  // 3360

constexpr int MMV_MAX_SEGS = 4;
constexpr int MMV_WARPS = 15;                   // consumer warps; one more issues the copies
constexpr int MMV_THREADS = 32 * (MMV_WARPS + 1);
constexpr int MMV_MAX_STAGES = 32;
constexpr int MMV_MAX_GRID = 160;               // CTA item table entries (>= SM count + 1)
constexpr int MMV_MAX_KS = 128;                 // K slices per row tile
constexpr int MMV_MAX_CHUNK = 8;                // items per ring stage

// Bytes of a tiled matrix.
inline size_t mmv_tiled_bytes(uint32_t qt, uint32_t m, uint32_t k) {
  const size_t tb = (qt == T_Q4K_TILED || qt == T_Q4K) ? Q4T_BYTES : Q6T_BYTES;
  return (size_t)((m + 15) / 16) * (k / 256) * tb;
}

struct MmvSeg {
  const uint8_t* w;   // tiled matrix
  const uint8_t* w2;  // dual (gate/up): the up matrix, same shape
  float* y;           // output rows
  uint32_t m;         // valid rows
  uint32_t nb;        // blocks per row
  uint32_t ntiles;    // ceil(m / 16)
  uint32_t items;     // ntiles * ks
  uint32_t item0;     // global index of this segment's first item
  uint32_t rope_hd;   // EPI_ROPE head size
  uint16_t sw;        // blocks per K slice (the last slice may be shorter)
  uint8_t ks;         // K slices per row tile
  uint8_t qt;         // T_Q4K or T_Q6K (tiled)
  uint8_t epi;        // GemvEpi
  uint8_t dual;       // 1: gate/up pair, SwiGLU epilogue
};

struct MmvArgs {
  MmvSeg seg[MMV_MAX_SEGS];
  uint32_t nseg;
  uint32_t k;
  const float* x;
  const float* norm_w;      // optional RMSNorm weights (eps 1e-5), applied as an output scale
  const uint32_t* pos;      // EPI_ROPE position (device)
  const float* rope_freq;   // EPI_ROPE: freq[i/2] = powf(1/theta, i/head_dim)
  uint32_t stage_bytes;     // bytes of one item slot (>= the largest item)
  uint32_t n_stages;        // ring stages, one chunk of `chunk` item slots each
  uint32_t chunk, lg_chunk; // items per chunk (a power of two) and its log2
  uint32_t pre_items;       // items issued before the consumers have converted x
  uint32_t has4, has6;      // quant types present (x region parts)
  uint32_t red_slots;       // K-slice partial slots in shared memory
  uint32_t red_stride;      // floats per slot: 16, or 32 for a dual (gate/up) plan
  uint32_t grid;            // CTAs with items; CTAs >= grid take none (persistent launches)
  uint32_t cta_item[MMV_MAX_GRID + 1];  // CTA c takes global items [cta_item[c], cta_item[c+1])
  // A row tile whose K slices straddle the boundary b between CTAs b-1 and b
  // (at most two CTAs share one) is combined through global memory: the two
  // CTAs' partial sums go to xpart[b][0 lower | 1 upper][32] and the second
  // to count xcnt[b] adds them (lower + upper) and stores.  xcnt is zero
  // between launches (the second arriver resets it).
  float* xpart;             // [MMV_MAX_GRID + 1][2][32]
  int* xcnt;                // [MMV_MAX_GRID + 1]
  int* err;
};

struct MmvPlan {
  MmvArgs args;
  int grid = 0;
  size_t smem = 0;
};

struct MmvMat {
  const void* w;   // tiled
  const void* w2;  // non-null: dual (gate/up)
  float* y;
  uint32_t m;
  uint32_t qt;     // T_Q4K_TILED or T_Q6K_TILED
  uint8_t epi;
  uint32_t rope_hd;
};

// Bytes of the cross-CTA combine scratch (MmvArgs::xpart, then xcnt), zeroed once.
constexpr size_t MMV_SCRATCH_BYTES = (size_t)(MMV_MAX_GRID + 1) * (2 * 32 * 4 + 4);

// Returns 0 or a negative code (-1 bad argument, -2 unsupported, -4 does not fit).
// scratch: MMV_SCRATCH_BYTES of zeroed device memory shared by the launches of
// one stream (launches that overlap on the GPU must not share it).
// max_item_bytes (0 = none): items no larger than this where a slice of one
// block allows it (a persistent launch shares one ring among its plans).
int mmv_plan(MmvPlan& p, const MmvMat* mats, int nmats, uint32_t k, const float* x, const float* norm_w,
             const uint32_t* pos, const float* rope_freq, int* err, int num_sms, void* scratch,
             uint32_t max_item_bytes = 0);
cudaError_t mmv_init();
cudaError_t mmv_launch(const MmvPlan& p, cudaStream_t stream);

// GGUF rows (qt = T_Q4K or T_Q6K, src_stride bytes apart, 0 = dense) -> tiled
// layout at dst (mmv_tiled_bytes(qt, m, k) bytes, 16-byte aligned).
cudaError_t mmv_tile_launch(uint32_t qt, const void* src, uint32_t src_stride, uint32_t m, uint32_t k,
                            void* dst, cudaStream_t stream);

}  // namespace shk
