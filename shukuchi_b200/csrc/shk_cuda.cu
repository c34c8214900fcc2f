// shk_cuda.cu -- C ABI (include/shk_cuda.h) over the sm_100a decode kernels.
#include "../../include/shk_cuda.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "attn.cuh"
#include "common.cuh"
#include "decode.cuh"
#include "gemv.cuh"
#include "glue.cuh"
#include "mmv.cuh"
#include "q5k.cuh"
#include "prefill_layer.cuh"
#include "tp_ll.cuh"

using // Fewest cached positions per attention split (CTA of a KV head's cluster).
#ifndef SHK_ATT_MIN_SPLIT
#define SHK_ATT_MIN_SPLIT 32
#endif

namespace shk;

#define CK(expr)                                              \
  do {                                                        \
    cudaError_t e_ = (expr);                                  \
    if (e_ != cudaSuccess) {                                  \
      fprintf(stderr, "shk_cuda: %s: %s\n", #expr, cudaGetErrorString(e_)); \
      return SHK_ECUDA;                                       \
    }                                                         \
  } while (0)

// NCCL, loaded at first use: the process's libnccl.so.2 (the one a framework
// already loaded, else the system's), so no second copy is linked in.
namespace {
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*comm_count)(const ncclComm_t, int*);
};
const NcclApi* nccl() {
  static NcclApi api;
  static int state = 0;  // 0 untried, 1 loaded, -1 unavailable
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (state == 0) {
    state = -1;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
      api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
      api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
      api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
      api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
      api.comm_count = reinterpret_cast<decltype(api.comm_count)>(dlsym(h, "ncclCommCount"));
      if (api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather && api.comm_destroy &&
          api.comm_count)
        state = 1;
    }
  }
  return state == 1 ? &api : nullptr;
}
}  // namespace

struct shk_ctx {
  int device = 0;
  int tp_rank = 0, tp_world = 1;  // tensor parallelism (shk_cuda_tp_init)
  ncclComm_t comm = nullptr;
  uint32_t flags = 0;  // SHK_CUDA_FLAG_*
  int num_sms = 148;
  cudaStream_t compute = nullptr;
  cudaStream_t copy = nullptr;
  int* d_err = nullptr;
  int* h_err = nullptr;  // pinned
  // op-level scratch
  uint32_t* d_u32 = nullptr;   // [0] pos for op rope, [1] token for op embed, [2] argmax result
  uint32_t* h_u32 = nullptr;   // pinned mirror
  float* am_v = nullptr;
  uint32_t* am_i = nullptr;
  int* am_cnt = nullptr;
  float* d_freq = nullptr;  // RoPE frequency table for shk_cuda_rope (<= 512 entries)
  void* mmv_scratch = nullptr;  // tensor-core matvec: cross-CTA combine of split row tiles
  float* h_freq = nullptr;  // pinned
  // synchronous host-pointer matvec scratch
  void* hv_w = nullptr;
  size_t hv_w_cap = 0;
  void* q6_scratch = nullptr;  // GGUF-layout Q6_K rows repacked for the staged GEMV
  size_t q6_scratch_cap = 0;
  void* pf_x = nullptr;  // f16 copy of the prefill activations + per-token scales
  size_t pf_x_cap = 0;
  float* hv_x = nullptr;
  size_t hv_x_cap = 0;
  float* hv_y = nullptr;
  size_t hv_y_cap = 0;
  // staging
  std::mutex stage_mu;
  std::unordered_map<uint32_t, cudaEvent_t> slot_ev;
  std::unordered_map<uint32_t, cudaEvent_t> rel_ev;    // shk_cuda_layer_release
  std::unordered_map<uint32_t, bool> rel_pending;
  // counters (shk_cuda_report)
  uint64_t n_matvec = 0, n_matvec_host = 0, n_fwd = 0, n_steps = 0, n_staged = 0, bytes_staged = 0;
};

struct shk_kv {
  shk_ctx* ctx = nullptr;
  KvLayout L{};
  std::vector<uint32_t> seq;
  float* part = nullptr;
  int* counters = nullptr;
  uint32_t max_splits = 1;
  uint32_t* d_iota = nullptr;  // d_iota[p] == p, used as a device position pointer
  // partials and ticket counters of batched attention (shk_cuda_kv_attend_batch)
  float* part_batch = nullptr;
  int* counters_batch = nullptr;
  uint32_t batch_cap = 0;  // sequences they are sized for
};

namespace {

// One projection: the staged dp4a GEMV over GGUF / planar rows, or the
// tensor-core matvec over row-tiled weights (tiled = true); its Q5_K matrices
// (if any) run on the Q5_K matvec, a second launch after the first when the
// projection mixes Q5_K with other types (main = false: Q5_K only).
struct ProjPlan {
  GemvPlan g;
  MmvPlan mm;
  Q5Plan q5;
  bool tiled = false;
  bool main = true;
  bool has_q5 = false;
};

cudaError_t proj_launch(const ProjPlan& p, cudaStream_t st, const uint32_t* pos = nullptr) {
  cudaError_t e = cudaSuccess;
  if (!p.main) {
  } else if (p.tiled) {
    if (!pos) {
      e = mmv_launch(p.mm, st);
    } else {
      MmvPlan q = p.mm;
      q.args.pos = pos;
      e = mmv_launch(q, st);
    }
  } else if (!pos) {
    e = gemv_launch(p.g, st);
  } else {
    GemvPlan q = p.g;
    q.args.pos = pos;
    e = gemv_launch(q, st);
  }
  if (e != cudaSuccess || !p.has_q5) return e;
  if (!pos) return q5k_launch(p.q5, st);
  Q5Plan q = p.q5;
  q.args.pos = pos;
  return q5k_launch(q, st);
}

// Launches of one projection.
int proj_launches(const ProjPlan& p) { return (p.main ? 1 : 0) + (p.has_q5 ? 1 : 0); }

// Weight bytes one launch reads.
uint64_t proj_weight_bytes(const ProjPlan& p) {
  uint64_t b = 0;
  if (p.has_q5)
    for (uint32_t i = 0; i < p.q5.args.nseg; ++i) {
      const Q5Seg& g = p.q5.args.seg[i];
      b += (uint64_t)g.m * (p.q5.args.k / QK) * Q5K_BYTES * (g.w2 ? 2 : 1);
    }
  if (!p.main) return b;
  if (p.tiled) {
    for (uint32_t i = 0; i < p.mm.args.nseg; ++i) {
      const MmvSeg& g = p.mm.args.seg[i];
      b += (uint64_t)g.ntiles * g.nb * (g.qt == T_Q4K ? Q4T_BYTES : Q6T_BYTES) * (g.dual ? 2 : 1);
    }
    return b;
  }
  for (uint32_t i = 0; i < p.g.args.nseg; ++i) {
    const GemvSeg& g = p.g.args.seg[i];
    const uint64_t bb = g.qt == T_Q4K ? Q4K_BYTES : Q6K_BYTES;
    b += (uint64_t)g.m * g.nb * bb * (g.dual ? 2 : 1);
  }
  return b;
}

bool dt_tiled(uint32_t dt) { return dt == (uint32_t)T_Q4K_TILED || dt == (uint32_t)T_Q6K_TILED; }

struct LayerPlans {
  ProjPlan qkv, o, gateup, down;
  bool ok = false;
};

}  // namespace

struct shk_model {
  shk_ctx* ctx = nullptr;
  shk_model_desc d{};
  shk_kv* kv = nullptr;
  float *hidden = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr,
        *act = nullptr, *logits = nullptr;
  uint32_t* d_tok = nullptr;  // [0] token, [1] position
  uint32_t* h_tok = nullptr;  // pinned: [0] token in, [1] pos in, [2] token out
  float* am_v = nullptr;
  uint32_t* am_i = nullptr;
  int* am_cnt = nullptr;
  std::vector<shk_layer_desc> layers;
  std::vector<uint8_t> have;
  std::vector<LayerPlans> plans;
  float* d_freq = nullptr;  // RoPE table: powf(1/theta, i/head_dim), host libm
  ProjPlan head;
  bool head_ok = false;      // staged plan available for the output head
  bool head_generic = false; // rows not 16-byte multiples: plain-load GEMV
  cudaGraphExec_t g_layers = nullptr, g_head = nullptr, g_loop = nullptr;
  // persistent decode kernel: program tables in device memory, built on first use
  struct Persist {
    int state = 0;  // 0 not built, 1 ready, -1 not usable (graphs are used)
    DecodeProgram P{};
    size_t smem = 0;
    int grid = 0;
    uint32_t n_phases_full = 0;
    MmvArgs* d_mmv = nullptr;
    AttnArgs* d_attn = nullptr;
    DecodePhase* d_phases = nullptr;
    uint32_t* d_bar = nullptr;
  } pk;
  uint32_t o_lo = 0, o_hi = 0;  // tensor parallel: this rank's rows of the O projection output
  uint32_t v_lo = 0, v_hi = 0;  // ... and of the output head (logits); all rows when replicated
  // Tensor-parallel exchange over NVLink peer memory (shk_cuda_model_tp_p2p_*):
  // a symmetric buffer per rank, [flags: slot][rank] then [parts: slot][rank][n_embd],
  // one slot per all-reduce of a token (2 per layer); the residual stream
  // alternates between hidden and res2.
  struct P2p {
    bool on = false;
    void* base = nullptr;          // this rank's symmetric buffer
    size_t flag_bytes = 0, bytes = 0;
    void* peer_base[GEMV_TP_MAX] = {};  // every rank's buffer (own included)
    bool opened[GEMV_TP_MAX] = {};
    uint32_t* counters = nullptr;  // per slot: producer CTAs done
    uint32_t* d_step = nullptr;    // epoch, advanced by the embedding kernel
    float* res2 = nullptr;
    uint32_t cov_lo[GEMV_TP_MAX] = {}, cov_hi[GEMV_TP_MAX] = {};
  } p2p;
  // Tensor-parallel all-reduce over NVLink peer memory with flags in the data
  // words (shk_cuda_model_tp_ll_*): one exchange buffer per rank,
  // [slot: 2 per layer][rank][n_embd] 8-byte words; replaces the NCCL
  // all-reduce after O and down.
  struct Ll {
    bool on = false;
    void* base = nullptr;          // this rank's buffer
    size_t bytes = 0;
    void* peer[LL_MAX_RANKS] = {};  // every rank's buffer (own included)
    bool opened[LL_MAX_RANKS] = {};
    uint32_t* d_step = nullptr;    // epoch, advanced by the embedding kernel
  } ll;
  uint32_t* tp_pairs = nullptr; // world x {max value bits, index}: argmax over the vocabulary slices
  bool tp_warm = false;          // the graphs' collectives have run once outside capture
  float* pf_buf = nullptr;      // prompt prefill: T-row activation blocks (shk_cuda_prefill)
  size_t pf_cap = 0;
  uint32_t* pf_tok = nullptr;
  size_t pf_tok_cap = 0;
  uint64_t* d_trace = nullptr;  // persistent-kernel timeline (shk_cuda_model_trace_enable)
  uint32_t trace_phases = 0;
  uint32_t trace_last = 0;      // phases recorded by the last launch
};

namespace {

// The status for a device error word already read into e: clears the word.
int ctx_err_take(shk_ctx* c, int e) {
  if (!e) return SHK_OK;
  fprintf(stderr, "shk_cuda: device %d reported error %d\n", c->device, e);
  CK(cudaMemset(c->d_err, 0, sizeof(int)));
  // a launch that gave up may have left a combine count behind
  if (c->mmv_scratch) CK(cudaMemset(c->mmv_scratch, 0, MMV_SCRATCH_BYTES));
  return (e == DERR_TIMEOUT_FULL || e == DERR_TIMEOUT_EMPTY || e == DERR_TIMEOUT_GRID) ? SHK_ETIMEOUT
                                                                                      : SHK_EDEVICE;
}

int ctx_err_check(shk_ctx* c) {
  CK(cudaStreamSynchronize(c->compute));
  CK(cudaMemcpy(c->h_err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  return ctx_err_take(c, *c->h_err);
}

cudaStream_t pick(shk_ctx* c, void* s) { return s ? static_cast<cudaStream_t>(s) : c->compute; }

template <typename T>
int grow(T** p, size_t* cap, size_t need) {
  if (*cap >= need) return SHK_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  if (cudaMalloc(reinterpret_cast<void**>(p), need) != cudaSuccess) return SHK_ENOMEM;
  *cap = need;
  return SHK_OK;
}

// qt: T_Q4K, T_Q6K (GGUF layout) or T_Q6K_PLANAR; row_stride 0 = dense rows.
int matvec_dev(shk_ctx* c, uint32_t qt, const void* w, uint32_t row_stride, const float* x, float* y,
               uint32_t m, uint32_t k, cudaStream_t st) {
  if (!w || !x || !y || k == 0 || k % QK) return SHK_EINVAL;
  if (dt_tiled(qt)) {
    if (m == 0) return SHK_OK;
    MmvMat mt{w, nullptr, y, m, qt, EPI_STORE, 0};
    MmvPlan p;
    const int rc = mmv_plan(p, &mt, 1, k, x, nullptr, nullptr, nullptr, c->d_err, c->num_sms, c->mmv_scratch);
    if (rc) return rc == -2 ? SHK_EUNSUPPORTED : SHK_EINVAL;
    CK(mmv_launch(p, st));
    c->n_matvec++;
    return SHK_OK;
  }
  if (qt == T_Q5K) {
    if (m == 0) return SHK_OK;
    if (row_stride && row_stride != (k / QK) * Q5K_BYTES) return SHK_EINVAL;
    Q5Mat mt{w, nullptr, y, m, EPI_STORE, 0};
    Q5Plan p;
    const int rc = q5k_plan(p, &mt, 1, k, x, nullptr, nullptr, nullptr, c->d_err, c->num_sms);
    if (rc) return rc == -2 ? SHK_EUNSUPPORTED : SHK_EINVAL;
    CK(q5k_launch(p, st));
    c->n_matvec++;
    return SHK_OK;
  }
  if (qt != T_Q4K && qt != T_Q6K && qt != T_Q6K_PLANAR) return SHK_EUNSUPPORTED;
  if (m == 0) return SHK_OK;
  const uint32_t nb = k / QK;
  if (qt == T_Q6K && !row_stride) {
    // GGUF-layout rows: copy into padded rows of a scratch buffer, repack
    // there, then the staged kernel (its weights must be planar) -- when the
    // staged kernel takes this shape; else the plain-load kernel below
    const uint32_t stride = (210u * nb + 15u) & ~15u;
    GemvMat probe{reinterpret_cast<const void*>(uintptr_t(256)), nullptr, y, m, T_Q6K_PLANAR, stride, EPI_STORE, 0};
    GemvPlan pp;
    if (stride <= 227u * 1024u &&
        gemv_plan(pp, &probe, 1, k, x, nullptr, nullptr, nullptr, c->d_err, c->num_sms) == 0) {
      int rc = grow(&c->q6_scratch, &c->q6_scratch_cap, (size_t)m * stride);
      if (rc) return rc;
      CK(cudaMemcpy2DAsync(c->q6_scratch, stride, w, 210u * nb, 210u * nb, m, cudaMemcpyDeviceToDevice, st));
      CK(q6k_repack_launch(c->q6_scratch, m, k, stride, true, c->num_sms, st));
      return matvec_dev(c, T_Q6K_PLANAR, c->q6_scratch, stride, x, y, m, k, st);
    }
  }
  GemvMat mt{w, nullptr, y, m, qt, row_stride, EPI_STORE, 0};
  GemvPlan p;
  const int rc = gemv_plan(p, &mt, 1, k, x, nullptr, nullptr, nullptr, c->d_err, c->num_sms);
  if (rc == 0) {
    CK(gemv_launch(p, st));
  } else if (qt != T_Q6K_PLANAR && !row_stride) {
    // rows not 16-byte multiples, unaligned base, or too large for the staged
    // kernel: plain-load kernel with the same math
    CK(gemv_generic_launch(qt, w, x, y, m, k, st));
  } else {
    return rc == -2 ? SHK_EUNSUPPORTED : SHK_EINVAL;
  }
  c->n_matvec++;
  return SHK_OK;
}

int matvec_host(shk_ctx* c, uint32_t qt, const void* w, const float* x, float* y, uint32_t m,
                uint32_t k) {
  if (!w || !x || !y || k == 0 || k % QK) return SHK_EINVAL;
  const size_t wb = (size_t)m * (k / QK) * (qt == T_Q4K ? Q4K_BYTES : qt == T_Q5K ? Q5K_BYTES : Q6K_BYTES);
  int rc;
  if ((rc = grow(&c->hv_w, &c->hv_w_cap, wb)) || (rc = grow(&c->hv_x, &c->hv_x_cap, (size_t)k * 4)) ||
      (rc = grow(&c->hv_y, &c->hv_y_cap, (size_t)m * 4)))
    return rc;
  CK(cudaMemcpyAsync(c->hv_w, w, wb, cudaMemcpyHostToDevice, c->compute));
  CK(cudaMemcpyAsync(c->hv_x, x, (size_t)k * 4, cudaMemcpyHostToDevice, c->compute));
  rc = matvec_dev(c, qt, c->hv_w, 0, c->hv_x, c->hv_y, m, k, c->compute);
  if (rc) return rc;
  CK(cudaMemcpyAsync(y, c->hv_y, (size_t)m * 4, cudaMemcpyDeviceToHost, c->compute));
  CK(cudaStreamSynchronize(c->compute));
  c->n_matvec_host++;
  return ctx_err_check(c);
}

}  // namespace

extern "C" {

// Every entry point runs on its context's device: a process may hold contexts
// on several GPUs (tensor-parallel ranks) and call them from any thread.
static void on_dev(const shk_ctx* c) {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess || d != c->device) cudaSetDevice(c->device);
}

int shk_cuda_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n > 0;
}

const char* shk_cuda_strerror(int s) {
  switch (s) {
    case SHK_OK: return "ok";
    case SHK_EINVAL: return "invalid argument";
    case SHK_ENOMEM: return "out of memory";
    case SHK_ECUDA: return "CUDA runtime error";
    case SHK_EUNSUPPORTED: return "unsupported dtype or shape";
    case SHK_ETIMEOUT: return "bounded device wait ran out";
    case SHK_ENODEV: return "no CUDA device";
    case SHK_ENCCL: return "collective failure";
    case SHK_EDEVICE: return "kernel reported an error";
    default: return "unknown";
  }
}

shk_ctx* shk_cuda_init(const shk_cuda_config* cfg) {
  if (!shk_cuda_available()) return nullptr;
  shk_ctx* c = new (std::nothrow) shk_ctx();
  if (!c) return nullptr;
  int dev = cfg ? cfg->device : -1;
  if (dev < 0) {
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  }
  c->device = dev;
  c->flags = cfg ? cfg->flags : 0u;
  bool ok = cudaSetDevice(dev) == cudaSuccess;
  ok = ok && cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess;
  ok = ok && cudaStreamCreateWithFlags(&c->compute, cudaStreamNonBlocking) == cudaSuccess;
  ok = ok && cudaStreamCreateWithFlags(&c->copy, cudaStreamNonBlocking) == cudaSuccess;
  ok = ok && cudaMalloc(&c->d_err, sizeof(int)) == cudaSuccess;
  ok = ok && cudaMemset(c->d_err, 0, sizeof(int)) == cudaSuccess;
  ok = ok && cudaMallocHost(&c->h_err, sizeof(int)) == cudaSuccess;
  ok = ok && cudaMalloc(&c->d_u32, 16 * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && cudaMallocHost(&c->h_u32, 16 * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && cudaMalloc(&c->am_v, 256 * sizeof(float)) == cudaSuccess;
  ok = ok && cudaMalloc(&c->am_i, 256 * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && cudaMalloc(&c->am_cnt, sizeof(int)) == cudaSuccess;
  ok = ok && cudaMemset(c->am_cnt, 0, sizeof(int)) == cudaSuccess;
  ok = ok && cudaMalloc(&c->d_freq, 512 * sizeof(float)) == cudaSuccess;
  ok = ok && cudaMallocHost(&c->h_freq, 512 * sizeof(float)) == cudaSuccess;
  ok = ok && gemv_init() == cudaSuccess;
  ok = ok && mmv_init() == cudaSuccess;
  ok = ok && q5k_init() == cudaSuccess;
  ok = ok && cudaMalloc(&c->mmv_scratch, MMV_SCRATCH_BYTES) == cudaSuccess;
  ok = ok && cudaMemset(c->mmv_scratch, 0, MMV_SCRATCH_BYTES) == cudaSuccess;
  if (!ok) {
    shk_cuda_shutdown(c);
    return nullptr;
  }
  return c;
}

void shk_cuda_shutdown(shk_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->compute) cudaStreamSynchronize(c->compute);
  if (c->copy) cudaStreamSynchronize(c->copy);
  for (auto& kv : c->slot_ev) cudaEventDestroy(kv.second);
  for (auto& kv : c->rel_ev) cudaEventDestroy(kv.second);
  if (c->comm && nccl()) nccl()->comm_destroy(c->comm);
  cudaFree(c->d_err);
  cudaFreeHost(c->h_err);
  cudaFree(c->d_u32);
  cudaFreeHost(c->h_u32);
  cudaFree(c->am_v);
  cudaFree(c->am_i);
  cudaFree(c->am_cnt);
  cudaFree(c->d_freq);
  cudaFree(c->mmv_scratch);
  cudaFreeHost(c->h_freq);
  cudaFree(c->hv_w);
  cudaFree(c->q6_scratch);
  cudaFree(c->pf_x);
  cudaFree(c->hv_x);
  cudaFree(c->hv_y);
  if (c->compute) cudaStreamDestroy(c->compute);
  if (c->copy) cudaStreamDestroy(c->copy);
  delete c;
}

void shk_cuda_report(shk_ctx* c) {
  if (c) on_dev(c);
  if (!c) return;
  fprintf(stderr,
          "shk_cuda: device=%d sms=%d matvec_calls=%llu matvec_host_calls=%llu layer_forwards=%llu "
          "token_steps=%llu staged_copies=%llu staged_bytes=%llu\n",
          c->device, c->num_sms, (unsigned long long)c->n_matvec,
          (unsigned long long)c->n_matvec_host, (unsigned long long)c->n_fwd,
          (unsigned long long)c->n_steps, (unsigned long long)c->n_staged,
          (unsigned long long)c->bytes_staged);
}

int shk_cuda_check(shk_ctx* c) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  return ctx_err_check(c);
}

void* shk_cuda_stream(shk_ctx* c) { return c ? c->compute : nullptr; }
int shk_cuda_num_sms(shk_ctx* c) { return c ? c->num_sms : 0; }

int shk_cuda_dev_alloc(shk_ctx* c, size_t bytes, void** out) {
  if (c) on_dev(c);
  if (!c || !out) return SHK_EINVAL;
  *out = nullptr;
  return cudaMalloc(out, bytes ? bytes : 1) == cudaSuccess ? SHK_OK : SHK_ENOMEM;
}
int shk_cuda_dev_free(shk_ctx* c, void* p) {
  if (c) on_dev(c);
  (void)c;
  return cudaFree(p) == cudaSuccess ? SHK_OK : SHK_ECUDA;
}
int shk_cuda_host_alloc(shk_ctx* c, size_t bytes, void** out) {
  if (c) on_dev(c);
  if (!c || !out) return SHK_EINVAL;
  *out = nullptr;
  return cudaMallocHost(out, bytes ? bytes : 1) == cudaSuccess ? SHK_OK : SHK_ENOMEM;
}
int shk_cuda_host_free(shk_ctx* c, void* p) {
  if (c) on_dev(c);
  (void)c;
  return cudaFreeHost(p) == cudaSuccess ? SHK_OK : SHK_ECUDA;
}
int shk_cuda_memcpy_h2d(shk_ctx* c, void* dst, const void* src, size_t bytes, void* s) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, pick(c, s)));
  return SHK_OK;
}
int shk_cuda_memcpy_d2h(shk_ctx* c, void* dst, const void* src, size_t bytes, void* s) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, pick(c, s)));
  return SHK_OK;
}
int shk_cuda_sync(shk_ctx* c, void* s) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  CK(cudaStreamSynchronize(pick(c, s)));
  return SHK_OK;
}

int shk_cuda_matmul_q4k_vec(shk_ctx* c, const void* w, const float* x, float* y, uint32_t m,
                            uint32_t k, void* s) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  return matvec_dev(c, T_Q4K, w, 0, x, y, m, k, pick(c, s));
}
int shk_cuda_matmul_q6k_vec(shk_ctx* c, const void* w, const float* x, float* y, uint32_t m,
                            uint32_t k, void* s) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  return matvec_dev(c, T_Q6K, w, 0, x, y, m, k, pick(c, s));
}
int shk_cuda_matmul_q5k_vec(shk_ctx* c, const void* w, const float* x, float* y, uint32_t m,
                            uint32_t k, void* s) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  return matvec_dev(c, T_Q5K, w, 0, x, y, m, k, pick(c, s));
}
int shk_cuda_matvec(shk_ctx* c, uint32_t dtype, const void* w, uint32_t row_stride, const float* x, float* y,
                    uint32_t m, uint32_t k, void* s) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  return matvec_dev(c, dtype, w, row_stride, x, y, m, k, pick(c, s));
}
int shk_cuda_prefill_matmul(shk_ctx* c, uint32_t dtype, const void* w, uint32_t row_stride, const float* x,
                            float* y, uint32_t m, uint32_t k, uint32_t n_tokens, void* s) {
  if (c) on_dev(c);
  if (!c || !w || !x || !y || k == 0 || k % QK) return SHK_EINVAL;
  if (dtype != T_Q4K && dtype != T_Q6K_PLANAR) return SHK_EUNSUPPORTED;
  if (m == 0 || n_tokens == 0) return SHK_OK;
  const uint32_t nb = k / QK;
  const uint32_t dense = nb * (dtype == T_Q4K ? Q4K_BYTES : Q6K_BYTES);
  const uint32_t stride = row_stride ? row_stride : dense;
  if (stride < dense || stride % 16 || (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 7))
    return SHK_EINVAL;
  int rc = grow(&c->pf_x, &c->pf_x_cap, prefill_x_bytes(k, n_tokens));
  if (rc) return rc;
  CK(prefill_launch(dtype, w, stride, x, c->pf_x, y, m, k, n_tokens, c->d_err, c->num_sms, pick(c, s)));
  return SHK_OK;
}

int shk_cuda_q6k_repack(shk_ctx* c, void* w, uint32_t rows, uint32_t k, uint32_t row_stride, int to_planar,
                        void* s) {
  if (c) on_dev(c);
  if (!c || !w || k == 0 || k % QK) return SHK_EINVAL;
  const uint32_t stride = row_stride ? row_stride : 210u * (k / QK);
  if (stride % 16 || stride < 210u * (k / QK) || stride > 227u * 1024u || (reinterpret_cast<uintptr_t>(w) & 15))
    return SHK_EINVAL;
  CK(q6k_repack_launch(w, rows, k, stride, to_planar != 0, c->num_sms, pick(c, s)));
  return SHK_OK;
}

size_t shk_cuda_tiled_bytes(uint32_t dtype, uint32_t rows, uint32_t k) {
  if (k == 0 || k % QK) return 0;
  if (dtype == T_Q4K || dtype == (uint32_t)T_Q4K_TILED) return mmv_tiled_bytes(T_Q4K_TILED, rows, k);
  if (dtype == T_Q6K || dtype == (uint32_t)T_Q6K_TILED) return mmv_tiled_bytes(T_Q6K_TILED, rows, k);
  return 0;
}

int shk_cuda_tile(shk_ctx* c, uint32_t dtype, const void* src, uint32_t src_row_stride, uint32_t rows, uint32_t k,
                  void* dst, void* s) {
  if (c) on_dev(c);
  if (!c || !src || !dst || rows == 0 || k == 0 || k % QK) return SHK_EINVAL;
  if (dtype != T_Q4K && dtype != T_Q6K) return SHK_EUNSUPPORTED;
  cudaSetDevice(c->device);
  const cudaError_t e = mmv_tile_launch(dtype, src, src_row_stride, rows, k, dst, pick(c, s));
  if (e == cudaErrorInvalidValue) return SHK_EINVAL;
  CK(e);
  return SHK_OK;
}
int shk_cuda_matmul_q4k_vec_host(shk_ctx* c, const void* w, const float* x, float* y, uint32_t m,
                                 uint32_t k) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  return matvec_host(c, T_Q4K, w, x, y, m, k);
}
int shk_cuda_matmul_q6k_vec_host(shk_ctx* c, const void* w, const float* x, float* y, uint32_t m,
                                 uint32_t k) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  return matvec_host(c, T_Q6K, w, x, y, m, k);
}
int shk_cuda_matmul_q5k_vec_host(shk_ctx* c, const void* w, const float* x, float* y, uint32_t m,
                                 uint32_t k) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  return matvec_host(c, T_Q5K, w, x, y, m, k);
}

int shk_cuda_rmsnorm(shk_ctx* c, const float* x, const float* w, float* y, uint32_t d, void* s) {
  if (c) on_dev(c);
  if (!c || !x || !w || !y || !d) return SHK_EINVAL;
  CK(rmsnorm_launch(x, w, y, d, pick(c, s)));
  return SHK_OK;
}

int shk_cuda_rope(shk_ctx* c, float* qk, uint32_t n_heads, uint32_t hd, uint32_t pos, float theta,
                  void* s) {
  if (c) on_dev(c);
  if (!c || !qk || hd == 0 || (hd & 1) || hd > 1024 || !(theta > 0.f)) return SHK_EINVAL;
  cudaStream_t st = pick(c, s);
  // position and frequency table go through stream-ordered copies
  CK(cudaStreamSynchronize(st));
  c->h_u32[0] = pos;
  rope_freq_table(theta, hd, c->h_freq);
  CK(cudaMemcpyAsync(c->d_u32, c->h_u32, 4, cudaMemcpyHostToDevice, st));
  CK(cudaMemcpyAsync(c->d_freq, c->h_freq, (hd / 2) * sizeof(float), cudaMemcpyHostToDevice, st));
  CK(rope_launch(qk, n_heads, hd, c->d_u32, c->d_freq, st));
  return SHK_OK;
}

int shk_cuda_swiglu(shk_ctx* c, const float* g, const float* u, float* h, uint32_t n, void* s) {
  if (c) on_dev(c);
  if (!c || !g || !u || !h) return SHK_EINVAL;
  CK(swiglu_launch(g, u, h, n, pick(c, s)));
  return SHK_OK;
}

int shk_cuda_embed(shk_ctx* c, const void* table, uint32_t dtype, uint32_t n_vocab, uint32_t token,
                   float* out, uint32_t n_embd, void* s) {
  if (c) on_dev(c);
  if (!c || !table || !out || !n_embd) return SHK_EINVAL;
  if (dtype != 1 && dtype != T_Q4K) return SHK_EUNSUPPORTED;
  if (dtype == T_Q4K && n_embd % QK) return SHK_EINVAL;
  if (token >= n_vocab) return SHK_EINVAL;
  cudaStream_t st = pick(c, s);
  CK(cudaStreamSynchronize(st));
  c->h_u32[1] = token;
  CK(cudaMemcpyAsync(c->d_u32 + 1, c->h_u32 + 1, 4, cudaMemcpyHostToDevice, st));
  CK(embed_launch(table, dtype, c->d_u32 + 1, n_vocab, out, n_embd, c->d_err, st));
  return SHK_OK;
}

int shk_cuda_argmax(shk_ctx* c, const float* x, uint32_t n, uint32_t* out) {
  if (c) on_dev(c);
  // index 0xFFFFFFFF marks an empty block partial, so n stops one below it
  if (!c || !x || !out || !n || n > SHK_ARGMAX_NOALLOC_MAX_N) return SHK_EINVAL;
  CK(argmax_launch(x, n, c->am_v, c->am_i, c->am_cnt, c->d_u32 + 2, nullptr, c->compute));
  CK(cudaMemcpyAsync(c->h_u32 + 2, c->d_u32 + 2, 4, cudaMemcpyDeviceToHost, c->compute));
  CK(cudaStreamSynchronize(c->compute));
  *out = c->h_u32[2];
  return SHK_OK;
}

// ------------------------------- KV cache -------------------------------------

shk_kv* shk_cuda_kv_create(shk_ctx* c, const shk_kv_config* cfg) {
  if (c) on_dev(c);
  if (!c || !cfg || !cfg->n_layers || !cfg->n_kv_heads || !cfg->max_seq_len) return nullptr;
  if (cfg->head_dim != 64 && cfg->head_dim != 128) return nullptr;
  shk_kv* kv = new (std::nothrow) shk_kv();
  if (!kv) return nullptr;
  kv->ctx = c;
  kv->L = kv_layout_make(cfg->n_layers, cfg->n_kv_heads, cfg->head_dim, cfg->max_seq_len);
  kv->seq.assign(cfg->n_layers, 0);
  // split-K fan-out: about two CTAs per SM across the KV heads
  kv->max_splits = std::max<uint32_t>(1, std::min<uint32_t>(128, (4 * c->num_sms + cfg->n_kv_heads - 1) / cfg->n_kv_heads));
  const size_t bytes = kv->L.head_bytes * cfg->n_layers * cfg->n_kv_heads;
  // partials sized for up to 8 query heads per KV head
  const size_t part = attn_part_floats(8 * cfg->n_kv_heads, cfg->n_kv_heads, cfg->head_dim, kv->max_splits);
  bool ok = cudaMalloc(&kv->L.base, bytes) == cudaSuccess;
  ok = ok && cudaMemset(kv->L.base, 0, bytes) == cudaSuccess;
  ok = ok && cudaMalloc(&kv->part, part * sizeof(float)) == cudaSuccess;
  // one ticket counter per KV head, or per (KV head, cluster rank) in the
  // long-cache attention kernel: 8 per head
  ok = ok && cudaMalloc(&kv->counters, 8 * cfg->n_kv_heads * sizeof(int)) == cudaSuccess;
  ok = ok && cudaMemset(kv->counters, 0, 8 * cfg->n_kv_heads * sizeof(int)) == cudaSuccess;
  ok = ok && cudaMalloc(&kv->d_iota, (size_t)cfg->max_seq_len * sizeof(uint32_t)) == cudaSuccess;
  if (ok) {
    std::vector<uint32_t> io(cfg->max_seq_len);
    for (uint32_t i = 0; i < cfg->max_seq_len; ++i) io[i] = i;
    ok = cudaMemcpy(kv->d_iota, io.data(), io.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
  }
  if (!ok) {
    shk_cuda_kv_destroy(kv);
    return nullptr;
  }
  return kv;
}

void shk_cuda_kv_destroy(shk_kv* kv) {
  if (kv) on_dev(kv->ctx);
  if (!kv) return;
  if (kv->ctx) cudaStreamSynchronize(kv->ctx->compute);
  cudaFree(kv->L.base);
  cudaFree(kv->part);
  cudaFree(kv->counters);
  cudaFree(kv->d_iota);
  cudaFree(kv->part_batch);
  cudaFree(kv->counters_batch);
  delete kv;
}

int shk_cuda_kv_append(shk_kv* kv, uint32_t layer, uint32_t pos, const float* k, const float* v,
                       void* s) {
  if (kv) on_dev(kv->ctx);
  if (!kv || !k || !v || layer >= kv->L.n_layers || pos >= kv->L.max_seq) return SHK_EINVAL;
  CK(kv_append_launch(kv->L, layer, kv->d_iota + pos, k, v, kv->ctx->d_err, pick(kv->ctx, s)));
  kv->seq[layer] = std::max(kv->seq[layer], pos + 1);
  return SHK_OK;
}

int shk_cuda_kv_append_range(shk_kv* kv, uint32_t layer, uint32_t start, uint32_t n,
                             const float* k, const float* v, void* s) {
  if (kv) on_dev(kv->ctx);
  if (!kv || !k || !v || layer >= kv->L.n_layers || start > kv->L.max_seq ||
      n > kv->L.max_seq - start)
    return SHK_EINVAL;
  if (n == 0) return SHK_OK;
  CK(kv_append_range_launch(kv->L, layer, start, n, k, v, pick(kv->ctx, s)));
  kv->seq[layer] = std::max(kv->seq[layer], start + n);
  return SHK_OK;
}

int shk_cuda_kv_read_range(shk_kv* kv, uint32_t layer, uint32_t start, uint32_t end, float* k,
                           float* v, void* s) {
  if (kv) on_dev(kv->ctx);
  if (!kv || !k || !v || end < start || layer >= kv->L.n_layers || end > kv->L.max_seq)
    return SHK_EINVAL;
  CK(kv_read_range_launch(kv->L, layer, start, end, k, v, pick(kv->ctx, s)));
  return SHK_OK;
}

int shk_cuda_kv_read_blocks(shk_kv* kv, uint32_t layer, uint32_t start, uint32_t end, void* k,
                            void* v, void* s) {
  if (kv) on_dev(kv->ctx);
  if (!kv || !k || !v || end < start || layer >= kv->L.n_layers || end > kv->L.max_seq)
    return SHK_EINVAL;
  CK(kv_read_blocks_launch(kv->L, layer, start, end, static_cast<uint8_t*>(k),
                           static_cast<uint8_t*>(v), pick(kv->ctx, s)));
  return SHK_OK;
}

int shk_cuda_kv_attend(shk_kv* kv, uint32_t layer, const float* q, const float* k_new,
                       const float* v_new, float* out, uint32_t n_heads, uint32_t seq_len,
                       float scale, void* s) {
  if (kv) on_dev(kv->ctx);
  if (!kv || !q || !out || layer >= kv->L.n_layers || seq_len == 0 || seq_len > kv->L.max_seq)
    return SHK_EINVAL;
  if (n_heads % kv->L.n_kv || n_heads / kv->L.n_kv > 8) return SHK_EUNSUPPORTED;
  if ((k_new == nullptr) != (v_new == nullptr)) return SHK_EINVAL;
  AttnArgs a{};
  a.kv = kv->L;
  a.layer = layer;
  a.n_heads = n_heads;
  a.scale = scale;
  a.q = q;
  a.k_new = k_new;
  a.v_new = v_new;
  a.pos = kv->d_iota + (seq_len - 1);
  a.out = out;
  a.part = kv->part;
  a.counters = kv->counters;
  a.max_splits = kv->max_splits;
  a.min_per_split = SHK_ATT_MIN_SPLIT;
  a.err = kv->ctx->d_err;
  CK(attn_decode_launch(a, pick(kv->ctx, s)));
  if (k_new) kv->seq[layer] = std::max(kv->seq[layer], seq_len);
  return SHK_OK;
}

int shk_cuda_kv_attend_batch(shk_kv* kv, uint32_t layer0, uint32_t n_seq, const float* q, const float* k_new,
                             const float* v_new, float* out, uint32_t n_heads, uint32_t seq_len, float scale,
                             void* s) {
  if (kv) on_dev(kv->ctx);
  if (!kv || !q || !out || n_seq == 0 || layer0 + n_seq > kv->L.n_layers || layer0 + n_seq < layer0 ||
      seq_len == 0 || seq_len > kv->L.max_seq)
    return SHK_EINVAL;
  if (n_heads % kv->L.n_kv || n_heads / kv->L.n_kv > 8) return SHK_EUNSUPPORTED;
  if ((k_new == nullptr) != (v_new == nullptr)) return SHK_EINVAL;
  const size_t per = attn_part_floats(8 * kv->L.n_kv, kv->L.n_kv, kv->L.hd, kv->max_splits);
  if (n_seq > kv->batch_cap) {  // grown outside any capture (first call of a size)
    cudaStream_t st = pick(kv->ctx, s);
    CK(cudaStreamSynchronize(st));
    cudaFree(kv->part_batch);
    cudaFree(kv->counters_batch);
    kv->part_batch = nullptr;
    kv->counters_batch = nullptr;
    kv->batch_cap = 0;
    if (cudaMalloc(&kv->part_batch, per * n_seq * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&kv->counters_batch, (size_t)8 * kv->L.n_kv * n_seq * sizeof(int)) != cudaSuccess)
      return SHK_ENOMEM;
    CK(cudaMemset(kv->counters_batch, 0, (size_t)8 * kv->L.n_kv * n_seq * sizeof(int)));
    kv->batch_cap = n_seq;
  }
  AttnArgs a{};
  a.kv = kv->L;
  a.layer = layer0;
  a.n_heads = n_heads;
  a.scale = scale;
  a.q = q;
  a.k_new = k_new;
  a.v_new = v_new;
  a.pos = kv->d_iota + (seq_len - 1);
  a.out = out;
  a.part = kv->part_batch;
  a.counters = kv->counters_batch;
  a.max_splits = kv->max_splits;
  a.min_per_split = SHK_ATT_MIN_SPLIT;
  a.err = kv->ctx->d_err;
  a.n_seq = n_seq;
  a.qo_stride = (size_t)n_heads * kv->L.hd;
  a.kv_stride = (size_t)kv->L.n_kv * kv->L.hd;
  a.part_stride = per;
  const cudaError_t e = attn_decode_batch_launch(a, pick(kv->ctx, s));
  if (e == cudaErrorNotSupported) {  // unaligned rows: one launch per sequence
    for (uint32_t z = 0; z < n_seq; ++z) {
      const int rc = shk_cuda_kv_attend(kv, layer0 + z, q + z * a.qo_stride, k_new ? k_new + z * a.kv_stride : nullptr,
                                        v_new ? v_new + z * a.kv_stride : nullptr, out + z * a.qo_stride, n_heads,
                                        seq_len, scale, s);
      if (rc) return rc;
    }
    return SHK_OK;
  }
  CK(e);
  if (k_new)
    for (uint32_t z = 0; z < n_seq; ++z) kv->seq[layer0 + z] = std::max(kv->seq[layer0 + z], seq_len);
  return SHK_OK;
}

void shk_cuda_kv_clear(shk_kv* kv) {
  if (kv) std::fill(kv->seq.begin(), kv->seq.end(), 0u);
}

uint32_t shk_cuda_kv_seq_len(shk_kv* kv, uint32_t layer) {
  return (kv && layer < kv->L.n_layers) ? kv->seq[layer] : 0;
}

// --------------------------------- model --------------------------------------

namespace {

void model_free_graphs(shk_model* m) {
  if (m->g_layers) cudaGraphExecDestroy(m->g_layers);
  if (m->g_head) cudaGraphExecDestroy(m->g_head);
  if (m->g_loop) cudaGraphExecDestroy(m->g_loop);
  m->g_layers = m->g_head = m->g_loop = nullptr;
  auto& k = m->pk;
  cudaFree(k.d_mmv);
  cudaFree(k.d_attn);
  cudaFree(k.d_phases);
  cudaFree(k.d_bar);
  k = shk_model::Persist{};
}

// Tensor-parallel exchange fields of a plan: slot j's consumer (in) or producer
// (out); see GemvTp.
void p2p_in(shk_model* m, GemvArgs& a, uint32_t j, const float* res_in, float* res_out) {
  const auto& q = m->p2p;
  const uint32_t W = (uint32_t)m->ctx->tp_world, D = m->d.n_embd;
  GemvTp& t = a.tp;
  t.in = 1;
  t.rank = (uint8_t)m->ctx->tp_rank;
  t.world = (uint8_t)W;
  t.d = D;
  t.flags_in = reinterpret_cast<const uint32_t*>(static_cast<uint8_t*>(q.base)) + (size_t)j * W;
  t.parts_in = reinterpret_cast<const float*>(static_cast<uint8_t*>(q.base) + q.flag_bytes) + (size_t)j * W * D;
  t.res_out = res_out;
  t.epoch = q.d_step;
  const bool after_o = (j & 1) == 0;  // O partials cover each rank's O rows; down partials all rows
  for (uint32_t r = 0; r < W; ++r) {
    t.cov_lo[r] = after_o ? q.cov_lo[r] : 0;
    t.cov_hi[r] = after_o ? q.cov_hi[r] : D;
  }
  a.x = res_in;
}
void p2p_out(shk_model* m, GemvArgs& a, uint32_t j, uint32_t row_off) {
  const auto& q = m->p2p;
  const uint32_t W = (uint32_t)m->ctx->tp_world, D = m->d.n_embd;
  GemvTp& t = a.tp;
  t.out = 1;
  t.rank = (uint8_t)m->ctx->tp_rank;
  t.world = (uint8_t)W;
  t.d = D;
  t.row_off = row_off;
  t.counter = q.counters + j;
  t.epoch = q.d_step;
  for (uint32_t p = 0; p < W; ++p) {
    uint8_t* b = static_cast<uint8_t*>(q.peer_base[p]);
    t.flags_out[p] = reinterpret_cast<uint32_t*>(b) + (size_t)j * W;
    t.parts_out[p] = reinterpret_cast<float*>(b + q.flag_bytes) + (size_t)j * W * D;
  }
}

// Plans one projection: the tensor-core matvec when every matrix is row-tiled,
// else the staged GEMV (a mix is not supported).
int plan_proj(shk_model* m, ProjPlan& P, const GemvMat* all, int n_all, uint32_t k, const float* x,
              const float* norm_w, const uint32_t* pos) {
  shk_ctx* c = m->ctx;
  // Q5_K matrices go to their own kernel (the reference's Q5_K layout, rows
  // dense), the rest to one staged GEMV or tensor-core matvec launch
  GemvMat mats[GEMV_MAX_SEGS];
  Q5Mat q5[Q5_MAX_SEGS];
  int n = 0, n5 = 0;
  for (int i = 0; i < n_all; ++i) {
    if (all[i].qt == (uint32_t)T_Q5K) {
      if (all[i].row_stride && all[i].row_stride != (k / QK) * Q5K_BYTES) return SHK_EINVAL;
      if (all[i].epi == EPI_TP) return SHK_EUNSUPPORTED;
      q5[n5++] = Q5Mat{all[i].w, all[i].w2, all[i].y, all[i].m, all[i].epi, all[i].rope_hd};
    } else {
      mats[n++] = all[i];
    }
  }
  P.has_q5 = n5 > 0;
  P.main = n > 0;
  if (P.has_q5) {
    const int r5 = q5k_plan(P.q5, q5, n5, k, x, norm_w, pos, m->d_freq, c->d_err, c->num_sms);
    if (r5) return r5 == -2 ? SHK_EUNSUPPORTED : SHK_EINVAL;
  }
  if (!P.main) {
    P.tiled = false;
    return SHK_OK;
  }
  int nt = 0;
  for (int i = 0; i < n; ++i) nt += dt_tiled(mats[i].qt) ? 1 : 0;
  if (nt != 0 && nt != n) return SHK_EUNSUPPORTED;
  P.tiled = nt == n;
  int rc;
  if (P.tiled) {
    MmvMat mm[MMV_MAX_SEGS];
    for (int i = 0; i < n; ++i)
      mm[i] = MmvMat{mats[i].w, mats[i].w2, mats[i].y, mats[i].m, mats[i].qt, mats[i].epi, mats[i].rope_hd};
    // the persistent kernel's shared ring: items of at most two Q6_K tiles
    const uint32_t cap = (c->flags & SHK_CUDA_FLAG_PERSISTENT) ? 2u * Q6T_BYTES : 0u;
    rc = mmv_plan(P.mm, mm, n, k, x, norm_w, pos, m->d_freq, c->d_err, c->num_sms, c->mmv_scratch, cap);
  } else {
    rc = gemv_plan(P.g, mats, n, k, x, norm_w, pos, m->d_freq, c->d_err, c->num_sms);
  }
  return rc == 0 ? SHK_OK : rc == -2 ? SHK_EUNSUPPORTED : SHK_EINVAL;
}

int build_layer_plans(shk_model* m, const shk_layer_desc& lv, LayerPlans& P, uint32_t layer) {
  const shk_model_desc& d = m->d;
  shk_ctx* c = m->ctx;
  const uint32_t hd = d.head_dim, qd = d.n_heads * hd, kvd = d.n_kv_heads * hd;
  const uint32_t* pos = m->d_tok + 1;
  GemvMat qkv[3] = {
      {lv.attn_q, nullptr, m->q, qd, lv.attn_q_dtype, 0, EPI_ROPE, hd},
      {lv.attn_k, nullptr, m->k, kvd, lv.attn_k_dtype, 0, EPI_ROPE, hd},
      {lv.attn_v, nullptr, m->v, kvd, lv.attn_v_dtype, lv.row_stride_v, EPI_STORE, 0},
  };
  int rc = plan_proj(m, P.qkv, qkv, 3, d.n_embd, m->hidden, lv.attn_norm, pos);
  if (rc) return rc;
  // Tensor parallel over NCCL: rank 0 adds the residual, the others store
  // their partial sums (all-reduced afterwards); the O projection covers rows
  // [o_lo, o_hi).  Over peer memory (p2p): every rank sends pure partials
  // (EPI_TP) and the consumer adds the residual.
  const bool p2p = m->p2p.on;
  const uint8_t res_epi = p2p ? EPI_TP : (c->tp_rank == 0 ? EPI_ADD : EPI_STORE);
  GemvMat o{lv.attn_o, nullptr, m->hidden + m->o_lo, m->o_hi - m->o_lo, lv.attn_o_dtype, 0, res_epi, 0};
  if ((rc = plan_proj(m, P.o, &o, 1, qd, m->att, nullptr, nullptr))) return rc;
  if (lv.ffn_gate_dtype != lv.ffn_up_dtype) return SHK_EUNSUPPORTED;
  GemvMat gu{lv.ffn_gate, lv.ffn_up, m->act, d.n_ff, lv.ffn_gate_dtype, 0, EPI_SWIGLU, 0};
  if ((rc = plan_proj(m, P.gateup, &gu, 1, d.n_embd, m->hidden, lv.ffn_norm, nullptr))) return rc;
  GemvMat dn{lv.ffn_down, nullptr, m->hidden, d.n_embd, lv.ffn_down_dtype, lv.row_stride_down, res_epi, 0};
  if ((rc = plan_proj(m, P.down, &dn, 1, d.n_ff, m->act, nullptr, nullptr))) return rc;
  if (p2p) {
    for (const ProjPlan* pp : {&P.qkv, &P.o, &P.gateup, &P.down})
      if (pp->tiled || pp->has_q5 || !pp->main) return SHK_EUNSUPPORTED;
    // slots: 2l = O of layer l (consumed by gate/up), 2l + 1 = down (consumed
    // by the next layer's QKV or the head); consumer j reads the residual
    // from buffer j % 2 (0 = hidden, 1 = res2) and writes it to the other
    if (layer > 0) p2p_in(m, P.qkv.g.args, 2 * layer - 1, m->p2p.res2, m->hidden);
    p2p_out(m, P.o.g.args, 2 * layer, m->o_lo);
    p2p_in(m, P.gateup.g.args, 2 * layer, m->hidden, m->p2p.res2);
    p2p_out(m, P.down.g.args, 2 * layer + 1, 0);
  }
  P.ok = true;
  return SHK_OK;
}

AttnArgs layer_attn_args(shk_model* m, uint32_t layer, const uint32_t* pos) {
  AttnArgs a{};
  a.kv = m->kv->L;
  a.layer = layer;
  a.n_heads = m->d.n_heads;
  a.scale = 1.0f / sqrtf((float)m->d.head_dim);
  a.q = m->q;
  a.k_new = m->k;
  a.v_new = m->v;
  a.pos = pos;
  a.out = m->att;
  a.part = m->kv->part;
  a.counters = m->kv->counters;
  a.max_splits = m->kv->max_splits;
  a.min_per_split = SHK_ATT_MIN_SPLIT;
  a.err = m->ctx->d_err;
  return a;
}

// Enqueues one layer: fused RMSNorm+QKV(+RoPE), append+attention, O(+residual),
// RMSNorm+gate/up(+SwiGLU), down(+residual).  `pos` is a device pointer.
//
// Tensor parallel (world > 1): the residual stream is replicated; after the O
// and down projections the ranks' partial sums are all-reduced (rank 0's
// epilogue adds the residual, the others store).  `pdl`: launches that follow
// one of our kernels may be programmatic dependents; a launch that follows a
// collective or a memset never is (the dependency edge is only defined
// between kernels), and the caller's launch after this layer inherits
// pdl_enabled() as left here.
LlArgs ll_args(const shk_model* m) {
  LlArgs a{};
  for (int p = 0; p < m->ctx->tp_world && p < LL_MAX_RANKS; ++p) a.peer[p] = static_cast<uint64_t*>(m->ll.peer[p]);
  a.epoch = m->ll.d_step;
  a.err = m->ctx->d_err;
  a.rank = (uint32_t)m->ctx->tp_rank;
  a.world = (uint32_t)m->ctx->tp_world;
  a.d = m->d.n_embd;
  return a;
}

int enqueue_layer(shk_model* m, const LayerPlans& P, uint32_t layer, const uint32_t* pos,
                  cudaStream_t st, bool pdl) {
  shk_ctx* c = m->ctx;
  const bool tp = c->tp_world > 1;
  CK(proj_launch(P.qkv, st, pos));
  pdl_enabled() = pdl;
  const AttnArgs a = layer_attn_args(m, layer, pos);
  CK(attn_decode_launch(a, st));
  const bool ll = tp && m->ll.on;  // all-reduce over peer memory, flags in the data words
  const bool nccl_ar = tp && !m->p2p.on && !ll;
  if ((nccl_ar || ll) && c->tp_rank != 0 && m->o_hi - m->o_lo < m->d.n_embd) {  // rows this rank does not write
    CK(cudaMemsetAsync(m->hidden, 0, (size_t)m->d.n_embd * sizeof(float), st));
    pdl_enabled() = false;
  }
  CK(proj_launch(P.o, st));
  if (nccl_ar) {
    if (nccl()->all_reduce(m->hidden, m->hidden, m->d.n_embd, ncclFloat, ncclSum, c->comm, st) != ncclSuccess)
      return SHK_ENCCL;
    pdl_enabled() = false;
  } else if (ll) {
    pdl_enabled() = pdl;
    CK(ar_ll_launch(ll_args(m), m->hidden, 2 * layer, st));
  }
  pdl_enabled() = nccl_ar ? false : pdl;
  CK(proj_launch(P.gateup, st));
  pdl_enabled() = pdl;
  CK(proj_launch(P.down, st));
  if (nccl_ar) {
    if (nccl()->all_reduce(m->hidden, m->hidden, m->d.n_embd, ncclFloat, ncclSum, c->comm, st) != ncclSuccess)
      return SHK_ENCCL;
    pdl_enabled() = false;
  } else if (ll) {
    CK(ar_ll_launch(ll_args(m), m->hidden, 2 * layer + 1, st));
  }
  return SHK_OK;
}

// The output head runs staged (plan 0) or, for Q4_K / GGUF-layout Q6_K, on the
// plain-load kernel; a planar head must plan.
bool head_plan_ok(uint32_t dtype, int hp) {
  if (hp == 0) return true;
  return dtype == T_Q4K ? hp != -2 : dtype == T_Q6K;
}

bool vocab_split(const shk_model* m) { return m->v_hi - m->v_lo < m->d.n_vocab; }

// (Re)plans the output head over rows [v_lo, v_hi); with the peer-memory
// exchange the head is the consumer of the last layer's down partials.
int plan_head(shk_model* m) {
  shk_ctx* c = m->ctx;
  const uint32_t nv = m->v_hi - m->v_lo;
  m->head.main = true;
  m->head.has_q5 = false;
  if (m->d.output_dtype == (uint32_t)T_Q5K) {  // engine/src/engine.c:410 (a Q5_K head)
    if (m->p2p.on) return SHK_EUNSUPPORTED;
    Q5Mat hm{m->d.output_dev, nullptr, m->logits + m->v_lo, nv, EPI_STORE, 0};
    m->head.tiled = false;
    m->head.main = false;
    m->head.has_q5 = true;
    m->head_generic = false;
    if (q5k_plan(m->head.q5, &hm, 1, m->d.n_embd, m->hidden, nullptr, nullptr, nullptr, c->d_err, c->num_sms))
      return SHK_EUNSUPPORTED;
    m->head_ok = true;
    return SHK_OK;
  }
  if (dt_tiled(m->d.output_dtype)) {
    if (m->p2p.on) return SHK_EUNSUPPORTED;
    MmvMat hm{m->d.output_dev, nullptr, m->logits + m->v_lo, nv, m->d.output_dtype, EPI_STORE, 0};
    m->head.tiled = true;
    m->head_generic = false;
    if (mmv_plan(m->head.mm, &hm, 1, m->d.n_embd, m->hidden, nullptr, nullptr, nullptr, c->d_err, c->num_sms,
                 c->mmv_scratch))
      return SHK_EUNSUPPORTED;
    m->head_ok = true;
    return SHK_OK;
  }
  m->head.tiled = false;
  GemvMat hm{m->d.output_dev, nullptr, m->logits + m->v_lo, nv, m->d.output_dtype, 0, EPI_STORE, 0};
  // 48 KB stages for the head (431 MB at the 8B shape): 84 against 86 us with
  // the layers' 32 KB, 99 us with 64 KB
  const int hp = gemv_plan(m->head.g, &hm, 1, m->d.n_embd, m->hidden, nullptr, nullptr, nullptr, c->d_err,
                           c->num_sms, 49152);
  if (!head_plan_ok(m->d.output_dtype, hp)) return SHK_EUNSUPPORTED;
  m->head_generic = hp != 0;
  if (m->p2p.on) {
    // the head consumes the last down partials: in its prologue, or (plain-load
    // head) through a sum kernel before it that writes hidden
    p2p_in(m, m->head.g.args, 2 * m->d.n_layers - 1, m->p2p.res2, m->hidden);
  }
  m->head_ok = true;
  return SHK_OK;
}

// Tensor parallel with a split output head: every rank's logits slice is
// gathered into the full vector (in place), e.g. before a copy to the host.
int gather_logits(shk_model* m, cudaStream_t st) {
  if (!vocab_split(m)) return SHK_OK;
  const uint32_t n = m->v_hi - m->v_lo;
  if (nccl()->all_gather(m->logits + m->v_lo, m->logits, n, ncclFloat, m->ctx->comm, st) != ncclSuccess)
    return SHK_ENCCL;
  return SHK_OK;
}

// pdl_after_first: launches after the first one carry the programmatic
// dependent launch attribute (used while capturing the decode-step graphs).
// With the output head split over tensor-parallel ranks, each rank takes the
// first maximum of its slice, the (value, index) pairs are all-gathered and
// merged in rank order.
int enqueue_head(shk_model* m, cudaStream_t st, bool advance_pos, bool pdl_after_first = false) {
  const uint32_t nv = m->v_hi - m->v_lo;
  if (m->head_generic) {
    if (m->p2p.on) {
      CK(gemv_tp_sum_launch(m->head.g.args, st));
      pdl_enabled() = false;
    }
    CK(gemv_generic_launch(m->d.output_dtype, m->d.output_dev, m->hidden, m->logits + m->v_lo, nv,
                           m->d.n_embd, st));
  } else {
    CK(proj_launch(m->head, st));
  }
  if (pdl_after_first) pdl_enabled() = true;
  uint32_t* pos_inc = advance_pos ? m->d_tok + 1 : nullptr;
  if (!vocab_split(m)) {
    CK(argmax_launch(m->logits, m->d.n_vocab, m->am_v, m->am_i, m->am_cnt, m->d_tok, pos_inc, st));
    return SHK_OK;
  }
  shk_ctx* c = m->ctx;
  uint32_t* mine = m->tp_pairs + 2 * c->tp_rank;
  CK(argmax_launch(m->logits + m->v_lo, nv, m->am_v, m->am_i, m->am_cnt, mine + 1, nullptr, st, m->v_lo,
                   reinterpret_cast<float*>(mine)));
  if (nccl()->all_gather(mine, m->tp_pairs, 2, ncclUint32, c->comm, st) != ncclSuccess) return SHK_ENCCL;
  const bool pdl = pdl_enabled();
  pdl_enabled() = false;
  CK(argmax_ranks_launch(m->tp_pairs, c->tp_world, m->d_tok, pos_inc, st));
  pdl_enabled() = pdl;
  return SHK_OK;
}

int enqueue_layers(shk_model* m, cudaStream_t st, bool pdl_after_first = false) {
  CK(embed_launch(m->d.tok_embd_dev, m->d.tok_embd_dtype, m->d_tok, m->d.n_vocab, m->hidden,
                  m->d.n_embd, m->ctx->d_err, st,
                  m->p2p.on ? m->p2p.d_step : m->ll.on ? m->ll.d_step : nullptr));
  if (pdl_after_first) pdl_enabled() = true;
  for (uint32_t l = 0; l < m->d.n_layers; ++l) {
    const int rc = enqueue_layer(m, m->plans[l], l, m->d_tok + 1, st, pdl_after_first);
    if (rc) return rc;
  }
  return SHK_OK;
}

// The collectives the captured graphs hold, run once outside any capture:
// NCCL connects its peers on a communicator's first use of an algorithm, and
// with several GPUs in one process that enables peer access, which is not
// allowed while a stream captures.  The residual all-reduce runs in place on
// the hidden state, which every step's embedding overwrites.
int tp_warm(shk_model* m) {
  shk_ctx* c = m->ctx;
  if (!c->comm || c->tp_world < 2 || m->tp_warm) return SHK_OK;
  cudaStream_t st = c->compute;
  if (nccl()->all_reduce(m->hidden, m->hidden, m->d.n_embd, ncclFloat, ncclSum, c->comm, st) != ncclSuccess)
    return SHK_ENCCL;
  if (vocab_split(m) &&
      nccl()->all_gather(m->tp_pairs + 2 * c->tp_rank, m->tp_pairs, 2, ncclUint32, c->comm, st) != ncclSuccess)
    return SHK_ENCCL;
  CK(cudaStreamSynchronize(st));
  m->tp_warm = true;
  return SHK_OK;
}

int capture(shk_model* m, int which, cudaGraphExec_t* out) {
  cudaStream_t st = m->ctx->compute;
  cudaGraph_t g = nullptr;
  if (const int wr = tp_warm(m)) return wr;
  CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  // 0: embed + all layers;  1: lm_head + argmax;  2: both, argmax advancing *pos.
  // Every kernel after the first is a programmatic dependent launch: it is
  // scheduled while its predecessor drains and waits for it before its reads.
  const bool pdl = !(m->ctx->flags & SHK_CUDA_FLAG_NO_PDL);
  pdl_enabled() = false;
  int rc = which == 1 ? SHK_OK : enqueue_layers(m, st, pdl);
  if (!rc && which != 0) rc = enqueue_head(m, st, which == 2, pdl);
  pdl_enabled() = false;
  const cudaError_t ee = cudaStreamEndCapture(st, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ee != cudaSuccess) {
    fprintf(stderr, "shk_cuda: graph capture %d: %s\n", which, cudaGetErrorString(ee));
    return SHK_ECUDA;
  }
  const cudaError_t ie = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) fprintf(stderr, "shk_cuda: graph instantiate %d: %s\n", which, cudaGetErrorString(ie));
  return ie == cudaSuccess ? SHK_OK : SHK_ECUDA;
}

// Builds the persistent decode kernel's program: the layers' and the head's
// tensor-core matvec plans (row-tiled weights) with one common ring geometry,
// per-layer attention args and the phase list embed, [QKV, attention, O,
// gate/up, down] x L, lm_head, argmax.  Leaves state -1 (graph path) when the
// weights are not all tiled or the shapes do not fit it.
int build_persist(shk_model* m) {
  auto& k = m->pk;
  shk_ctx* c = m->ctx;
  const shk_model_desc& d = m->d;
  k.state = -1;
  if (!(c->flags & SHK_CUDA_FLAG_PERSISTENT) || !m->head.tiled || c->tp_world > 1) return SHK_OK;
  const uint32_t G = d.n_heads / d.n_kv_heads;
  if (d.n_heads % d.n_kv_heads) return SHK_OK;
  const uint32_t L = d.n_layers;
  std::vector<MmvArgs> ma;
  uint32_t slot = 0, kmax = 0;
  for (uint32_t l = 0; l < L; ++l) {
    const LayerPlans& P = m->plans[l];
    for (const ProjPlan* pp : {&P.qkv, &P.o, &P.gateup, &P.down}) {
      if (!pp->tiled || !pp->main || pp->has_q5) return SHK_OK;
      ma.push_back(pp->mm.args);
    }
  }
  ma.push_back(m->head.mm.args);
  for (const MmvArgs& a : ma) {
    slot = std::max(slot, a.stage_bytes);
    kmax = std::max(kmax, a.k);
    if ((int)a.grid > c->num_sms) return SHK_OK;
  }
  // one ring for every plan: the largest slot, then the largest chunk whose
  // stage count keeps the parity waits unambiguous
  DecodeProgram& P = k.P;
  P = DecodeProgram{};
  P.kmax = kmax;
  P.slot_bytes = slot;
  P.ns = 1;
  P.chunk = 1;
  size_t fixed = 0;
  decode_smem(P, d.head_dim, G, &fixed);
  const size_t budget = 227 * 1024;
  if (fixed >= budget) return SHK_OK;
  uint32_t chunk = MMV_MAX_CHUNK, ns = 0;
  for (;; chunk >>= 1) {
    if (chunk == 0) return SHK_OK;
    ns = (uint32_t)std::min<size_t>(MMV_MAX_STAGES, (budget - fixed) / ((size_t)chunk * slot));
    if (ns >= (MMV_WARPS + chunk - 1) / chunk + 2) break;
  }
  P.ns = ns;
  P.chunk = chunk;
  P.lg_chunk = (uint32_t)__builtin_ctz(chunk);
  for (MmvArgs& a : ma) {
    for (uint32_t i = 0; i < a.nseg; ++i)
      if (a.seg[i].ks + ns * chunk + MMV_WARPS + 1 >= a.red_slots) return SHK_OK;
    a.stage_bytes = slot;
    a.n_stages = ns;
    a.chunk = chunk;
    a.lg_chunk = P.lg_chunk;
  }
  k.smem = decode_smem(P, d.head_dim, G);
  k.grid = c->num_sms;
  if (!decode_supported(d.head_dim, G, k.smem, k.grid)) return SHK_OK;
  const uint32_t* pos = m->d_tok + 1;
  std::vector<AttnArgs> aa(L);
  for (uint32_t l = 0; l < L; ++l) aa[l] = layer_attn_args(m, l, pos);
  std::vector<DecodePhase> ph;
  ph.push_back({PH_EMBED, 0});
  for (uint32_t l = 0; l < L; ++l) {
    ph.push_back({PH_GEMV, 4 * l});
    ph.push_back({PH_ATTN, l});
    ph.push_back({PH_GEMV, 4 * l + 1});
    ph.push_back({PH_GEMV, 4 * l + 2});
    ph.push_back({PH_GEMV, 4 * l + 3});
  }
  ph.push_back({PH_GEMV, 4 * L});
  ph.push_back({PH_ARGMAX, 0});
  bool ok = cudaMalloc(&k.d_mmv, ma.size() * sizeof(MmvArgs)) == cudaSuccess;
  ok = ok && cudaMalloc(&k.d_attn, aa.size() * sizeof(AttnArgs)) == cudaSuccess;
  ok = ok && cudaMalloc(&k.d_phases, ph.size() * sizeof(DecodePhase)) == cudaSuccess;
  ok = ok && cudaMalloc(&k.d_bar, sizeof(uint32_t)) == cudaSuccess;
  ok = ok && cudaMemcpy(k.d_mmv, ma.data(), ma.size() * sizeof(MmvArgs), cudaMemcpyHostToDevice) == cudaSuccess;
  ok = ok && cudaMemcpy(k.d_attn, aa.data(), aa.size() * sizeof(AttnArgs), cudaMemcpyHostToDevice) == cudaSuccess;
  ok = ok && cudaMemcpy(k.d_phases, ph.data(), ph.size() * sizeof(DecodePhase), cudaMemcpyHostToDevice) == cudaSuccess;
  if (!ok) {
    model_free_graphs(m);
    m->pk.state = -1;
    return SHK_ENOMEM;
  }
  P.mmv = k.d_mmv;
  P.attn = k.d_attn;
  P.phases = k.d_phases;
  k.n_phases_full = (uint32_t)ph.size();
  P.tok_embd = static_cast<const uint8_t*>(d.tok_embd_dev);
  P.embd_dtype = d.tok_embd_dtype;
  P.n_vocab = d.n_vocab;
  P.n_embd = d.n_embd;
  P.hidden = m->hidden;
  P.logits = m->logits;
  P.am_v = m->am_v;
  P.am_i = m->am_i;
  P.am_cnt = m->am_cnt;
  P.tok = m->d_tok;
  P.n_kv = d.n_kv_heads;
  P.attn_nsplit = std::max<uint32_t>(1, std::min<uint32_t>(m->kv->max_splits, (uint32_t)k.grid / d.n_kv_heads));
  P.bar = k.d_bar;
  P.err = c->d_err;
  k.state = 1;
  return SHK_OK;
}

// One cooperative launch: n_steps tokens (with_head: lm_head + argmax per step).
int launch_persist(shk_model* m, uint32_t n_steps, bool with_head, bool advance_pos, cudaStream_t st) {
  auto& k = m->pk;
  DecodeProgram P = k.P;
  P.n_steps = n_steps;
  P.n_phases = with_head ? k.n_phases_full : k.n_phases_full - 2;
  P.advance_pos = advance_pos ? 1u : 0u;
  P.trace = m->d_trace;
  P.trace_cap_phases = m->trace_phases;
  m->trace_last = m->d_trace ? std::min<uint32_t>(m->trace_phases, n_steps * P.n_phases) : 0;
  CK(decode_launch(P, m->d.head_dim, m->d.n_heads / m->d.n_kv_heads, k.smem, k.grid, st));
  return SHK_OK;
}

bool model_ready(shk_model* m) {
  for (uint32_t l = 0; l < m->d.n_layers; ++l)
    if (!m->have[l] || !m->plans[l].ok) return false;
  return m->head_ok;
}

}  // namespace

shk_model* shk_cuda_model_create(shk_ctx* c, const shk_model_desc* d, shk_kv* kv) {
  if (c) on_dev(c);
  if (!c || !d || !kv) return nullptr;
  if (!d->n_layers || !d->n_embd || !d->n_heads || !d->n_kv_heads || !d->n_ff || !d->n_vocab)
    return nullptr;
  // (a tensor-parallel rank holds n_heads / world query heads: q width != n_embd)
  if ((c->tp_world == 1 && d->head_dim * d->n_heads != d->n_embd) || kv->L.hd != d->head_dim ||
      kv->L.n_kv != d->n_kv_heads || kv->L.n_layers != d->n_layers)
    return nullptr;
  shk_model* m = new (std::nothrow) shk_model();
  if (!m) return nullptr;
  m->ctx = c;
  m->d = *d;
  m->kv = kv;
  m->o_lo = 0;
  m->o_hi = d->n_embd;
  m->v_lo = 0;
  m->v_hi = d->n_vocab;
  const uint32_t qd = d->n_heads * d->head_dim, kvd = d->n_kv_heads * d->head_dim;
  bool ok = true;
  auto A = [&](float** p, size_t n) { ok = ok && cudaMalloc(p, n * sizeof(float)) == cudaSuccess; };
  A(&m->hidden, d->n_embd);
  A(&m->q, qd);
  A(&m->k, kvd);
  A(&m->v, kvd);
  A(&m->att, qd);
  A(&m->act, d->n_ff);
  A(&m->logits, d->n_vocab);
  A(&m->am_v, 256);
  ok = ok && cudaMalloc(&m->am_i, 256 * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && cudaMalloc(&m->am_cnt, sizeof(int)) == cudaSuccess;
  ok = ok && cudaMemset(m->am_cnt, 0, sizeof(int)) == cudaSuccess;
  ok = ok && cudaMalloc(&m->d_tok, 4 * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && cudaMemset(m->d_tok, 0, 4 * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && cudaMallocHost(&m->h_tok, 4 * sizeof(uint32_t)) == cudaSuccess;
  if (ok) ok = cudaMemset(m->hidden, 0, d->n_embd * sizeof(float)) == cudaSuccess;
  if (!ok) {
    shk_cuda_model_destroy(m);
    return nullptr;
  }
  m->layers.resize(d->n_layers);
  m->have.assign(d->n_layers, 0);
  m->plans.resize(d->n_layers);
  // GGUF-layout Q6_K (or rows the staged kernel cannot take): plain-load GEMV
  if (d->n_embd % QK || plan_head(m) != SHK_OK) {
    shk_cuda_model_destroy(m);
    return nullptr;
  }
  // RoPE frequencies with the host C library (engine/src/ops.c:223-227)
  std::vector<float> fr(d->head_dim / 2);
  rope_freq_table(d->rope_theta > 0.f ? d->rope_theta : 10000.0f, d->head_dim, fr.data());
  if (cudaMalloc(&m->d_freq, fr.size() * sizeof(float)) != cudaSuccess ||
      cudaMemcpy(m->d_freq, fr.data(), fr.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
    shk_cuda_model_destroy(m);
    return nullptr;
  }
  return m;
}

void shk_cuda_model_destroy(shk_model* m) {
  if (m) on_dev(m->ctx);
  if (!m) return;
  if (m->ctx) cudaStreamSynchronize(m->ctx->compute);
  model_free_graphs(m);
  cudaFree(m->hidden);
  cudaFree(m->q);
  cudaFree(m->k);
  cudaFree(m->v);
  cudaFree(m->att);
  cudaFree(m->act);
  cudaFree(m->logits);
  cudaFree(m->tp_pairs);
  for (int p = 0; p < GEMV_TP_MAX; ++p)
    if (m->p2p.opened[p]) cudaIpcCloseMemHandle(m->p2p.peer_base[p]);
  cudaFree(m->p2p.base);
  cudaFree(m->p2p.counters);
  cudaFree(m->p2p.d_step);
  for (int p = 0; p < LL_MAX_RANKS; ++p)
    if (m->ll.opened[p]) cudaIpcCloseMemHandle(m->ll.peer[p]);
  cudaFree(m->ll.base);
  cudaFree(m->ll.d_step);
  cudaFree(m->p2p.res2);
  cudaFree(m->am_v);
  cudaFree(m->am_i);
  cudaFree(m->am_cnt);
  cudaFree(m->d_tok);
  cudaFreeHost(m->h_tok);
  cudaFree(m->d_freq);
  cudaFree(m->d_trace);
  cudaFree(m->pf_buf);
  cudaFree(m->pf_tok);
  delete m;
}

float* shk_cuda_model_hidden(shk_model* m) { return m ? m->hidden : nullptr; }

int shk_cuda_model_set_layer(shk_model* m, uint32_t layer, const shk_layer_desc* lv) {
  if (m) on_dev(m->ctx);
  if (!m || !lv || layer >= m->d.n_layers) return SHK_EINVAL;
  LayerPlans P;
  const int rc = build_layer_plans(m, *lv, P, layer);
  if (rc) return rc;
  m->layers[layer] = *lv;
  m->plans[layer] = P;
  m->have[layer] = 1;
  model_free_graphs(m);
  return SHK_OK;
}

int shk_cuda_forward_layer(shk_model* m, const shk_layer_desc* lv, uint32_t layer, uint32_t pos,
                           float* hidden, void* s) {
  if (m) on_dev(m->ctx);
  if (!m || !lv || !hidden || layer >= m->d.n_layers || pos >= m->kv->L.max_seq) return SHK_EINVAL;
  cudaStream_t st = pick(m->ctx, s);
  if (m->p2p.on || m->ll.on) return SHK_EUNSUPPORTED;  // the exchanges run inside whole-token steps
  LayerPlans P;
  int rc = build_layer_plans(m, *lv, P, layer);
  if (rc) return rc;
  if (hidden != m->hidden) CK(cudaMemcpyAsync(m->hidden, hidden, m->d.n_embd * 4, cudaMemcpyDeviceToDevice, st));
  rc = enqueue_layer(m, P, layer, m->kv->d_iota + pos, st, false);
  pdl_enabled() = false;
  if (rc) return rc;
  if (hidden != m->hidden) CK(cudaMemcpyAsync(hidden, m->hidden, m->d.n_embd * 4, cudaMemcpyDeviceToDevice, st));
  m->kv->seq[layer] = std::max(m->kv->seq[layer], pos + 1);
  m->ctx->n_fwd++;
  return SHK_OK;
}

int shk_cuda_model_embed(shk_model* m, uint32_t token, void* s) {
  if (m) on_dev(m->ctx);
  if (!m) return SHK_EINVAL;
  if (token >= m->d.n_vocab) return SHK_EINVAL;
  cudaStream_t st = pick(m->ctx, s);
  CK(cudaStreamSynchronize(st));
  m->h_tok[0] = token;
  CK(cudaMemcpyAsync(m->d_tok, m->h_tok, 4, cudaMemcpyHostToDevice, st));
  CK(embed_launch(m->d.tok_embd_dev, m->d.tok_embd_dtype, m->d_tok, m->d.n_vocab, m->hidden,
                  m->d.n_embd, m->ctx->d_err, st));
  return SHK_OK;
}

int shk_cuda_model_lm_head(shk_model* m, uint32_t* token, float* logits, void* s) {
  if (m) on_dev(m->ctx);
  if (!m || !m->head_ok) return SHK_EINVAL;
  cudaStream_t st = pick(m->ctx, s);
  int rc = enqueue_head(m, st, false);
  if (rc) return rc;
  CK(cudaMemcpyAsync(m->h_tok + 2, m->d_tok, 4, cudaMemcpyDeviceToHost, st));
  if (logits && (rc = gather_logits(m, st))) return rc;
  if (logits) CK(cudaMemcpyAsync(logits, m->logits, (size_t)m->d.n_vocab * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  if (token) *token = m->h_tok[2];
  return ctx_err_check(m->ctx);
}

int shk_cuda_prefill(shk_model* m, const uint32_t* tokens, uint32_t n, uint32_t pos0, uint32_t* next,
                     float* logits, void* s) {
  if (m) on_dev(m->ctx);
  if (!m || !tokens || !n || (uint64_t)pos0 + n > m->kv->L.max_seq) return SHK_EINVAL;
  if (!model_ready(m)) return SHK_EINVAL;
  shk_ctx* c = m->ctx;
  if (c->tp_world > 1 || m->p2p.on || m->ll.on || n > 65535) return SHK_EUNSUPPORTED;
  const shk_model_desc& d = m->d;
  const uint32_t D = d.n_embd, hd = d.head_dim, qd = d.n_heads * hd, kvd = d.n_kv_heads * hd, F = d.n_ff;
  for (uint32_t i = 0; i < n; ++i)
    if (tokens[i] >= d.n_vocab) return SHK_EINVAL;
  // the tensor-core matmul takes Q4_K and planar Q6_K rows
  auto ok_dt = [](uint32_t t) { return t == (uint32_t)T_Q4K || t == (uint32_t)T_Q6K_PLANAR; };
  for (uint32_t l = 0; l < d.n_layers; ++l) {
    const shk_layer_desc& lv = m->layers[l];
    if (!ok_dt(lv.attn_q_dtype) || !ok_dt(lv.attn_k_dtype) || !ok_dt(lv.attn_v_dtype) ||
        !ok_dt(lv.attn_o_dtype) || !ok_dt(lv.ffn_gate_dtype) || !ok_dt(lv.ffn_up_dtype) ||
        !ok_dt(lv.ffn_down_dtype))
      return SHK_EUNSUPPORTED;
  }
  cudaStream_t st = pick(c, s);
  const size_t per = 2 * (size_t)D + qd + 2 * (size_t)kvd + qd + D + 3 * (size_t)F;  // floats per row
  int rc;
  if ((rc = grow(&m->pf_buf, &m->pf_cap, per * n * sizeof(float))) ||
      (rc = grow(&m->pf_tok, &m->pf_tok_cap, (size_t)n * sizeof(uint32_t))) ||
      (rc = grow(&c->pf_x, &c->pf_x_cap, prefill_x_bytes(std::max(std::max(D, qd), F), n))))
    return rc;
  float* X = m->pf_buf;
  float* Xn = X + (size_t)n * D;
  float* Q = Xn + (size_t)n * D;
  float* K = Q + (size_t)n * qd;
  float* V = K + (size_t)n * kvd;
  float* A = V + (size_t)n * kvd;
  float* P = A + (size_t)n * qd;
  float* G = P + (size_t)n * D;
  float* U = G + (size_t)n * F;
  float* H = U + (size_t)n * F;
  CK(cudaMemcpyAsync(m->pf_tok, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, st));
  for (uint32_t t = 0; t < n; ++t)
    CK(embed_launch(d.tok_embd_dev, d.tok_embd_dtype, m->pf_tok + t, d.n_vocab, X + (size_t)t * D, D, c->d_err, st));
  auto mm = [&](uint32_t dt, const void* w, uint32_t stride, const float* x, float* y, uint32_t rows,
                uint32_t k) -> cudaError_t {
    const uint32_t dense = (k / QK) * (dt == (uint32_t)T_Q4K ? Q4K_BYTES : Q6K_BYTES);
    return prefill_launch(dt, w, stride ? stride : dense, x, c->pf_x, y, rows, k, n, c->d_err, c->num_sms, st);
  };
  for (uint32_t l = 0; l < d.n_layers; ++l) {
    const shk_layer_desc& lv = m->layers[l];
    // attention block (engine/src/engine.c:105-167), T rows at a time
    CK(rmsnorm_rows_launch(X, lv.attn_norm, Xn, D, n, st));
    CK(mm(lv.attn_q_dtype, lv.attn_q, 0, Xn, Q, qd, D));
    CK(mm(lv.attn_k_dtype, lv.attn_k, 0, Xn, K, kvd, D));
    CK(mm(lv.attn_v_dtype, lv.attn_v, lv.row_stride_v, Xn, V, kvd, D));
    CK(rope_rows_launch(Q, d.n_heads, hd, pos0, n, m->d_freq, st));
    CK(rope_rows_launch(K, d.n_kv_heads, hd, pos0, n, m->d_freq, st));
    CK(kv_append_range_launch(m->kv->L, l, pos0, n, K, V, st));
    AttnArgs a = layer_attn_args(m, l, nullptr);
    a.q = Q;
    a.out = A;
    CK(attn_prefill_launch(a, m->kv->d_iota, pos0, n, st));
    CK(mm(lv.attn_o_dtype, lv.attn_o, 0, A, P, D, qd));
    CK(add_launch(X, P, n * D, st));
    // FFN block (engine/src/engine.c:170-221)
    CK(rmsnorm_rows_launch(X, lv.ffn_norm, Xn, D, n, st));
    CK(mm(lv.ffn_gate_dtype, lv.ffn_gate, 0, Xn, G, F, D));
    CK(mm(lv.ffn_up_dtype, lv.ffn_up, 0, Xn, U, F, D));
    CK(swiglu_launch(G, U, H, n * F, st));
    CK(mm(lv.ffn_down_dtype, lv.ffn_down, lv.row_stride_down, H, P, D, F));
    CK(add_launch(X, P, n * D, st));
  }
  for (uint32_t l = 0; l < d.n_layers; ++l) m->kv->seq[l] = std::max(m->kv->seq[l], pos0 + n);
  // the last row is the hidden state the output head reads
  CK(cudaMemcpyAsync(m->hidden, X + (size_t)(n - 1) * D, (size_t)D * 4, cudaMemcpyDeviceToDevice, st));
  return shk_cuda_model_lm_head(m, next, logits, s);
}

int shk_cuda_token_step(shk_model* m, uint32_t token, uint32_t pos, int want_next, uint32_t* next,
                        float* logits) {
  if (m) on_dev(m->ctx);
  if (!m || token >= m->d.n_vocab || pos >= m->kv->L.max_seq) return SHK_EINVAL;
  if (!model_ready(m)) return SHK_EINVAL;
  cudaStream_t st = m->ctx->compute;
  int rc;
  if (m->pk.state == 0 && (rc = build_persist(m))) return rc;
  const bool persist = m->pk.state == 1;
  if (!persist) {
    if (!m->g_layers && (rc = capture(m, 0, &m->g_layers))) return rc;
    if (!m->g_head && (rc = capture(m, 1, &m->g_head))) return rc;
  }
  CK(cudaStreamSynchronize(st));  // h_tok is reused below
  m->h_tok[0] = token;
  m->h_tok[1] = pos;
  CK(cudaMemcpyAsync(m->d_tok, m->h_tok, 8, cudaMemcpyHostToDevice, st));
  if (persist) {
    if ((rc = launch_persist(m, 1, want_next != 0, false, st))) return rc;
  } else {
    CK(cudaGraphLaunch(m->g_layers, st));
    if (want_next) CK(cudaGraphLaunch(m->g_head, st));
  }
  if (want_next) {
    CK(cudaMemcpyAsync(m->h_tok + 2, m->d_tok, 4, cudaMemcpyDeviceToHost, st));
    if (logits && (rc = gather_logits(m, st))) return rc;
    if (logits) CK(cudaMemcpyAsync(logits, m->logits, (size_t)m->d.n_vocab * 4, cudaMemcpyDeviceToHost, st));
  }
  // the step's device error word comes back with the token: one stream sync
  CK(cudaMemcpyAsync(m->ctx->h_err, m->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  for (uint32_t l = 0; l < m->d.n_layers; ++l) m->kv->seq[l] = std::max(m->kv->seq[l], pos + 1);
  m->ctx->n_steps++;
  rc = ctx_err_take(m->ctx, *m->ctx->h_err);
  if (rc) return rc;
  if (want_next && next) *next = m->h_tok[2];
  return SHK_OK;
}

int shk_cuda_decode_steps(shk_model* m, uint32_t first_token, uint32_t first_pos, uint32_t n,
                          void* s) {
  if (m) on_dev(m->ctx);
  if (!m || first_token >= m->d.n_vocab || (uint64_t)first_pos + n > m->kv->L.max_seq) return SHK_EINVAL;
  if (!model_ready(m)) return SHK_EINVAL;
  cudaStream_t st = pick(m->ctx, s);
  int rc;
  if (m->pk.state == 0 && (rc = build_persist(m))) return rc;
  const bool persist = m->pk.state == 1;
  CK(cudaStreamSynchronize(st));
  m->h_tok[0] = first_token;
  m->h_tok[1] = first_pos;
  CK(cudaMemcpyAsync(m->d_tok, m->h_tok, 8, cudaMemcpyHostToDevice, st));
  // Each step: embed(*tok) + layers at *pos, then lm_head + argmax writes the
  // next token and advances *pos.  No host round trip between steps.
  if (persist) {
    if (n && (rc = launch_persist(m, n, true, true, st))) return rc;
  } else {
    if (!m->g_loop && (rc = capture(m, 2, &m->g_loop))) return rc;
    for (uint32_t i = 0; i < n; ++i) CK(cudaGraphLaunch(m->g_loop, st));
  }
  for (uint32_t l = 0; l < m->d.n_layers; ++l)
    m->kv->seq[l] = std::max(m->kv->seq[l], first_pos + n);
  m->ctx->n_steps += n;
  return SHK_OK;
}

int shk_cuda_selftest_wait_timeout(shk_ctx* c, uint32_t budget_us) {
  if (c) on_dev(c);
  if (!c || budget_us == 0 || budget_us > 1000000u) return SHK_EINVAL;
  CK(wait_selftest_launch(c->d_err, 1000ull * budget_us, c->compute));
  return ctx_err_check(c);
}

int shk_cuda_tp_unique_id(void* out, size_t cap) {
  if (!out || cap < sizeof(ncclUniqueId)) return SHK_EINVAL;
  if (!nccl()) return SHK_EUNSUPPORTED;
  ncclUniqueId id;
  if (nccl()->get_unique_id(&id) != ncclSuccess) return SHK_ENCCL;
  memcpy(out, &id, sizeof(id));
  return (int)sizeof(id);
}

int shk_cuda_tp_init(shk_ctx* c, int rank, int world, const void* id) {
  if (c) on_dev(c);
  if (!c || !id || world < 1 || rank < 0 || rank >= world || c->comm) return SHK_EINVAL;
  if (world == 1) return SHK_OK;
  if (!nccl()) return SHK_EUNSUPPORTED;
  cudaSetDevice(c->device);
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  if (nccl()->comm_init_rank(&c->comm, world, uid, rank) != ncclSuccess) {
    c->comm = nullptr;
    return SHK_ENCCL;
  }
  c->tp_rank = rank;
  c->tp_world = world;
  return SHK_OK;
}

int shk_cuda_tp_comm_size(shk_ctx* c) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  if (!c->comm) return 1;
  int n = 0;
  if (nccl()->comm_count(c->comm, &n) != ncclSuccess) return SHK_ENCCL;
  return n;
}

int shk_cuda_model_set_tp_rows(shk_model* m, uint32_t o_lo, uint32_t o_hi, uint32_t v_lo, uint32_t v_hi) {
  if (m) on_dev(m->ctx);
  if (!m || o_lo >= o_hi || o_hi > m->d.n_embd || v_lo >= v_hi || v_hi > m->d.n_vocab) return SHK_EINVAL;
  for (uint32_t l = 0; l < m->d.n_layers; ++l)
    if (m->have[l]) return SHK_EINVAL;  // before any layer is registered
  if (m->g_layers || m->g_head || m->g_loop || m->p2p.on) return SHK_EINVAL;  // graphs / exchange set up
  shk_ctx* c = m->ctx;
  const uint32_t nv = v_hi - v_lo;
  if (nv < m->d.n_vocab) {  // equal slices in rank order (the gathers need equal counts)
    if (c->tp_world < 2 || (uint64_t)nv * c->tp_world != m->d.n_vocab || v_lo != nv * (uint32_t)c->tp_rank)
      return SHK_EINVAL;
    if (!m->tp_pairs && cudaMalloc(&m->tp_pairs, 2 * sizeof(uint32_t) * c->tp_world) != cudaSuccess)
      return SHK_ENOMEM;
  }
  const uint32_t ov_lo = m->v_lo, ov_hi = m->v_hi;
  m->v_lo = v_lo;
  m->v_hi = v_hi;
  const int rc = plan_head(m);
  if (rc) {
    m->v_lo = ov_lo;
    m->v_hi = ov_hi;
    return rc;
  }
  m->o_lo = o_lo;
  m->o_hi = o_hi;
  return SHK_OK;
}

int shk_cuda_model_tp_p2p_export(shk_model* m, void* handle_out, size_t cap) {
  if (m) on_dev(m->ctx);
  if (!m || !handle_out || cap < sizeof(cudaIpcMemHandle_t)) return SHK_EINVAL;
  shk_ctx* c = m->ctx;
  if (c->tp_world < 2 || c->tp_world > GEMV_TP_MAX) return SHK_EINVAL;
  auto& q = m->p2p;
  cudaSetDevice(c->device);
  if (!q.base) {
    const size_t W = (size_t)c->tp_world, D = m->d.n_embd, NS = 2 * (size_t)m->d.n_layers;
    q.flag_bytes = (NS * W * 4 + 255) & ~(size_t)255;
    q.bytes = q.flag_bytes + NS * W * D * 4;
    if (cudaMalloc(&q.base, q.bytes) != cudaSuccess || cudaMalloc(&q.counters, NS * 4) != cudaSuccess ||
        cudaMalloc(&q.d_step, 4) != cudaSuccess || cudaMalloc(&q.res2, D * 4) != cudaSuccess)
      return SHK_ENOMEM;
    CK(cudaMemset(q.base, 0, q.bytes));
    CK(cudaMemset(q.counters, 0, NS * 4));
    CK(cudaMemset(q.d_step, 0, 4));
    CK(cudaMemset(q.res2, 0, D * 4));
  }
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, q.base));
  memcpy(handle_out, &h, sizeof(h));
  return (int)sizeof(h);
}

int shk_cuda_model_tp_ll_export(shk_model* m, void* handle_out, size_t cap) {
  if (m) on_dev(m->ctx);
  if (!m || !handle_out || cap < sizeof(cudaIpcMemHandle_t)) return SHK_EINVAL;
  shk_ctx* c = m->ctx;
  if (c->tp_world < 2 || c->tp_world > LL_MAX_RANKS || m->p2p.on) return SHK_EINVAL;
  auto& q = m->ll;
  cudaSetDevice(c->device);
  if (!q.base) {
    q.bytes = ll_buffer_bytes(2 * m->d.n_layers, (uint32_t)c->tp_world, m->d.n_embd);
    if (cudaMalloc(&q.base, q.bytes) != cudaSuccess || cudaMalloc(&q.d_step, 4) != cudaSuccess) return SHK_ENOMEM;
    CK(cudaMemset(q.base, 0, q.bytes));
    CK(cudaMemset(q.d_step, 0, 4));
  }
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, q.base));
  memcpy(handle_out, &h, sizeof(h));
  return (int)sizeof(h);
}

int shk_cuda_model_tp_ll_import(shk_model* m, const void* handles) {
  if (m) on_dev(m->ctx);
  if (!m || !handles) return SHK_EINVAL;
  shk_ctx* c = m->ctx;
  auto& q = m->ll;
  if (!q.base || q.on || m->g_layers || m->g_head || m->g_loop) return SHK_EINVAL;
  cudaSetDevice(c->device);
  for (int p = 0; p < c->tp_world; ++p) {
    if (p == c->tp_rank) {
      q.peer[p] = q.base;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)p * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return SHK_ECUDA;
    q.peer[p] = ptr;
    q.opened[p] = true;
  }
  q.on = true;
  return SHK_OK;
}

int shk_cuda_model_tp_p2p_import(shk_model* m, const void* handles, const uint32_t* o_ranges) {
  if (m) on_dev(m->ctx);
  if (!m || !handles || !o_ranges) return SHK_EINVAL;
  shk_ctx* c = m->ctx;
  auto& q = m->p2p;
  if (!q.base || q.on || m->g_layers || m->g_head || m->g_loop) return SHK_EINVAL;
  for (uint32_t l = 0; l < m->d.n_layers; ++l)
    if (m->have[l]) return SHK_EINVAL;  // before any layer is registered
  cudaSetDevice(c->device);
  const int W = c->tp_world;
  for (int p = 0; p < W; ++p) {
    if (o_ranges[2 * p] >= o_ranges[2 * p + 1] || o_ranges[2 * p + 1] > m->d.n_embd ||
        o_ranges[2 * p] % 8 || o_ranges[2 * p + 1] % 8)
      return SHK_EINVAL;
    q.cov_lo[p] = o_ranges[2 * p];
    q.cov_hi[p] = o_ranges[2 * p + 1];
    if (p == c->tp_rank) {
      q.peer_base[p] = q.base;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)p * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return SHK_ECUDA;
    q.peer_base[p] = ptr;
    q.opened[p] = true;
  }
  q.on = true;
  const int rc = plan_head(m);
  if (rc) q.on = false;
  return rc;
}

int shk_cuda_model_trace_enable(shk_model* m, uint32_t n_phases) {
  if (m) on_dev(m->ctx);
  if (!m) return SHK_EINVAL;
  CK(cudaStreamSynchronize(m->ctx->compute));
  cudaFree(m->d_trace);
  m->d_trace = nullptr;
  m->trace_phases = 0;
  m->trace_last = 0;
  if (n_phases == 0) return SHK_OK;
  if (cudaMalloc(&m->d_trace, (1 + 2 * (size_t)n_phases) * sizeof(uint64_t)) != cudaSuccess) {
    m->d_trace = nullptr;
    return SHK_ENOMEM;
  }
  m->trace_phases = n_phases;
  return SHK_OK;
}

int shk_cuda_model_trace_read(shk_model* m, uint64_t* out, uint32_t cap) {
  if (m) on_dev(m->ctx);
  if (!m || !out) return SHK_EINVAL;
  if (!m->d_trace || m->trace_last == 0) return 0;
  const uint32_t n = std::min<uint32_t>(cap, 1 + 2 * m->trace_last);
  CK(cudaStreamSynchronize(m->ctx->compute));
  CK(cudaMemcpy(out, m->d_trace, (size_t)n * sizeof(uint64_t), cudaMemcpyDeviceToHost));
  return (int)n;
}

int shk_cuda_model_token(shk_model* m, uint32_t* token) {
  if (m) on_dev(m->ctx);
  if (!m || !token) return SHK_EINVAL;
  CK(cudaMemcpyAsync(m->h_tok + 2, m->d_tok, 4, cudaMemcpyDeviceToHost, m->ctx->compute));
  CK(cudaStreamSynchronize(m->ctx->compute));
  *token = m->h_tok[2];
  return ctx_err_check(m->ctx);
}

int shk_cuda_model_launch_part(shk_model* m, uint32_t layer, uint32_t part, void* s,
                               uint64_t* bytes_out) {
  if (m) on_dev(m->ctx);
  if (!m || part > 5 || (part < 5 && (layer >= m->d.n_layers || !m->have[layer] || !m->plans[layer].ok)))
    return SHK_EINVAL;
  if (m->p2p.on) return SHK_EUNSUPPORTED;  // parts wait on peers' partials
  cudaStream_t st = pick(m->ctx, s);
  uint64_t bytes = 0;
  if (part == 5) {
    if (!m->head_ok || m->head_generic) return SHK_EINVAL;
    CK(proj_launch(m->head, st));
    bytes = proj_weight_bytes(m->head);
  } else if (part == 1) {
    AttnArgs a{};
    a.kv = m->kv->L;
    a.layer = layer;
    a.n_heads = m->d.n_heads;
    a.scale = 1.0f / sqrtf((float)m->d.head_dim);
    a.q = m->q;
    a.k_new = nullptr;  // read-only: attend over [0, *pos] without appending
    a.v_new = nullptr;
    a.pos = m->d_tok + 1;
    a.out = m->att;
    a.part = m->kv->part;
    a.counters = m->kv->counters;
    a.max_splits = m->kv->max_splits;
    a.min_per_split = SHK_ATT_MIN_SPLIT;
    a.err = m->ctx->d_err;
    CK(attn_decode_launch(a, st));
  } else {
    const LayerPlans& P = m->plans[layer];
    const ProjPlan* p = part == 0 ? &P.qkv : part == 2 ? &P.o : part == 3 ? &P.gateup : &P.down;
    CK(proj_launch(*p, st));
    bytes = proj_weight_bytes(*p);
  }
  if (bytes_out) *bytes_out = bytes;
  return SHK_OK;
}

// ------------------------------- staging ---------------------------------------

static cudaEvent_t slot_event(shk_ctx* c, uint32_t slot) {
  std::lock_guard<std::mutex> g(c->stage_mu);
  auto it = c->slot_ev.find(slot);
  if (it != c->slot_ev.end()) return it->second;
  cudaEvent_t e = nullptr;
  if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
  c->slot_ev[slot] = e;
  return e;
}

// Before the first copy into a released slot, the copy stream waits for the
// work the release recorded (kernels still reading the slot's old contents).
static int stage_prepare(shk_ctx* c, uint32_t slot) {
  cudaSetDevice(c->device);  // may run on the loader thread
  std::lock_guard<std::mutex> g(c->stage_mu);
  auto it = c->rel_pending.find(slot);
  if (it != c->rel_pending.end() && it->second) {
    it->second = false;
    CK(cudaStreamWaitEvent(c->copy, c->rel_ev[slot], 0));
  }
  return SHK_OK;
}

int shk_cuda_layer_release(shk_ctx* c, uint32_t slot, void* s) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  cudaSetDevice(c->device);
  cudaStream_t st = pick(c, s);
  std::lock_guard<std::mutex> g(c->stage_mu);
  cudaEvent_t& e = c->rel_ev[slot];
  if (!e && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
    e = nullptr;
    return SHK_ECUDA;
  }
  CK(cudaEventRecord(e, st));
  c->rel_pending[slot] = true;
  return SHK_OK;
}

int shk_cuda_layer_stage(shk_ctx* c, uint32_t slot, void* dst, const void* src, size_t bytes) {
  if (c) on_dev(c);
  if (!c || !dst || !src) return SHK_EINVAL;
  const int rc = stage_prepare(c, slot);
  if (rc) return rc;
  CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->copy));
  {
    std::lock_guard<std::mutex> g(c->stage_mu);
    c->n_staged++;
    c->bytes_staged += bytes;
  }
  return SHK_OK;
}

int shk_cuda_layer_stage_rows(shk_ctx* c, uint32_t slot, void* dst, size_t dst_row,
                              const void* src, size_t src_row, size_t rows) {
  if (c) on_dev(c);
  if (!c || !dst || !src || dst_row < src_row) return SHK_EINVAL;
  const int rc = stage_prepare(c, slot);
  if (rc) return rc;
  CK(cudaMemcpy2DAsync(dst, dst_row, src, src_row, src_row, rows, cudaMemcpyHostToDevice, c->copy));
  {
    std::lock_guard<std::mutex> g(c->stage_mu);
    c->n_staged++;
    c->bytes_staged += src_row * rows;
  }
  return SHK_OK;
}

int shk_cuda_layer_stage_2d(shk_ctx* c, uint32_t slot, void* dst, size_t dst_pitch, const void* src,
                            size_t src_pitch, size_t width, size_t rows) {
  if (c) on_dev(c);
  if (!c || !dst || !src || width > dst_pitch || width > src_pitch) return SHK_EINVAL;
  if (!width || !rows) return SHK_OK;
  const int rc = stage_prepare(c, slot);
  if (rc) return rc;
  CK(cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width, rows, cudaMemcpyHostToDevice, c->copy));
  {
    std::lock_guard<std::mutex> g(c->stage_mu);
    c->n_staged++;
    c->bytes_staged += width * rows;
  }
  return SHK_OK;
}

int shk_cuda_layer_stage_q6k_planar(shk_ctx* c, uint32_t slot, void* dst, uint32_t rows, uint32_t k,
                                    uint32_t row_stride) {
  if (c) on_dev(c);
  if (!c || !dst || k == 0 || k % QK) return SHK_EINVAL;
  (void)slot;  // same copy stream as the slot's copies: ordered after them, covered by its commit
  const uint32_t stride = row_stride ? row_stride : 210u * (k / QK);
  if (stride % 16 || stride < 210u * (k / QK) || stride > 227u * 1024u || (reinterpret_cast<uintptr_t>(dst) & 15))
    return SHK_EINVAL;
  cudaSetDevice(c->device);
  CK(q6k_repack_launch(dst, rows, k, stride, true, c->num_sms, c->copy));
  return SHK_OK;
}

int shk_cuda_layer_commit(shk_ctx* c, uint32_t slot) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  cudaSetDevice(c->device);
  cudaEvent_t e = slot_event(c, slot);
  if (!e) return SHK_ECUDA;
  CK(cudaEventRecord(e, c->copy));
  return SHK_OK;
}

int shk_cuda_layer_ready(shk_ctx* c, uint32_t slot, int wait) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  cudaSetDevice(c->device);
  cudaEvent_t e = slot_event(c, slot);
  if (!e) return SHK_ECUDA;
  if (wait) {
    CK(cudaEventSynchronize(e));
    return 1;
  }
  const cudaError_t q = cudaEventQuery(e);
  if (q == cudaSuccess) return 1;
  if (q == cudaErrorNotReady) return 0;
  return SHK_ECUDA;
}

int shk_cuda_layer_wait(shk_ctx* c, uint32_t slot, void* s) {
  if (c) on_dev(c);
  if (!c) return SHK_EINVAL;
  cudaEvent_t e = slot_event(c, slot);
  if (!e) return SHK_ECUDA;
  CK(cudaStreamWaitEvent(pick(c, s), e, 0));
  return SHK_OK;
}

}  // extern "C"
