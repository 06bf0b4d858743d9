// Host runtime of the B200 decoder: handle, weight upload (with the Q8_0
// quantiser of linear.rs:194-202), paged KV pool, per-pass plans, the forward
// pass, the continuous-batching engine loop with CUDA-graph replay, and the
// extern "C" entry points declared in include/fmd_decoder.h.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/fmd_decoder.h"
#include "fmd_kernels.cuh"
#include "fmd_scheduler.cuh"
#include "fmd_watch.h"

namespace fmd {
cudaError_t init_kernels();
}

using namespace fmd;

namespace {

constexpr int kVersion = 1;
constexpr int kMaxSlotsLimit = 256;
constexpr int kEngineCheckEvery = 16;
constexpr int kEngineIdlePolls = 4;  // polls without progress before FMD_ETIMEDOUT

struct Status {
  int code;
  std::string msg;
};

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
};

struct LayerDev {
  void* in_norm = nullptr;
  void* post_norm = nullptr;
  void* q_norm = nullptr;
  void* k_norm = nullptr;
  LinW qkv, o, gate_up, down;
  TcLinear tc_qkv, tc_o, tc_gate_up, tc_down;  // the same projections for mixed steps (tcgen05)
};

uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&b);
}
uint16_t f32_to_f16_bits(float f) {
  __half h = __float2half_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}
float bf16_bits_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
float f16_bits_to_f32(uint16_t b) {
  __half h = *reinterpret_cast<__half*>(&b);
  return __half2float(h);
}

// GGML Q8_0 quantisation of one row-major (rows, cols) f32 matrix into the
// structure-of-arrays device layout (int8 [rows][cols] + f16 [rows][cols/32]).
// d = amax/127; id = 1/d (0 if d == 0); q = roundf(x * id) (half away from 0).
void quantize_rows(const float* src, int64_t rows, int64_t cols, int8_t* qs, uint16_t* d) {
  auto work = [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) {
      for (int64_t b = 0; b < cols / 32; ++b) {
        const float* x = src + r * cols + b * 32;
        float amax = 0.f;
        for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(x[j]));
        const float dd = amax / 127.f;
        const float id = dd != 0.f ? 1.f / dd : 0.f;
        d[r * (cols / 32) + b] = f32_to_f16_bits(dd);
        for (int j = 0; j < 32; ++j) qs[r * cols + b * 32 + j] = (int8_t)std::roundf(x[j] * id);
      }
    }
  };
  const int64_t nt = std::max<int64_t>(1, std::min<int64_t>(std::thread::hardware_concurrency(), rows / 256));
  std::vector<std::thread> th;
  for (int64_t i = 0; i < nt; ++i) th.emplace_back(work, rows * i / nt, rows * (i + 1) / nt);
  for (auto& t : th) t.join();
}

}  // namespace

struct fmd_handle {
  fmd_config cfg{};
  int precision = 0;
  bool q8 = false;
  ActType at = kBF16;
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string err;
  std::vector<DevBuf> allocs;
  int64_t weight_bytes = 0, kv_bytes = 0, work_bytes = 0;

  // model
  bool loaded = false;
  void* embed = nullptr;
  void* final_norm = nullptr;
  LinW lm_head;
  std::vector<LayerDev> layers;
  void* rope_cos = nullptr;
  void* rope_sin = nullptr;
  int rope_len = 0;
  float attn_scale = 0.f;

  // kv pool + work buffers
  bool reserved = false;
  int max_slots = 0, max_rows = 0, n_pages = 0, max_pages_per_slot = 0;
  int pb_max = 0, di_max = 0, di_grid = 0;
  KvView kv{};
  alignas(64) CUtensorMap kv_tmap;  // the KV pool as [rows][128] for TMA tile loads
  // activation operands of the mixed-step tensor-core projections
  alignas(64) CUtensorMap amap_xn, amap_ctx, amap_hbuf;
  alignas(64) CUtensorMap qmap;  // the query buffer as [rows][Hq x 128] (prefill attention tiles)
  bool q_ready = false;
  bool tc_ready = false;
  void* tmap_encode = nullptr;      // cuTensorMapEncodeTiled
  int* attn_counters = nullptr;     // [max_slots][kv_heads] split-KV merge counters
  // persistent layer tail (fmd_chain.cu) of decode steps: Q8_0 weights and
  // at most kChainMaxRows rows, opt-in with FMD_LAYER_TAIL=1 in the
  // environment at fmd_create.
  int n_sm = 0;
  bool proj_allowed = true;  // mixed steps on k_proj_tc (fused epilogues); FMD_PROJ_TC=0 selects k_gemm_tc
  bool lm_tc_allowed = false;  // Q8_0 lm_head on the tensor cores (FMD_LM_HEAD_TC=1); else the mma.sync kernel
  bool lm_f16_allowed = true;  // mma.sync lm_head: f16 operands for Q8_0 with bf16 rows (FMD_LM_HEAD_F16=0: bf16)
  bool lm_tc_used = false;     // the last lm_head launch (or graph capture) used the tensor-core kernel
  bool pf_pp_allowed = true;  // persistent two-tile prefill attention; FMD_PREFILL_PP=0 selects one CTA per block
  bool chain_allowed = false;
  bool chain_ok = false;
  size_t chain_smem = 0;
  int chain_clusters = 0;
  int* chain_sync = nullptr;        // [layers][kChainSyncInts], cleared by each decode step's first kernel
  int* d_status = nullptr;          // device-side error status (bounded waits)
  bool launch_refused = false;      // a decode projection could not be launched
  int* d_page_table = nullptr;
  std::vector<int> h_page_table;
  std::vector<int> free_pages;           // host allocator (operator mode)
  std::vector<int> slot_cap, slot_len, slot_npages;
  void *x = nullptr, *xn = nullptr, *qbuf = nullptr, *ctx = nullptr, *hbuf = nullptr, *arena = nullptr;
  float *part = nullptr, *pacc = nullptr, *pml = nullptr, *logits = nullptr;
  // decode-only steps split over two streams (FMD_DECODE_SPLIT=1): rows
  // [0, max_slots / 2) on `stream`, the rest on `stream2`, so that one half's
  // latency-bound projections overlap the other half's attention
  bool split_allowed = false;
  bool split_ok = false;
  cudaStream_t stream2 = nullptr;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
  PlanCounts* half_counts = nullptr;  // [2]
  float *pacc2 = nullptr, *pml2 = nullptr;
  float* ssq = nullptr;       // [max_slots][hidden / 64] per-tile sums of squares of the residual stream
  float* best_val = nullptr;  // [max_slots][vocab / 64] greedy candidates of the decode path
  int* best_idx = nullptr;
  size_t split_stride = 0;
  int* next_ids = nullptr;
  PlanLayout layout{};
  int* d_plan = nullptr;
  int* h_plan = nullptr;  // pinned mirror
  Plan plan{};
  int64_t arena_rows = 0;

  // engine
  DevBuf eng_reqs, eng_arena, eng_tokens, eng_results;
  DevBuf splice_src;  // per-position source codes of fmd_splice_audio
  int eng_n_reqs = 0, eng_tok_stride = 0;
  int* eng_slot = nullptr;  // 7 arrays of max_slots
  int* eng_free = nullptr;
  EngineCounters* eng_ctr = nullptr;
  EngineCounters* h_ctr = nullptr;
  cudaGraphExec_t graph_exec = nullptr;  // engine step that may carry a prefill chunk ("M")
  cudaGraphExec_t graph_dec = nullptr;   // decode-only engine step ("D")
  int graph_batch = -1, graph_chunk = -1;
  int64_t graph_kernels_mixed = 0, graph_kernels_decode = 0;
  bool first_block = true;               // no counters polled since fmd_engine_start
  int64_t launched_mixed = 0;
  bool engine_started = false;
  ProgressWatch watch{kEngineIdlePolls};  // polls without progress, over every fmd_engine_step call since the start
  bool record_attn_events = false;             // set while capturing the step graph
  // around the decode attention of one layer only: an event node between two
  // kernels of the graph removes their programmatic-dependent-launch overlap
  std::vector<cudaEvent_t> attn_events;        // [4]: the probe layer's attention, then the lm_head
  int attn_probe_layer() const { return cfg.num_hidden_layers / 2; }
  cudaEvent_t win_begin = nullptr, win_end = nullptr;

  int elem() const { return 2; }
  int H() const { return cfg.hidden_size; }
  int Hq() const { return cfg.num_attention_heads; }
  int Hkv() const { return cfg.num_key_value_heads; }
  int qkvN() const { return (Hq() + 2 * Hkv()) * kHeadDim; }
};

namespace {

int fail(fmd_handle* h, int code, const std::string& msg) {
  if (h) h->err = msg;
  return code;
}

#define CK(call)                                                                                         \
  do {                                                                                                   \
    cudaError_t e_ = (call);                                                                             \
    if (e_ != cudaSuccess)                                                                               \
      return fail(h, e_ == cudaErrorMemoryAllocation ? FMD_ENOMEM : FMD_EIO,                              \
                  std::string(#call) + ": " + cudaGetErrorString(e_));                                    \
  } while (0)

int dev_alloc(fmd_handle* h, size_t bytes, void** out, int64_t* counter) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(h, FMD_ENOMEM, "cudaMalloc of " + std::to_string(bytes) + " bytes failed: " + cudaGetErrorString(e));
  }
  h->allocs.push_back({p, bytes});
  if (counter) *counter += (int64_t)bytes;
  *out = p;
  return FMD_OK;
}

int upload(fmd_handle* h, void* dst, const void* src, size_t bytes) {
  CK(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
  return FMD_OK;
}

// Host tensor -> f32 vector
bool to_f32(const fmd_tensor& t, size_t n, std::vector<float>& out) {
  out.resize(n);
  if (t.data == nullptr) return false;
  switch (t.dtype) {
    case FMD_DT_F32: std::memcpy(out.data(), t.data, n * 4); return true;
    case FMD_DT_BF16: {
      const uint16_t* s = (const uint16_t*)t.data;
      for (size_t i = 0; i < n; ++i) out[i] = bf16_bits_to_f32(s[i]);
      return true;
    }
    case FMD_DT_F16: {
      const uint16_t* s = (const uint16_t*)t.data;
      for (size_t i = 0; i < n; ++i) out[i] = f16_bits_to_f32(s[i]);
      return true;
    }
    default: return false;
  }
}

// Dense host tensor -> activation dtype on the device.
int upload_dense(fmd_handle* h, const fmd_tensor& t, size_t n, void** out, const char* what) {
  if (t.data == nullptr) return fail(h, FMD_EINVAL, std::string("missing tensor ") + what);
  if (t.dtype == FMD_DT_Q8_0) return fail(h, FMD_EINVAL, std::string(what) + " must be dense");
  std::vector<uint16_t> bits(n);
  const bool bf = h->at == kBF16;
  if ((bf && t.dtype == FMD_DT_BF16) || (!bf && t.dtype == FMD_DT_F16)) {
    std::memcpy(bits.data(), t.data, n * 2);
  } else {
    std::vector<float> f;
    if (!to_f32(t, n, f)) return fail(h, FMD_EINVAL, std::string("bad dtype for ") + what);
    for (size_t i = 0; i < n; ++i) bits[i] = bf ? f32_to_bf16_bits(f[i]) : f32_to_f16_bits(f[i]);
  }
  int rc = dev_alloc(h, n * 2, out, &h->weight_bytes);
  if (rc) return rc;
  return upload(h, *out, bits.data(), n * 2);
}

// Projection parts stacked along the output axis (linear.rs:220-265).
// Reorder the rows of a two-part (N = 2 x half) matrix into 32-row groups
// [a0..a31, b0..b31, a32..a63, b32..b63, ...] (see gate_col / up_col).
template <typename E>
void interleave_rows(std::vector<E>& m, int N, int cols) {
  std::vector<E> out(m.size());
  const int half = N / 2;
  for (int r = 0; r < N; ++r) {
    const int part = r / half, i = r % half;
    std::memcpy(&out[(size_t)(part ? up_col(i) : gate_col(i)) * cols], &m[(size_t)r * cols], sizeof(E) * cols);
  }
  m.swap(out);
}

// `interleave16`: store the two parts' rows interleaved in 32-row groups.
// Uploads one projection twice: [N][K] for the mixed-step k_linear and the
// decode-packed tiles of the decode-step GEMV whose epilogue is `epi`.
// `row_major` false: only the packed copy (W.w is set by the caller, as for
// a 16-bit lm_head tied to the embedding table).
// cuTensorMapEncodeTiled, looked up once through the runtime's driver entry point.
int tmap_encoder(fmd_handle* h, void** fn) {
  if (h->tmap_encode == nullptr) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult qr;
    CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr));
    if (f == nullptr || qr != cudaDriverEntryPointSuccess)
      return fail(h, FMD_EIO, "cuTensorMapEncodeTiled is unavailable in this driver");
    h->tmap_encode = f;
  }
  *fn = h->tmap_encode;
  return FMD_OK;
}

// Tensor-core plan and weight map of one projection; a shape without a plan
// keeps tc->ok false and mixed steps use k_linear for it.
int tc_prepare(fmd_handle* h, const void* w16, int N, int K, TcLinear* tc, int want_bn) {
  tc->N = N;
  tc->K = K;
  tc->ok = false;
  if (!tc_plan(N, K, &tc->bn, &tc->split)) return FMD_OK;
  if (N % want_bn == 0) tc->bn = want_bn;
  void* fn;
  int rc = tmap_encoder(h, &fn);
  if (rc) return rc;
  if (!tc_make_map(fn, &tc->wmap, w16, (uint64_t)K, (uint64_t)N, (uint32_t)tc->bn))
    return fail(h, FMD_EIO, "tensor map of a projection's weights could not be encoded");
  tc->ok = true;
  return FMD_OK;
}

// Tile width of a projection on the persistent mixed-step GEMM: qkv and
// gate/up fuse their epilogues over 256-feature tiles, o and down write f32
// rows in 128-feature tiles.
int proj_bn(int epi) { return (epi == kGemvQkv || epi == kGemvSwiglu) ? 256 : 128; }

// The same for Q8_0 weights: the GEMM reads the int8 [N][K] quants through
// the map and their f16 scales directly, and dequantises in shared memory.
int tc_prepare_q8(fmd_handle* h, const int8_t* qs, const uint16_t* d, int N, int K, TcLinear* tc, int want_bn) {
  tc->N = N;
  tc->K = K;
  tc->ok = false;
  if (!tc_plan(N, K, &tc->bn, &tc->split)) return FMD_OK;
  if (N % want_bn == 0) tc->bn = want_bn;
  void* fn;
  int rc = tmap_encoder(h, &fn);
  if (rc) return rc;
  if (!tc_make_map_i8(fn, &tc->wmap, qs, (uint64_t)K, (uint64_t)N, (uint32_t)tc->bn))
    return fail(h, FMD_EIO, "tensor map of a projection's Q8_0 weights could not be encoded");
  tc->q8 = true;
  tc->d = d;
  tc->ok = true;
  return FMD_OK;
}

// `tc`: also build the tensor-core operand of mixed steps (the dense 16-bit
// [N][K] weights themselves, or the Q8_0 quants and scales).
int upload_linear(fmd_handle* h, const std::vector<std::pair<const fmd_tensor*, int>>& parts, int K, LinW& W,
                  const char* what, int epi, bool interleave16 = false, bool row_major = true,
                  TcLinear* tc = nullptr) {
  int N = 0;
  for (auto& p : parts) N += p.second;
  if (N % 64 || K % 64) return fail(h, FMD_ENOTSUP, std::string(what) + ": dims must be multiples of 64");
  W.N = N;
  W.K = K;
  W.q8 = h->q8;
  if (!h->q8) {
    std::vector<uint16_t> bits((size_t)N * K);
    size_t off = 0;
    for (auto& p : parts) {
      const size_t n = (size_t)p.second * K;
      const fmd_tensor& t = *p.first;
      if (t.data == nullptr) return fail(h, FMD_EINVAL, std::string("missing tensor ") + what);
      const bool bf = h->at == kBF16;
      if ((bf && t.dtype == FMD_DT_BF16) || (!bf && t.dtype == FMD_DT_F16)) {
        std::memcpy(bits.data() + off, t.data, n * 2);
      } else {
        std::vector<float> f;
        if (!to_f32(t, n, f)) return fail(h, FMD_EINVAL, std::string("bad dtype for ") + what);
        for (size_t i = 0; i < n; ++i) bits[off + i] = bf ? f32_to_bf16_bits(f[i]) : f32_to_f16_bits(f[i]);
      }
      off += n;
    }
    if (interleave16) interleave_rows(bits, N, K);
    void* d;
    int rc;
    if (row_major) {
      if ((rc = dev_alloc(h, bits.size() * 2, &d, &h->weight_bytes))) return rc;
      if ((rc = upload(h, d, bits.data(), bits.size() * 2))) return rc;
      W.w = d;
    }
    std::vector<uint8_t> pk(gemv_packed_bytes(epi, N, K, false));
    gemv_pack(epi, N, K, false, nullptr, nullptr, bits.data(), pk.data());
    if ((rc = dev_alloc(h, pk.size(), &d, &h->weight_bytes))) return rc;
    if ((rc = upload(h, d, pk.data(), pk.size()))) return rc;
    W.pk = (const uint8_t*)d;
    if (tc && (rc = tc_prepare(h, W.w, N, K, tc, proj_bn(epi)))) return rc;
  } else {
    std::vector<int8_t> qs((size_t)N * K);
    std::vector<uint16_t> sc((size_t)N * (K / 32));
    size_t row = 0;
    for (auto& p : parts) {
      const fmd_tensor& t = *p.first;
      const size_t rows = p.second;
      if (t.data == nullptr) return fail(h, FMD_EINVAL, std::string("missing tensor ") + what);
      if (t.dtype == FMD_DT_Q8_0) {
        const uint8_t* b = (const uint8_t*)t.data;
        for (size_t r = 0; r < rows; ++r)
          for (int kb = 0; kb < K / 32; ++kb) {
            const uint8_t* blk = b + (r * (K / 32) + kb) * 34;
            std::memcpy(&sc[(row + r) * (K / 32) + kb], blk, 2);
            std::memcpy(&qs[(row + r) * K + kb * 32], blk + 2, 32);
          }
      } else {
        std::vector<float> f;
        if (!to_f32(t, rows * K, f)) return fail(h, FMD_EINVAL, std::string("bad dtype for ") + what);
        quantize_rows(f.data(), rows, K, qs.data() + row * K, sc.data() + row * (K / 32));
      }
      row += rows;
    }
    if (interleave16) {
      interleave_rows(qs, N, K);
      interleave_rows(sc, N, K / 32);
    }
    void *dq, *dd;
    int rc = dev_alloc(h, qs.size(), &dq, &h->weight_bytes);
    if (rc) return rc;
    if ((rc = dev_alloc(h, sc.size() * 2, &dd, &h->weight_bytes))) return rc;
    if ((rc = upload(h, dq, qs.data(), qs.size()))) return rc;
    if ((rc = upload(h, dd, sc.data(), sc.size() * 2))) return rc;
    W.qs = (const int8_t*)dq;
    W.d = (const uint16_t*)dd;
    std::vector<uint8_t> pk(gemv_packed_bytes(epi, N, K, true));
    gemv_pack(epi, N, K, true, qs.data(), sc.data(), nullptr, pk.data());
    void* dp;
    if ((rc = dev_alloc(h, pk.size(), &dp, &h->weight_bytes))) return rc;
    if ((rc = upload(h, dp, pk.data(), pk.size()))) return rc;
    W.pk = (const uint8_t*)dp;
    if (tc && (rc = tc_prepare_q8(h, W.qs, W.d, N, K, tc, proj_bn(epi)))) return rc;
  }
  // K split for passes with <= 64 rows: aim for >= ~2 CTAs per SM.
  int split = 1;
  const int ctas = N / 64;
  while (split < 16 && ctas * split < 296 && K % (64 * split * 2) == 0 && K / (split * 2) >= 128) split *= 2;
  W.split = split;
  return FMD_OK;
}

void release_graph(fmd_handle* h) {
  if (h->graph_exec) {
    cudaGraphExecDestroy(h->graph_exec);
    h->graph_exec = nullptr;
  }
  if (h->graph_dec) {
    cudaGraphExecDestroy(h->graph_dec);
    h->graph_dec = nullptr;
  }
  h->graph_batch = h->graph_chunk = -1;
}

// Opt-in launch tracing (FMD_TRACE=1): synchronise after every launch and log
// it, so a kernel that stalls or faults is identified by name.
bool trace_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FMD_TRACE");
    return v != nullptr && v[0] == '1';
  }();
  return on;
}
void trace(fmd_handle* h, const char* what, int layer) {
  if (!trace_enabled()) return;
  const auto t0 = std::chrono::steady_clock::now();
  cudaError_t e = cudaStreamSynchronize(h->stream);
  const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  std::fprintf(stderr, "[fmd] %-16s layer %3d  %8.3f ms  %s\n", what, layer, ms, cudaGetErrorString(e));
}

// The layer tail of layer l: its o, gate/up and down projections and, except
// for the last layer, the next layer's qkv.
ChainArgs make_chain(fmd_handle* h, int l) {
  const fmd_config& c = h->cfg;
  const LayerDev& L = h->layers[l];
  const int H = c.hidden_size, I = c.intermediate_size, qd = h->Hq() * kHeadDim;
  ChainArgs a;
  a.ph[0] = ChainPhase{L.o.pk, H, qd, gemv_tile_features(kGemvResid), gemv_split(kGemvResid, qd)};
  a.ph[1] = ChainPhase{L.gate_up.pk, 2 * I, H, gemv_tile_features(kGemvSwiglu), gemv_split(kGemvSwiglu, H)};
  a.ph[2] = ChainPhase{L.down.pk, H, I, gemv_tile_features(kGemvResid), gemv_split(kGemvResid, I)};
  const bool last = l + 1 >= c.num_hidden_layers;
  a.n_phases = last ? 3 : 4;
  if (!last) {
    const LayerDev& Ln = h->layers[l + 1];
    a.ph[3] = ChainPhase{Ln.qkv.pk, h->qkvN(), H, gemv_tile_features(kGemvQkv), gemv_split(kGemvQkv, H)};
    a.in_norm = Ln.in_norm;
    a.qn_w = Ln.q_norm;
    a.kn_w = Ln.k_norm;
    a.layer = l + 1;
  }
  a.n_rows_ptr = &h->plan.counts->n_rows;
  a.ctx = h->ctx;
  a.x = h->x;
  a.h = h->hbuf;
  a.ssq = h->ssq;
  a.ssq_tiles = H / 64;
  a.eps = c.rms_norm_eps;
  a.post_norm = L.post_norm;
  a.cos = h->rope_cos;
  a.sin = h->rope_sin;
  a.q_out = h->qbuf;
  a.kv = h->kv;
  a.plan = h->plan;
  a.Hq = h->Hq();
  a.Hkv = h->Hkv();
  a.H = H;
  a.I = I;
  a.sync = h->chain_sync ? h->chain_sync + (size_t)l * kChainSyncInts : nullptr;
  a.status = h->d_status;
  return a;
}

// ---- forward pass ------------------------------------------------------------------
// Decode-only forward pass (every row is a one-token decode row): per layer
// QKV (input norm folded in, q/k norm + RoPE + KV write fused) -> attention
// -> O (+ residual) -> gate/up (post-attention norm folded in, SwiGLU fused)
// -> down (+ residual); the split-K of each projection is reduced inside a
// thread-block cluster.
// Rows [r0, r0 + max_rows) of a decode-only pass: the plan's counts for
// them (plan.counts) and every per-row array and buffer from row r0.
struct DecodeView {
  Plan plan;
  int max_rows;
  void *x, *qbuf, *ctx, *hbuf;
  float *ssq, *pacc, *pml;
  int* counters;
  int grid;  // decode attention CTAs
};

// half = -1: every row; 0 / 1: the rows of that half of a split step.
DecodeView decode_view(fmd_handle* h, int half) {
  const fmd_config& c = h->cfg;
  const int R = h->max_slots, H = c.hidden_size, I = c.intermediate_size, HqD = h->Hq() * kHeadDim;
  DecodeView v;
  v.plan = h->plan;
  v.max_rows = R;
  v.x = h->x;
  v.qbuf = h->qbuf;
  v.ctx = h->ctx;
  v.hbuf = h->hbuf;
  v.ssq = h->ssq;
  v.pacc = h->pacc;
  v.pml = h->pml;
  v.counters = h->attn_counters;
  v.grid = h->di_grid;
  if (half < 0) return v;
  const int S = R / 2, r0 = half * S;
  v.plan.counts = h->half_counts + half;
  v.plan.row_slot += r0;
  v.plan.row_pos += r0;
  v.plan.row_tok += r0;
  v.plan.row_emb += r0;
  v.max_rows = half ? R - S : S;
  v.x = (uint16_t*)h->x + (size_t)r0 * H;
  v.qbuf = (uint16_t*)h->qbuf + (size_t)r0 * HqD;
  v.ctx = (uint16_t*)h->ctx + (size_t)r0 * HqD;
  v.hbuf = (uint16_t*)h->hbuf + (size_t)r0 * I;
  v.ssq = h->ssq + (size_t)r0 * (H / 64);
  if (half) {
    v.pacc = h->pacc2;
    v.pml = h->pml2;
  }
  v.counters = h->attn_counters + (size_t)r0 * h->Hkv();
  v.grid = h->n_sm;  // one attention CTA per SM leaves room for the other half's projections
  return v;
}

// The layer loop of a decode-only pass over the rows of `v` on stream `s`.
void decode_layers(fmd_handle* h, const DecodeView& v, cudaStream_t s, bool probe_attn) {
  const fmd_config& c = h->cfg;
  const int H = c.hidden_size, I = c.intermediate_size;
  const int R = v.max_rows;
  const int* nrows = &v.plan.counts->n_rows;
  const float eps = c.rms_norm_eps;
  const int ssq_tiles = H / 64;
  const int L = c.num_hidden_layers;
  GemvEpi qkv;
  qkv.ssq = v.ssq;
  qkv.ssq_tiles = ssq_tiles;
  qkv.eps = eps;
  qkv.plan = v.plan;
  qkv.cos = h->rope_cos;
  qkv.sin = h->rope_sin;
  qkv.q_out = v.qbuf;
  qkv.kv = h->kv;
  qkv.Hq = h->Hq();
  qkv.Hkv = h->Hkv();
  GemvEpi res;
  res.x = v.x;
  res.ssq_out = v.ssq;
  res.ssq_tiles = ssq_tiles;
  GemvEpi glu = qkv;
  glu.h = v.hbuf;
  glu.I = I;
  for (int l = 0; l < L; ++l) {
    const LayerDev& Ly = h->layers[l];
    if (l == 0 || !h->chain_ok) {
      qkv.norm_w = Ly.in_norm;
      qkv.qn_w = Ly.q_norm;
      qkv.kn_w = Ly.k_norm;
      qkv.layer = l;
      if (!launch_gemv(h->at, kGemvQkv, true, Ly.qkv, v.x, H, nullptr, nrows, R, qkv, h->d_status, s)) h->launch_refused = true;
      trace(h, "qkv", l);
    }
    const bool probe = probe_attn && h->record_attn_events && l == h->attn_probe_layer();
    if (probe) cudaEventRecordWithFlags(h->attn_events[0], s, cudaEventRecordExternal);
    launch_attn_decode_tma(h->at, &h->kv_tmap, v.plan, v.grid, h->Hq(), h->Hkv(), v.qbuf, h->kv, l,
                           h->attn_scale, v.pacc, v.pml, v.counters, v.ctx, h->d_status, s);
    if (probe) cudaEventRecordWithFlags(h->attn_events[1], s, cudaEventRecordExternal);
    trace(h, "attn_decode", l);
    if (h->chain_ok) {
      // o -> gate/up -> down -> the next layer's qkv in one persistent launch
      launch_layer_tail(h->at, make_chain(h, l), h->chain_clusters, h->chain_smem, s);
      trace(h, "layer_tail", l);
      continue;
    }
    if (!launch_gemv(h->at, kGemvResid, false, Ly.o, v.ctx, h->Hq() * kHeadDim, nullptr, nrows, R, res, h->d_status, s)) h->launch_refused = true;
    trace(h, "o_proj", l);
    glu.norm_w = Ly.post_norm;
    if (!launch_gemv(h->at, kGemvSwiglu, true, Ly.gate_up, v.x, H, nullptr, nrows, R, glu, h->d_status, s)) h->launch_refused = true;
    trace(h, "gate_up", l);
    if (!launch_gemv(h->at, kGemvResid, false, Ly.down, v.hbuf, I, nullptr, nrows, R, res, h->d_status, s)) h->launch_refused = true;
    trace(h, "down", l);
  }
}

// Decode-only forward pass (every row is a one-token decode row): per layer
// QKV (input norm folded in, q/k norm + RoPE + KV write fused) -> attention
// -> O (+ residual) -> gate/up (post-attention norm folded in, SwiGLU fused)
// -> down (+ residual); the split-K of each projection is reduced inside a
// thread-block cluster. A split step runs the layer loop of each half of the
// rows on its own stream (rows are independent in every kernel of the loop,
// so the results are those of one pass over all rows).
void run_forward_decode(fmd_handle* h, float* logits_dev, const void* arena) {
  cudaStream_t s = h->stream;
  const fmd_config& c = h->cfg;
  const int R = h->max_slots, H = c.hidden_size;
  const int row_grid = std::min(R, 296);
  const int* nsamp = &h->plan.counts->n_sample;
  const float eps = c.rms_norm_eps;
  const int ssq_tiles = H / 64;
  const int L = c.num_hidden_layers;
  // the halves' row counts before the embedding: the projections read their
  // row count ahead of their dependency wait, so it must come from a kernel
  // at least two launches back
  if (h->split_ok) launch_half_counts(h->plan.counts, h->half_counts, R / 2, s);
  launch_embed_norm(h->at, h->plan, row_grid, h->embed, arena, h->x, h->layers[0].in_norm, h->xn, H, eps, h->ssq,
                    ssq_tiles, s, h->chain_ok ? h->chain_sync : nullptr, h->chain_ok ? L * kChainSyncInts : 0);
  trace(h, "embed_norm", -1);
  if (h->split_ok) {
    cudaEventRecord(h->fork_ev, s);
    cudaStreamWaitEvent(h->stream2, h->fork_ev, 0);
    decode_layers(h, decode_view(h, 0), s, true);
    decode_layers(h, decode_view(h, 1), h->stream2, false);
    cudaEventRecord(h->join_ev, h->stream2);
    cudaStreamWaitEvent(s, h->join_ev, 0);
  } else {
    decode_layers(h, decode_view(h, -1), s, true);
  }
  GemvEpi head;
  head.ssq = h->ssq;
  head.ssq_tiles = ssq_tiles;
  head.eps = eps;
  head.norm_w = h->final_norm;
  head.logits = logits_dev;
  head.best_val = h->best_val;
  head.best_idx = h->best_idx;
  if (h->record_attn_events) cudaEventRecordWithFlags(h->attn_events[2], s, cudaEventRecordExternal);
  const int parts = launch_lm_head(h->at, h->lm_head, h->x, H, h->plan.sample_row, nsamp, h->max_slots, head,
                                   h->d_status, s, h->lm_tc_allowed, h->lm_f16_allowed, &h->lm_tc_used);
  if (h->record_attn_events) cudaEventRecordWithFlags(h->attn_events[3], s, cudaEventRecordExternal);
  if (parts == 0) h->launch_refused = true;
  trace(h, "lm_head", -1);
  launch_pick_reduce(nsamp, h->max_slots, h->best_val, h->best_idx, parts, h->next_ids, c.vocab_size,
                       h->d_status, s);
  trace(h, "argmax", -1);
}

// One projection of a mixed step over all of its rows: tcgen05 GEMM when the
// projection has a tensor-core plan, else k_linear. Returns the K splits the
// f32 partials in h->part carry.
PartSplit mixed_linear(fmd_handle* h, const LinW& W, const TcLinear& tc, const void* x, const CUtensorMap& amap,
                       int ldx) {
  if (h->tc_ready && launch_gemm_tc(h->at, amap, tc, &h->plan.counts->n_rows, h->max_rows, h->part, h->split_stride,
                                    h->d_status, h->stream))
    return PartSplit{tc.split, tc.split};
  launch_linear(h->at, W, x, ldx, nullptr, &h->plan.counts->n_rows, h->max_rows, h->part, h->split_stride, false,
                h->stream);
  return linear_split(W.split);
}

// `decode_only`: every row is a one-token decode row (no prefill attention,
// weights prefetched ahead of each projection's dependency wait).
void run_forward(fmd_handle* h, float* logits_dev, const void* arena, bool decode_only = false) {
  cudaStream_t s = h->stream;
  const fmd_config& c = h->cfg;
  const int R = h->max_rows, H = c.hidden_size, I = c.intermediate_size;
  const int row_grid = std::min(R, 296);
  const int* nrows = &h->plan.counts->n_rows;
  const int* nsamp = &h->plan.counts->n_sample;
  const float eps = c.rms_norm_eps;
  const size_t ss = h->split_stride;
  if (decode_only) {
    run_forward_decode(h, logits_dev, arena);
    return;
  }
  launch_embed_norm(h->at, h->plan, row_grid, h->embed, arena, h->x, h->layers[0].in_norm, h->xn, H, eps, nullptr,
                    0, s);
  trace(h, "embed_norm", -1);
  // the persistent projection GEMM with fused epilogues when the projection
  // has a plan for it (k_gemm_tc + the split-K epilogue kernels otherwise)
  const bool proj = h->tc_ready && h->proj_allowed;
  auto run_proj = [&](const TcLinear& tc, const CUtensorMap& amap, int epi, const ProjEpi& ep) {
    return proj && launch_proj_tc(h->at, epi, amap, tc, nrows, R, ep, h->n_sm, h->d_status, s);
  };
  ProjEpi pf32;
  pf32.out = h->part;
  for (int l = 0; l < c.num_hidden_layers; ++l) {
    const LayerDev& L = h->layers[l];
    ProjEpi pq;
    pq.plan = h->plan;
    pq.kv = h->kv;
    pq.qn_w = L.q_norm;
    pq.kn_w = L.k_norm;
    pq.cos = h->rope_cos;
    pq.sin = h->rope_sin;
    pq.q_out = h->qbuf;
    pq.layer = l;
    pq.Hq = h->Hq();
    pq.Hkv = h->Hkv();
    pq.eps = eps;
    if (run_proj(L.tc_qkv, h->amap_xn, kProjQkv, pq)) {
      trace(h, "qkv_proj", l);
    } else {
      const PartSplit sp_qkv = mixed_linear(h, L.qkv, L.tc_qkv, h->xn, h->amap_xn, H);
      trace(h, "qkv", l);
      launch_qkv_epilogue(h->at, h->plan, row_grid, h->part, sp_qkv, ss, h->Hq(), h->Hkv(), L.q_norm, L.k_norm,
                          h->rope_cos, h->rope_sin, h->qbuf, h->kv, l, eps, s);
      trace(h, "qkv_epi", l);
    }
    const bool probe = h->record_attn_events && l == h->attn_probe_layer();
    if (probe) cudaEventRecordWithFlags(h->attn_events[0], s, cudaEventRecordExternal);
    launch_attn_decode_tma(h->at, &h->kv_tmap, h->plan, h->di_grid, h->Hq(), h->Hkv(), h->qbuf, h->kv, l,
                           h->attn_scale, h->pacc, h->pml, h->attn_counters, h->ctx, h->d_status, s);
    if (probe) cudaEventRecordWithFlags(h->attn_events[1], s, cudaEventRecordExternal);
    trace(h, "attn_decode", l);
    launch_attn_prefill_tc(h->at, &h->kv_tmap, &h->qmap, h->plan, h->pb_max, h->Hq(), h->Hkv(), h->kv, l,
                           h->attn_scale, h->ctx, h->d_status, s, h->pf_pp_allowed ? h->n_sm : 0);
    trace(h, "attn_prefill", l);
    const PartSplit sp_o = run_proj(L.tc_o, h->amap_ctx, kProjF32, pf32)
                               ? PartSplit{1, 1}
                               : mixed_linear(h, L.o, L.tc_o, h->ctx, h->amap_ctx, h->Hq() * kHeadDim);
    trace(h, "o_proj", l);
    launch_residual_norm(h->at, nrows, row_grid, h->x, h->part, sp_o, ss, L.post_norm, h->xn, H, eps, s);
    trace(h, "res_norm1", l);
    ProjEpi pg;
    pg.h = h->hbuf;
    pg.I = I;
    if (run_proj(L.tc_gate_up, h->amap_xn, kProjSwiglu, pg)) {
      trace(h, "gate_up_proj", l);
    } else {
      const PartSplit sp_gu = mixed_linear(h, L.gate_up, L.tc_gate_up, h->xn, h->amap_xn, H);
      trace(h, "gate_up", l);
      launch_silu_mul(h->at, nrows, row_grid, h->part, sp_gu, ss, I, h->hbuf, s);
      trace(h, "silu", l);
    }
    const PartSplit sp_down = run_proj(L.tc_down, h->amap_hbuf, kProjF32, pf32)
                                  ? PartSplit{1, 1}
                                  : mixed_linear(h, L.down, L.tc_down, h->hbuf, h->amap_hbuf, I);
    trace(h, "down", l);
    const void* next_norm = l + 1 < c.num_hidden_layers ? h->layers[l + 1].in_norm : h->final_norm;
    launch_residual_norm(h->at, nrows, row_grid, h->x, h->part, sp_down, ss, next_norm, h->xn, H, eps, s);
    trace(h, "res_norm2", l);
  }
  // the rows are normalised already (the last residual_norm applied the final norm)
  GemvEpi head{};
  head.logits = logits_dev;
  head.best_val = h->best_val;
  head.best_idx = h->best_idx;
  if (h->record_attn_events) cudaEventRecordWithFlags(h->attn_events[2], s, cudaEventRecordExternal);
  const int parts = launch_lm_head(h->at, h->lm_head, h->xn, H, h->plan.sample_row, nsamp, h->max_slots, head,
                                   h->d_status, s, h->lm_tc_allowed, h->lm_f16_allowed, &h->lm_tc_used);
  if (h->record_attn_events) cudaEventRecordWithFlags(h->attn_events[3], s, cudaEventRecordExternal);
  trace(h, "lm_head", -1);
  if (parts > 0) {
    launch_pick_reduce(nsamp, h->max_slots, h->best_val, h->best_idx, parts, h->next_ids, c.vocab_size,
                       h->d_status, s);
  } else {
    launch_linear(h->at, h->lm_head, h->xn, H, h->plan.sample_row, nsamp, h->max_slots, h->part, ss, decode_only, s);
    launch_logits_argmax(h->at, nsamp, h->max_slots, h->part, c.vocab_size, logits_dev, h->next_ids, s);
  }
  trace(h, "argmax", -1);
}

// ---- host plan helpers -------------------------------------------------------------
struct HostPlan {
  fmd_handle* h;
  Plan p;  // bound to the pinned mirror
  int rows = 0, n_decode = 0, samples = 0, pblocks = 0, items = 0;
  explicit HostPlan(fmd_handle* hh) : h(hh) { p = hh->layout.bind(hh->h_plan); }
  void add_decode(int slot, int pos, int tok) {
    const int r = rows++;
    p.row_slot[r] = slot;
    p.row_pos[r] = pos;
    p.row_tok[r] = tok;
    p.row_emb[r] = 0;
    const int kv_len = pos + 1;
    const int nit = (kv_len + kDecodeItemTokens - 1) / kDecodeItemTokens;
    p.drow_item0[r] = items;
    p.drow_nitems[r] = nit;
    for (int j = 0; j < nit; ++j) {
      p.di_row[items + j] = r;
      p.di_start[items + j] = j * kDecodeItemTokens;
      p.di_end[items + j] = std::min(kv_len, (j + 1) * kDecodeItemTokens);
    }
    items += nit;
    p.sample_row[samples] = r;
    p.sample_slot[samples] = slot;
    ++samples;
    n_decode = rows;
  }
  // `n` prompt rows of `slot` at positions pos0.., arena rows emb0..; sample the last one if `sample`.
  void add_prefill(int slot, int pos0, int n, int emb0, bool sample) {
    const int r0 = rows;
    for (int i = 0; i < n; ++i) {
      p.row_slot[r0 + i] = slot;
      p.row_pos[r0 + i] = pos0 + i;
      p.row_tok[r0 + i] = -1;
      p.row_emb[r0 + i] = emb0 + i;
    }
    for (int j = 0; j < n; j += kRowsPerPBlock) {
      p.pb_row0[pblocks] = r0 + j;
      p.pb_n[pblocks] = std::min(kRowsPerPBlock, n - j);
      ++pblocks;
    }
    rows += n;
    if (sample) {
      p.sample_row[samples] = r0 + n - 1;
      p.sample_slot[samples] = slot;
      ++samples;
    }
  }
  int commit() {
    PlanCounts* c = p.counts;
    c->n_rows = rows;
    c->n_decode = n_decode;
    c->n_sample = samples;
    c->n_pblocks = pblocks;
    c->n_ditems = items;
    c->finished = 0;
    fmd_handle* hh = h;
    cudaError_t e = cudaMemcpyAsync(hh->d_plan, hh->h_plan, hh->layout.total * sizeof(int), cudaMemcpyHostToDevice,
                                    hh->stream);
    if (e != cudaSuccess) return fail(hh, FMD_EIO, std::string("plan upload: ") + cudaGetErrorString(e));
    return FMD_OK;
  }
};

int check_ready(fmd_handle* h) {
  if (!h) return FMD_EINVAL;
  if (!h->loaded) return fail(h, FMD_EBUSY, "no weights loaded (fmd_load_weights)");
  if (!h->reserved) return fail(h, FMD_EBUSY, "no KV pool reserved (fmd_kv_reserve)");
  return FMD_OK;
}

int sync_check(fmd_handle* h) {
  if (h->launch_refused) {
    h->launch_refused = false;
    return fail(h, FMD_EIO, "a decode projection was not launched (no packed weight tiles or no valid K split)");
  }
  cudaError_t e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return fail(h, FMD_EIO, std::string("device error: ") + cudaGetErrorString(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(h, FMD_EIO, std::string("launch error: ") + cudaGetErrorString(e));
  if (h->d_status) {
    int st[2] = {0, 0};
    e = cudaMemcpy(st, h->d_status, 2 * sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(h, FMD_EIO, std::string("status read: ") + cudaGetErrorString(e));
    if (st[0] != 0) {
      cudaMemset(h->d_status, 0, 2 * sizeof(int));
      static const char* const kSites[] = {"?", "k_gemv", "k_lm_head", "k_attn_decode_tma", "k_attn_prefill_tc",
                                           "k_gemm_tc", "k_layer_tail", "k_wait_probe", "k_proj_tc"};
      constexpr int kNumSites = (int)(sizeof(kSites) / sizeof(kSites[0]));
      const char* site = st[1] >= 1 && st[1] < kNumSites ? kSites[st[1]] : "?";
      return fail(h, st[0], st[0] == FMD_EIO ? std::string("a greedy pick found no finite logit (non-finite activations)")
                                             : "a bounded device-side wait gave up in " + std::string(site) +
                                                   " (status " + std::to_string(st[0]) + ")");
    }
  }
  return FMD_OK;
}

int convert_rows_to_act(fmd_handle* h, const void* src, int32_t dtype, size_t rows, std::vector<uint16_t>& out) {
  const size_t n = rows * h->H();
  out.resize(n);
  const bool bf = h->at == kBF16;
  if ((bf && dtype == FMD_DT_BF16) || (!bf && dtype == FMD_DT_F16)) {
    std::memcpy(out.data(), src, n * 2);
  } else if (dtype == FMD_DT_F32) {
    const float* f = (const float*)src;
    for (size_t i = 0; i < n; ++i) out[i] = bf ? f32_to_bf16_bits(f[i]) : f32_to_f16_bits(f[i]);
  } else {
    return fail(h, FMD_EINVAL, "embeds dtype must be f32 or the activation dtype");
  }
  return FMD_OK;
}

int copy_outputs(fmd_handle* h, int n_sample, const std::vector<int>& order, float* logits, int32_t* ids) {
  // order[i] = caller index of sample row i
  const int V = h->cfg.vocab_size;
  std::vector<int> tmp(n_sample);
  if (ids) {
    CK(cudaMemcpyAsync(tmp.data(), h->next_ids, n_sample * sizeof(int), cudaMemcpyDeviceToHost, h->stream));
  }
  if (logits) {
    for (int i = 0; i < n_sample; ++i)
      CK(cudaMemcpyAsync(logits + (size_t)order[i] * V, h->logits + (size_t)i * V, (size_t)V * 4,
                         cudaMemcpyDeviceToHost, h->stream));
  }
  int rc = sync_check(h);
  if (rc) return rc;
  if (ids)
    for (int i = 0; i < n_sample; ++i) ids[order[i]] = tmp[i];
  return FMD_OK;
}

int ensure_pages(fmd_handle* h, int slot, int upto_len) {
  const int need = (upto_len + kPageTokens - 1) / kPageTokens;
  if (need > h->max_pages_per_slot) return fail(h, FMD_EOVERFLOW, "sequence longer than the RoPE table / slot limit");
  bool changed = false;
  while (h->slot_npages[slot] < need) {
    if (h->free_pages.empty()) return fail(h, FMD_ENOMEM, "KV pool exhausted");
    h->h_page_table[(size_t)slot * h->max_pages_per_slot + h->slot_npages[slot]] = h->free_pages.back();
    h->free_pages.pop_back();
    h->slot_npages[slot] += 1;
    changed = true;
  }
  if (changed) {
    const size_t off = (size_t)slot * h->max_pages_per_slot;
    CK(cudaMemcpyAsync(h->d_page_table + off, h->h_page_table.data() + off, need * sizeof(int),
                       cudaMemcpyHostToDevice, h->stream));
  }
  return FMD_OK;
}

}  // namespace

// =====================================================================================
extern "C" {

int fmd_version(void) { return kVersion; }

const char* fmd_status_string(int32_t status) {
  switch (status) {
    case FMD_OK: return "ok";
    case FMD_EINVAL: return "invalid argument";
    case FMD_ENOMEM: return "out of device memory / KV pool exhausted";
    case FMD_EIO: return "CUDA error";
    case FMD_EBUSY: return "handle not ready";
    case FMD_EOVERFLOW: return "KV cache capacity exceeded";
    case FMD_ENOTSUP: return "not supported";
    case FMD_ETIMEDOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

const char* fmd_last_error(const fmd_handle* h) { return h ? h->err.c_str() : "null handle"; }

int fmd_create(const fmd_config* cfg, int32_t precision, int32_t device, fmd_handle** out) {
  if (!cfg || !out) return FMD_EINVAL;
  *out = nullptr;
  if (precision == FMD_PREC_F32) return FMD_ENOTSUP;
  if (precision < FMD_PREC_F16 || precision > FMD_PREC_INT8_BF16) return FMD_EINVAL;
  if (cfg->head_dim != kHeadDim) return FMD_ENOTSUP;
  if (cfg->num_attention_heads != 2 * cfg->num_key_value_heads) return FMD_ENOTSUP;
  if (cfg->hidden_size % 64 || cfg->intermediate_size % 64 || cfg->vocab_size % 64)
    return FMD_ENOTSUP;
  if (cfg->num_hidden_layers < 1 || cfg->hidden_size <= 0) return FMD_EINVAL;
  if (cfg->hidden_size > 64 * 64) return FMD_ENOTSUP;  // per-row norm partials: at most 64 tiles of 64
  // decode-path projections: lm_head tiles are 128 features wide, and each
  // contraction must split into slices the cluster GEMV holds
  if (cfg->vocab_size % gemv_tile_features(kGemvLogits) ||
      !gemv_split(kGemvQkv, cfg->hidden_size) || !gemv_split(kGemvLogits, cfg->hidden_size) ||
      !gemv_split(kGemvResid, cfg->num_attention_heads * cfg->head_dim) ||
      !gemv_split(kGemvResid, cfg->intermediate_size))
    return FMD_ENOTSUP;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return FMD_EIO;
  }
  fmd_handle* h = new fmd_handle();
  h->cfg = *cfg;
  h->precision = precision;
  h->q8 = precision == FMD_PREC_INT8 || precision == FMD_PREC_INT8_BF16;
  h->at = (precision == FMD_PREC_BF16 || precision == FMD_PREC_INT8_BF16) ? kBF16 : kF16;
  h->device = device;
  h->attn_scale = (float)(1.0 / std::sqrt((double)cfg->head_dim));
  {
    const char* v = std::getenv("FMD_LAYER_TAIL");
    h->chain_allowed = v != nullptr && v[0] == '1';
    const char* p = std::getenv("FMD_PROJ_TC");
    h->proj_allowed = !(p != nullptr && p[0] == '0');
    const char* lt = std::getenv("FMD_LM_HEAD_TC");
    h->lm_tc_allowed = lt != nullptr && lt[0] == '1';
    const char* lf = std::getenv("FMD_LM_HEAD_F16");
    h->lm_f16_allowed = !(lf != nullptr && lf[0] == '0');
    const char* pp = std::getenv("FMD_PREFILL_PP");
    h->pf_pp_allowed = !(pp != nullptr && pp[0] == '0');
    const char* sp = std::getenv("FMD_DECODE_SPLIT");
    h->split_allowed = sp != nullptr && sp[0] == '1';
  }
  if (cudaDeviceGetAttribute(&h->n_sm, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || h->n_sm < 1) {
    cudaGetLastError();
    delete h;
    return FMD_EIO;
  }
  if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess ||
      init_kernels() != cudaSuccess || init_attn_decode() != cudaSuccess || init_attn_prefill() != cudaSuccess || init_gemv() != cudaSuccess ||
      init_gemm_tc() != cudaSuccess || init_proj_tc() != cudaSuccess) {
    cudaGetLastError();
    delete h;
    return FMD_EIO;
  }
  *out = h;
  return FMD_OK;
}

int fmd_destroy(fmd_handle* h) {
  if (!h) return FMD_OK;
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  release_graph(h);
  for (cudaEvent_t e : h->attn_events) cudaEventDestroy(e);
  if (h->win_begin) cudaEventDestroy(h->win_begin);
  if (h->win_end) cudaEventDestroy(h->win_end);
  for (auto& a : h->allocs) cudaFree(a.p);
  for (DevBuf* b : {&h->eng_reqs, &h->eng_arena, &h->eng_tokens, &h->eng_results, &h->splice_src})
    if (b->p) cudaFree(b->p);
  if (h->h_plan) cudaFreeHost(h->h_plan);
  if (h->h_ctr) cudaFreeHost(h->h_ctr);
  if (h->fork_ev) cudaEventDestroy(h->fork_ev);
  if (h->join_ev) cudaEventDestroy(h->join_ev);
  if (h->stream2) cudaStreamDestroy(h->stream2);
  if (h->stream) cudaStreamDestroy(h->stream);
  delete h;
  return FMD_OK;
}

int fmd_load_weights(fmd_handle* h, const fmd_weights* w) {
  if (!h || !w || !w->layers) return fail(h, FMD_EINVAL, "null weights");
  if (h->loaded) return fail(h, FMD_EBUSY, "weights already loaded");
  CK(cudaSetDevice(h->device));
  const fmd_config& c = h->cfg;
  const int H = c.hidden_size, I = c.intermediate_size, qd = c.num_attention_heads * kHeadDim,
            kvd = c.num_key_value_heads * kHeadDim;
  int rc;
  if ((rc = upload_dense(h, w->embed_tokens, (size_t)c.vocab_size * H, &h->embed, "embed_tokens"))) return rc;
  if ((rc = upload_dense(h, w->norm, H, &h->final_norm, "norm"))) return rc;
  h->layers.resize(c.num_hidden_layers);
  for (int l = 0; l < c.num_hidden_layers; ++l) {
    const fmd_layer_weights& s = w->layers[l];
    LayerDev& L = h->layers[l];
    if ((rc = upload_dense(h, s.input_layernorm, H, &L.in_norm, "input_layernorm"))) return rc;
    if ((rc = upload_dense(h, s.post_attention_layernorm, H, &L.post_norm, "post_attention_layernorm"))) return rc;
    if ((rc = upload_dense(h, s.q_norm, kHeadDim, &L.q_norm, "q_norm"))) return rc;
    if ((rc = upload_dense(h, s.k_norm, kHeadDim, &L.k_norm, "k_norm"))) return rc;
    if ((rc = upload_linear(h, {{&s.q_proj, qd}, {&s.k_proj, kvd}, {&s.v_proj, kvd}}, H, L.qkv, "qkv", kGemvQkv, false, true, &L.tc_qkv)))
      return rc;
    if ((rc = upload_linear(h, {{&s.o_proj, H}}, qd, L.o, "o_proj", kGemvResid, false, true, &L.tc_o))) return rc;
    if ((rc = upload_linear(h, {{&s.gate_proj, I}, {&s.up_proj, I}}, H, L.gate_up, "gate_up", kGemvSwiglu, true, true,
                             &L.tc_gate_up)))
      return rc;
    if ((rc = upload_linear(h, {{&s.down_proj, H}}, I, L.down, "down_proj", kGemvResid, false, true, &L.tc_down)))
      return rc;
  }
  // lm_head: tied to the embedding unless given (qwen3.rs:366-372); in int8 it
  // is quantised from the source values (qwen3.rs:566-578).
  const fmd_tensor& head = w->lm_head.data ? w->lm_head : w->embed_tokens;
  if (!h->q8 && !w->lm_head.data) {
    h->lm_head.w = h->embed;
    if ((rc = upload_linear(h, {{&head, c.vocab_size}}, H, h->lm_head, "lm_head", kGemvLogits, false, false)))
      return rc;
  } else {
    if ((rc = upload_linear(h, {{&head, c.vocab_size}}, H, h->lm_head, "lm_head", kGemvLogits))) return rc;
  }
  h->lm_head.split = 1;
  // RoPE tables (qwen3.rs:116-136): inv_freq in f64 -> f32, pos*inv_freq in
  // f32, cos/sin in f32, stored in the activation dtype.
  h->rope_len = std::min(c.max_position_embeddings, 65536);
  const int half = kHeadDim / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = (float)(1.0 / std::pow(c.rope_theta, 2.0 * i / kHeadDim));
  std::vector<uint16_t> cs((size_t)h->rope_len * half), sn((size_t)h->rope_len * half);
  const bool bf = h->at == kBF16;
  for (int p = 0; p < h->rope_len; ++p)
    for (int i = 0; i < half; ++i) {
      const float f = (float)p * inv[i];
      const float cv = std::cos(f), sv = std::sin(f);
      cs[(size_t)p * half + i] = bf ? f32_to_bf16_bits(cv) : f32_to_f16_bits(cv);
      sn[(size_t)p * half + i] = bf ? f32_to_bf16_bits(sv) : f32_to_f16_bits(sv);
    }
  if ((rc = dev_alloc(h, cs.size() * 2, &h->rope_cos, &h->weight_bytes))) return rc;
  if ((rc = dev_alloc(h, sn.size() * 2, &h->rope_sin, &h->weight_bytes))) return rc;
  if ((rc = upload(h, h->rope_cos, cs.data(), cs.size() * 2))) return rc;
  if ((rc = upload(h, h->rope_sin, sn.data(), sn.size() * 2))) return rc;
  h->loaded = true;
  return FMD_OK;
}

int64_t fmd_cache_bytes(const fmd_config* cfg, int32_t precision, int64_t batch, int64_t capacity) {
  if (!cfg) return FMD_EINVAL;
  const int64_t elem = precision == FMD_PREC_F32 ? 4 : 2;
  return (int64_t)cfg->num_hidden_layers * 2 * batch * cfg->num_key_value_heads * capacity * cfg->head_dim * elem;
}

int fmd_memory_bytes(const fmd_handle* h, int64_t* weights, int64_t* kv_pool, int64_t* workspace) {
  if (!h) return FMD_EINVAL;
  if (weights) *weights = h->weight_bytes;
  if (kv_pool) *kv_pool = h->kv_bytes;
  if (workspace) *workspace = h->work_bytes;
  return FMD_OK;
}

int fmd_kv_reserve(fmd_handle* h, int32_t max_slots, int64_t max_tokens_total, int32_t max_rows_per_step) {
  if (!h) return FMD_EINVAL;
  if (!h->loaded) return fail(h, FMD_EBUSY, "load weights before reserving the KV pool");
  if (h->reserved) return fail(h, FMD_EBUSY, "KV pool already reserved");
  if (max_slots < 1 || max_slots > kMaxSlotsLimit || max_tokens_total < 1 || max_rows_per_step < max_slots)
    return fail(h, FMD_EINVAL, "bad KV reservation sizes (need 1 <= max_slots <= 256, rows >= slots)");
  if (max_rows_per_step / kRowsPerPBlock + max_slots > kMaxPrefillBlocks)
    return fail(h, FMD_ENOTSUP, "max_rows_per_step too large for the prefill attention");
  CK(cudaSetDevice(h->device));
  const fmd_config& c = h->cfg;
  const int H = c.hidden_size, I = c.intermediate_size, V = c.vocab_size;
  h->max_slots = max_slots;
  h->max_rows = max_rows_per_step;
  h->max_pages_per_slot = h->rope_len / kPageTokens;  // every position stays inside the RoPE table
  if (h->max_pages_per_slot < 1) return fail(h, FMD_ENOTSUP, "max_position_embeddings must be >= 64");
  const int64_t pages = (max_tokens_total + kPageTokens - 1) / kPageTokens + max_slots;
  if (pages > (1LL << 30)) return fail(h, FMD_ENOMEM, "KV pool too large");
  h->n_pages = (int)pages;
  int rc;
  // KV pool
  const size_t kv_elems = (size_t)c.num_hidden_layers * h->n_pages * 2 * c.num_key_value_heads * kPageTokens * kHeadDim;
  void* kvp;
  if ((rc = dev_alloc(h, kv_elems * 2, &kvp, &h->kv_bytes))) return rc;
  CK(cudaMemset(kvp, 0, kv_elems * 2));
  h->kv.base = kvp;
  h->kv.n_pages = h->n_pages;
  h->kv.max_pages_per_slot = h->max_pages_per_slot;
  h->kv.kv_heads = c.num_key_value_heads;
  {
    const uint64_t rows = (uint64_t)c.num_hidden_layers * h->n_pages * 2 * c.num_key_value_heads * kPageTokens;
    if (rows > (uint64_t)INT32_MAX) return fail(h, FMD_ENOTSUP, "KV pool too large for 32-bit TMA row coordinates");
    void* fn = nullptr;
    if ((rc = tmap_encoder(h, &fn))) return rc;
    auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    const cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kHeadDim * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)kPageTokens};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = encode(&h->kv_tmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, kvp, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(h, FMD_EIO, "cuTensorMapEncodeTiled failed: " + std::to_string((int)cr));
  }
  void* pt;
  if ((rc = dev_alloc(h, (size_t)max_slots * h->max_pages_per_slot * 4, &pt, &h->work_bytes))) return rc;
  CK(cudaMemset(pt, 0, (size_t)max_slots * h->max_pages_per_slot * 4));
  h->d_page_table = (int*)pt;
  h->kv.page_table = h->d_page_table;
  h->h_page_table.assign((size_t)max_slots * h->max_pages_per_slot, 0);
  h->free_pages.clear();
  for (int i = h->n_pages - 1; i >= 0; --i) h->free_pages.push_back(i);
  h->slot_cap.assign(max_slots, -1);
  h->slot_len.assign(max_slots, 0);
  h->slot_npages.assign(max_slots, 0);
  // work buffers
  const int R = h->max_rows;
  int max_split = 1;
  for (auto& L : h->layers) {
    for (const LinW* W : {&L.qkv, &L.o, &L.gate_up, &L.down}) max_split = std::max(max_split, W->split);
    for (const TcLinear* W : {&L.tc_qkv, &L.tc_o, &L.tc_gate_up, &L.tc_down})
      if (W->ok) max_split = std::max(max_split, W->split);
  }
  const int Nmax = std::max({h->qkvN(), 2 * I, H});
  h->split_stride = (size_t)std::max(R, 64) * Nmax;
  size_t part_elems = std::max({h->split_stride * max_split, (size_t)max_slots * V});
  // the persistent layer tail: Q8_0 weights, decode steps of <= 64 rows, one
  // CTA per SM with the layer's weights resident in shared memory
  h->chain_ok = false;
  if (h->q8 && h->chain_allowed && max_slots <= kChainMaxRows && c.num_hidden_layers > 0) {
    // every layer has the shapes of layer 0
    char why[160] = "";
    h->chain_ok = chain_plan(h->at, make_chain(h, 0), h->n_sm, max_slots, &h->chain_clusters, &h->chain_smem, why,
                             sizeof(why));
    cudaGetLastError();
    if (!h->chain_ok) std::fprintf(stderr, "[fmd] layer tail requested but unavailable: %s\n", why);
  }
  h->pb_max = R / kRowsPerPBlock + max_slots;
  h->di_max = (int)std::min<int64_t>((int64_t)max_slots * h->max_pages_per_slot,
                                     (int64_t)h->n_pages * kPageTokens / kDecodeItemTokens + 2 * max_slots + 1);
  h->di_grid = 296;
  const int HqD = h->Hq() * kHeadDim;
  void* p;
  auto A = [&](size_t bytes, void** dst) { return dev_alloc(h, bytes, dst, &h->work_bytes); };
  if ((rc = A((size_t)R * H * 2, &h->x))) return rc;
  if ((rc = A((size_t)R * H * 2, &h->xn))) return rc;
  if ((rc = A((size_t)R * HqD * 2, &h->qbuf))) return rc;
  if ((rc = A((size_t)R * HqD * 2, &h->ctx))) return rc;
  if ((rc = A((size_t)R * I * 2, &h->hbuf))) return rc;
  if ((rc = A((size_t)R * H * 2, &h->arena))) return rc;
  h->arena_rows = R;
  if ((rc = A(part_elems * 4, &p))) return rc;
  h->part = (float*)p;
  // decode attention split-segment partials: acc [2 * grid][2][128], then m/l [2 * grid][2][2]
  if ((rc = A(attn_decode_partial_floats(h->di_grid) * 4, &p))) return rc;
  h->pacc = (float*)p;
  h->pml = h->pacc + (size_t)2 * h->di_grid * 2 * kHeadDim;
  // a split decode step: the second half's attention partials, both halves' row counts
  h->split_ok = h->split_allowed && !h->chain_ok && max_slots >= 16 && max_slots % 2 == 0;
  if (h->split_ok) {
    if ((rc = A(attn_decode_partial_floats(h->di_grid) * 4, &p))) return rc;
    h->pacc2 = (float*)p;
    h->pml2 = h->pacc2 + (size_t)2 * h->di_grid * 2 * kHeadDim;
    if ((rc = A(2 * sizeof(PlanCounts), &p))) return rc;
    CK(cudaMemset(p, 0, 2 * sizeof(PlanCounts)));
    h->half_counts = (PlanCounts*)p;
    if (!h->stream2) CK(cudaStreamCreateWithFlags(&h->stream2, cudaStreamNonBlocking));
    if (!h->fork_ev) CK(cudaEventCreateWithFlags(&h->fork_ev, cudaEventDisableTiming));
    if (!h->join_ev) CK(cudaEventCreateWithFlags(&h->join_ev, cudaEventDisableTiming));
  }
  if ((rc = A((size_t)max_slots * V * 4, &p))) return rc;
  h->logits = (float*)p;
  if ((rc = A((size_t)max_slots * 4, &p))) return rc;
  h->next_ids = (int*)p;
  if ((rc = A((size_t)max_slots * (H / 64) * 4, &p))) return rc;
  h->ssq = (float*)p;
  if ((rc = A((size_t)max_slots * (V / 64) * 4, &p))) return rc;
  h->best_val = (float*)p;
  if ((rc = A((size_t)max_slots * (V / 64) * 4, &p))) return rc;
  h->best_idx = (int*)p;
  if ((rc = A((size_t)max_slots * c.num_key_value_heads * 4, &p))) return rc;
  CK(cudaMemset(p, 0, (size_t)max_slots * c.num_key_value_heads * 4));
  h->attn_counters = (int*)p;
  // status word, then the site of the first wait that gave up (TimeoutSite)
  if ((rc = A(4 * sizeof(int), &p))) return rc;
  CK(cudaMemset(p, 0, 4 * sizeof(int)));
  h->d_status = (int*)p;
  if (h->chain_ok) {
    const size_t n = (size_t)c.num_hidden_layers * kChainSyncInts * sizeof(int);
    if ((rc = A(n, &p))) return rc;
    CK(cudaMemset(p, 0, n));
    h->chain_sync = (int*)p;
  }
  h->layout.init(R, max_slots, h->pb_max, h->di_max);
  if ((rc = A(h->layout.total * 4, &p))) return rc;
  CK(cudaMemset(p, 0, h->layout.total * 4));
  h->d_plan = (int*)p;
  {
    // activation operands of the tensor-core projections: 128-row boxes
    void* fn = nullptr;
    if ((rc = tmap_encoder(h, &fn))) return rc;
    h->tc_ready = tc_make_map(fn, &h->amap_xn, h->xn, (uint64_t)H, (uint64_t)R, 128) &&
                  tc_make_map(fn, &h->amap_ctx, h->ctx, (uint64_t)HqD, (uint64_t)R, 128) &&
                  tc_make_map(fn, &h->amap_hbuf, h->hbuf, (uint64_t)I, (uint64_t)R, 128);
    h->q_ready = tc_make_map(fn, &h->qmap, h->qbuf, (uint64_t)HqD, (uint64_t)R, 64);
    if (!h->q_ready) return fail(h, FMD_EIO, "tensor map of the query buffer could not be encoded");
  }
  h->plan = h->layout.bind(h->d_plan);
  CK(cudaMallocHost((void**)&h->h_plan, h->layout.total * 4));
  std::memset(h->h_plan, 0, h->layout.total * 4);
  // engine slot arrays
  if ((rc = A((size_t)max_slots * 7 * 4, &p))) return rc;
  CK(cudaMemset(p, 0, (size_t)max_slots * 7 * 4));
  h->eng_slot = (int*)p;
  if ((rc = A((size_t)h->n_pages * 4, &p))) return rc;
  h->eng_free = (int*)p;
  if ((rc = A(sizeof(EngineCounters), &p))) return rc;
  h->eng_ctr = (EngineCounters*)p;
  CK(cudaMallocHost((void**)&h->h_ctr, sizeof(EngineCounters)));
  h->reserved = true;
  return FMD_OK;
}

int fmd_embed(fmd_handle* h, const int32_t* ids, int64_t n, void* out) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (!ids || !out || n < 0) return fail(h, FMD_EINVAL, "bad embed arguments");
  CK(cudaSetDevice(h->device));
  const int H = h->H();
  for (int64_t i = 0; i < n; ++i) {
    if (ids[i] < 0 || ids[i] >= h->cfg.vocab_size) return fail(h, FMD_EINVAL, "token id out of range");
    CK(cudaMemcpyAsync((char*)out + i * H * 2, (const char*)h->embed + (size_t)ids[i] * H * 2, H * 2,
                       cudaMemcpyDeviceToHost, h->stream));
  }
  return sync_check(h);
}

namespace {
// true when `p` is device memory of `device` (or managed memory)
bool on_device(const void* p, int device) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return (a.type == cudaMemoryTypeDevice && a.device == device) || a.type == cudaMemoryTypeManaged;
}
}  // namespace

int fmd_splice_audio(fmd_handle* h, const int32_t* token_ids, int64_t n_ids, const void* audio_embeds,
                     int64_t n_audio, int32_t audio_dtype, int32_t audio_token_id, void* out) {
  if (!h) return FMD_EINVAL;
  if (!h->loaded) return fail(h, FMD_EBUSY, "no weights loaded (fmd_load_weights)");
  const int H = h->H();
  if (!token_ids || n_ids < 1 || n_ids >= (1LL << 31) || !out || n_audio < 0 || (n_audio > 0 && !audio_embeds))
    return fail(h, FMD_EINVAL, "bad splice arguments");
  const bool f32 = audio_dtype == FMD_DT_F32;
  const bool act = (h->at == kBF16 && audio_dtype == FMD_DT_BF16) || (h->at == kF16 && audio_dtype == FMD_DT_F16);
  if (!f32 && !act) return fail(h, FMD_EINVAL, "audio embeddings must be f32 or the activation dtype");
  if (H % 8 != 0) return fail(h, FMD_ENOTSUP, "hidden size must be a multiple of 8");
  CK(cudaSetDevice(h->device));
  if (!on_device(out, h->device) || (n_audio > 0 && !on_device(audio_embeds, h->device)))
    return fail(h, FMD_EINVAL, "splice buffers must be device memory of the handle's device");
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(audio_embeds) & 15))
    return fail(h, FMD_EINVAL, "splice buffers must be 16-byte aligned");
  // one source code per position: the text id, or -(audio row) - 1, in
  // prompt order (the alternating text / audio runs of mod.rs:159-176)
  std::vector<int32_t> src((size_t)n_ids);
  int64_t used = 0;
  for (int64_t i = 0; i < n_ids; ++i) {
    const int32_t id = token_ids[i];
    if (id == audio_token_id) {
      src[i] = used < n_audio ? (int32_t)(-used - 1) : 0;
      ++used;
    } else {
      if (id < 0 || id >= h->cfg.vocab_size) return fail(h, FMD_EINVAL, "token id out of range");
      src[i] = id;
    }
  }
  if (used != n_audio)  // mod.rs:143-150
    return fail(h, FMD_EINVAL, "prompt has " + std::to_string(used) + " audio placeholders but the encoder produced " +
                                   std::to_string(n_audio) + " embeddings");
  const size_t bytes = (size_t)n_ids * sizeof(int32_t);
  if (h->splice_src.bytes < bytes) {
    if (h->splice_src.p) cudaFree(h->splice_src.p);
    h->splice_src = DevBuf{};
    if (cudaMalloc(&h->splice_src.p, bytes) != cudaSuccess) {
      cudaGetLastError();
      h->splice_src.p = nullptr;
      return fail(h, FMD_ENOMEM, "splice index allocation failed");
    }
    h->splice_src.bytes = bytes;
  }
  CK(cudaMemcpyAsync(h->splice_src.p, src.data(), bytes, cudaMemcpyHostToDevice, h->stream));
  launch_splice(h->at, (const int*)h->splice_src.p, n_ids, h->embed, audio_embeds, f32, H, out, h->stream);
  return sync_check(h);
}

int fmd_slot_open(fmd_handle* h, int32_t slot, int32_t capacity) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (slot < 0 || slot >= h->max_slots || capacity < 1) return fail(h, FMD_EINVAL, "bad slot or capacity");
  if (h->slot_cap[slot] >= 0) return fail(h, FMD_EBUSY, "slot already open");
  if (capacity > h->max_pages_per_slot * kPageTokens)
    return fail(h, FMD_EOVERFLOW, "capacity exceeds the RoPE table length");
  const int need = (capacity + kPageTokens - 1) / kPageTokens;
  if ((int)h->free_pages.size() < need) return fail(h, FMD_ENOMEM, "KV pool has too few free pages");
  h->slot_cap[slot] = capacity;
  h->slot_len[slot] = 0;
  CK(cudaSetDevice(h->device));
  if ((rc = ensure_pages(h, slot, capacity))) return rc;
  return sync_check(h);
}

int fmd_slot_release(fmd_handle* h, int32_t slot) {
  if (!h) return FMD_EINVAL;
  if (!h->reserved || slot < 0 || slot >= h->max_slots) return fail(h, FMD_EINVAL, "bad slot");
  for (int k = 0; k < h->slot_npages[slot]; ++k)
    h->free_pages.push_back(h->h_page_table[(size_t)slot * h->max_pages_per_slot + k]);
  h->slot_npages[slot] = 0;
  h->slot_cap[slot] = -1;
  h->slot_len[slot] = 0;
  return FMD_OK;
}

int fmd_slot_len(fmd_handle* h, int32_t slot, int32_t* len) {
  if (!h || !len) return FMD_EINVAL;
  if (!h->reserved || slot < 0 || slot >= h->max_slots || h->slot_cap[slot] < 0)
    return fail(h, FMD_EINVAL, "slot not open");
  *len = h->slot_len[slot];
  return FMD_OK;
}

int fmd_prefill(fmd_handle* h, int32_t n, const int32_t* slots, const int32_t* lens, const void* embeds,
                int32_t embeds_dtype, float* logits, int32_t* next_ids) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (n < 1 || n > h->max_slots || !slots || !lens || !embeds) return fail(h, FMD_EINVAL, "bad prefill arguments");
  CK(cudaSetDevice(h->device));
  int64_t total = 0;
  std::vector<char> seen(h->max_slots, 0);
  for (int i = 0; i < n; ++i) {
    const int s = slots[i];
    if (s < 0 || s >= h->max_slots || h->slot_cap[s] < 0) return fail(h, FMD_EINVAL, "prefill on a closed slot");
    if (seen[s]) return fail(h, FMD_EINVAL, "slot listed twice");
    seen[s] = 1;
    if (lens[i] < 1) return fail(h, FMD_EINVAL, "empty prompt");
    if (h->slot_len[s] + lens[i] > h->slot_cap[s])
      return fail(h, FMD_EOVERFLOW, "kv cache overflow: " + std::to_string(h->slot_len[s]) + " + " +
                                        std::to_string(lens[i]) + " exceeds capacity " +
                                        std::to_string(h->slot_cap[s]));
    total += lens[i];
  }
  const size_t rowb = (size_t)h->H() * (embeds_dtype == FMD_DT_F32 ? 4 : 2);
  // Passes of up to max_rows rows; a sequence may span passes (chunked prefill).
  std::vector<int> done(n, 0);
  std::vector<int64_t> src_off(n, 0);
  for (int i = 1; i < n; ++i) src_off[i] = src_off[i - 1] + lens[i - 1];
  int remaining = n;
  std::vector<int> order;
  std::vector<uint16_t> act;
  release_graph(h);
  while (remaining > 0) {
    HostPlan hp(h);
    order.clear();
    std::vector<std::pair<int, int>> segs;  // (seq, rows)
    int rows = 0;
    for (int i = 0; i < n && rows < h->max_rows; ++i) {
      const int left = lens[i] - done[i];
      if (left == 0) continue;
      const int take = std::min(left, h->max_rows - rows);
      segs.push_back({i, take});
      rows += take;
    }
    // stage the embeddings of this pass into the arena, back to back
    int arow = 0;
    for (auto& sg : segs) {
      const int i = sg.first, take = sg.second;
      const char* src = (const char*)embeds + (size_t)(src_off[i] + done[i]) * rowb;
      if ((rc = convert_rows_to_act(h, src, embeds_dtype, take, act))) return rc;
      CK(cudaMemcpyAsync((char*)h->arena + (size_t)arow * h->H() * 2, act.data(), act.size() * 2,
                         cudaMemcpyHostToDevice, h->stream));
      const int s = slots[i];
      const bool last = done[i] + take == lens[i];
      hp.add_prefill(s, h->slot_len[s], take, arow, last);
      if (last) order.push_back(i);
      arow += take;
      CK(cudaStreamSynchronize(h->stream));  // `act` is reused
    }
    if ((rc = hp.commit())) return rc;
    run_forward(h, logits ? h->logits : nullptr, h->arena);
    for (auto& sg : segs) {
      const int i = sg.first;
      h->slot_len[slots[i]] += sg.second;
      done[i] += sg.second;
      if (done[i] == lens[i]) --remaining;
    }
    if ((rc = copy_outputs(h, (int)order.size(), order, logits, next_ids))) return rc;
  }
  return FMD_OK;
}

int fmd_decode_step(fmd_handle* h, int32_t n, const int32_t* slots, const int32_t* ids, float* logits,
                    int32_t* next_ids) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (n < 1 || n > h->max_slots || !slots || !ids) return fail(h, FMD_EINVAL, "bad decode arguments");
  CK(cudaSetDevice(h->device));
  std::vector<char> seen(h->max_slots, 0);
  for (int i = 0; i < n; ++i) {
    const int s = slots[i];
    if (s < 0 || s >= h->max_slots || h->slot_cap[s] < 0) return fail(h, FMD_EINVAL, "decode on a closed slot");
    if (seen[s]) return fail(h, FMD_EINVAL, "slot listed twice");
    seen[s] = 1;
    if (ids[i] < 0 || ids[i] >= h->cfg.vocab_size) return fail(h, FMD_EINVAL, "token id out of range");
    if (h->slot_len[s] + 1 > h->slot_cap[s])
      return fail(h, FMD_EOVERFLOW, "kv cache overflow: " + std::to_string(h->slot_len[s]) +
                                        " + 1 exceeds capacity " + std::to_string(h->slot_cap[s]));
  }
  release_graph(h);
  HostPlan hp(h);
  std::vector<int> order(n);
  for (int i = 0; i < n; ++i) {
    hp.add_decode(slots[i], h->slot_len[slots[i]], ids[i]);
    order[i] = i;
  }
  if ((rc = hp.commit())) return rc;
  run_forward(h, logits ? h->logits : nullptr, h->arena, true);
  for (int i = 0; i < n; ++i) h->slot_len[slots[i]] += 1;
  return copy_outputs(h, n, order, logits, next_ids);
}

// ---- continuous-batching engine ------------------------------------------------------
int fmd_engine_load(fmd_handle* h, const fmd_request* reqs, int32_t n_reqs, const void* embeds, int64_t embed_rows,
                    int32_t embeds_dtype) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (n_reqs < 1 || !reqs || !embeds || embed_rows < 1 || embed_rows >= (1LL << 31))
    return fail(h, FMD_EINVAL, "bad engine queue");
  CK(cudaSetDevice(h->device));
  int max_new = 1;
  for (int i = 0; i < n_reqs; ++i) {
    if (reqs[i].prompt_len < 1 || reqs[i].embed_row < 0 || reqs[i].embed_row + reqs[i].prompt_len > embed_rows)
      return fail(h, FMD_EINVAL, "request " + std::to_string(i) + " reads outside the embedding arena");
    max_new = std::max(max_new, reqs[i].max_new_tokens);
  }
  for (int s = 0; s < h->max_slots; ++s)
    if (h->slot_cap[s] >= 0) return fail(h, FMD_EBUSY, "close operator-mode slots before running the engine");
  release_graph(h);
  for (DevBuf* b : {&h->eng_reqs, &h->eng_arena, &h->eng_tokens, &h->eng_results}) {
    if (b->p) cudaFree(b->p);
    b->p = nullptr;
    b->bytes = 0;
  }
  auto alloc = [&](DevBuf& b, size_t bytes) -> int {
    cudaError_t e = cudaMalloc(&b.p, bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      b.p = nullptr;
      return fail(h, FMD_ENOMEM, "engine buffer allocation failed");
    }
    b.bytes = bytes;
    return FMD_OK;
  };
  static_assert(sizeof(fmd_request) == sizeof(DevRequest), "request layout");
  if ((rc = alloc(h->eng_reqs, sizeof(DevRequest) * n_reqs))) return rc;
  CK(cudaMemcpy(h->eng_reqs.p, reqs, sizeof(DevRequest) * n_reqs, cudaMemcpyHostToDevice));
  const size_t arena_bytes = (size_t)embed_rows * h->H() * 2;
  if ((rc = alloc(h->eng_arena, arena_bytes))) return rc;
  // convert in slices to bound host memory; an arena already in the
  // activation dtype is copied straight from the caller's (possibly pinned)
  // buffer
  const size_t rowb = (size_t)h->H() * (embeds_dtype == FMD_DT_F32 ? 4 : 2);
  const bool same = (h->at == kBF16 && embeds_dtype == FMD_DT_BF16) || (h->at == kF16 && embeds_dtype == FMD_DT_F16);
  // an arena already in device memory (e.g. written by fmd_splice_audio) is
  // copied on the device; it must be in the activation dtype
  const bool dev_arena = on_device(embeds, h->device);
  if (dev_arena && !same) return fail(h, FMD_EINVAL, "a device-memory arena must be in the activation dtype");
  if (same) CK(cudaMemcpy(h->eng_arena.p, embeds, arena_bytes, dev_arena ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
  std::vector<uint16_t> act;
  for (int64_t r = 0; !same && r < embed_rows; r += 65536) {
    const int64_t nr = std::min<int64_t>(65536, embed_rows - r);
    if ((rc = convert_rows_to_act(h, (const char*)embeds + r * rowb, embeds_dtype, nr, act))) return rc;
    CK(cudaMemcpy((char*)h->eng_arena.p + (size_t)r * h->H() * 2, act.data(), act.size() * 2,
                  cudaMemcpyHostToDevice));
  }
  h->eng_n_reqs = n_reqs;
  h->eng_tok_stride = max_new;
  if ((rc = alloc(h->eng_tokens, (size_t)n_reqs * max_new * 4))) return rc;
  if ((rc = alloc(h->eng_results, sizeof(DevResult) * n_reqs))) return rc;
  CK(cudaMemset(h->eng_results.p, 0, sizeof(DevResult) * n_reqs));
  return FMD_OK;
}

namespace {
EngineDev make_engine_dev(fmd_handle* h, int max_batch, int chunk, int allow_prefill = 1) {
  EngineDev e{};
  e.allow_prefill = allow_prefill;
  e.n_reqs = h->eng_n_reqs;
  e.n_pages = h->n_pages;
  e.consume_only = 0;
  e.max_batch = max_batch;
  e.prefill_chunk = chunk;
  e.max_rows = h->max_rows;
  e.split_rows = h->split_ok ? h->max_slots / 2 : 0;
  e.max_pages_per_slot = h->max_pages_per_slot;
  e.eos = h->cfg.eos_token_id;
  e.vocab = h->cfg.vocab_size;
  e.page_tokens = kPageTokens;
  e.tok_stride = h->eng_tok_stride;
  e.reqs = (const DevRequest*)h->eng_reqs.p;
  const int S = h->max_slots;
  e.slot_state = h->eng_slot;
  e.slot_req = h->eng_slot + S;
  e.slot_len = h->eng_slot + 2 * S;
  e.slot_pdone = h->eng_slot + 3 * S;
  e.slot_ngen = h->eng_slot + 4 * S;
  e.slot_last = h->eng_slot + 5 * S;
  e.slot_npages = h->eng_slot + 6 * S;
  e.free_stack = h->eng_free;
  e.page_table = h->d_page_table;
  e.out_tokens = (int*)h->eng_tokens.p;
  e.results = (DevResult*)h->eng_results.p;
  e.ctr = h->eng_ctr;
  e.next_ids = h->next_ids;
  e.plan = h->plan;
  return e;
}
}  // namespace

int fmd_engine_start(fmd_handle* h, int32_t max_batch, int32_t prefill_chunk) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (!h->eng_reqs.p) return fail(h, FMD_EBUSY, "no queue loaded (fmd_engine_load)");
  if (max_batch < 1 || max_batch > h->max_slots) return fail(h, FMD_EINVAL, "max_batch exceeds reserved slots");
  if (prefill_chunk < 1 || max_batch + prefill_chunk > h->max_rows)
    return fail(h, FMD_EINVAL, "max_batch + prefill_chunk exceeds max_rows_per_step");
  for (int s = 0; s < h->max_slots; ++s)
    if (h->slot_cap[s] >= 0) return fail(h, FMD_EBUSY, "close operator-mode slots before running the engine");
  CK(cudaSetDevice(h->device));
  h->engine_started = false;
  // reset engine state: all slots free, all pages on the free stack, empty plan
  CK(cudaMemsetAsync(h->eng_slot, 0, (size_t)h->max_slots * 7 * 4, h->stream));
  std::vector<int> fs(h->n_pages);
  for (int i = 0; i < h->n_pages; ++i) fs[i] = h->n_pages - 1 - i;
  CK(cudaMemcpyAsync(h->eng_free, fs.data(), fs.size() * 4, cudaMemcpyHostToDevice, h->stream));
  EngineCounters c{};
  c.free_top = h->n_pages;
  *h->h_ctr = c;
  CK(cudaMemcpyAsync(h->eng_ctr, h->h_ctr, sizeof(c), cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemsetAsync(h->d_plan, 0, h->layout.total * 4, h->stream));
  CK(cudaMemsetAsync(h->eng_results.p, 0, sizeof(DevResult) * h->eng_n_reqs, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  if (h->attn_events.empty()) {
    h->attn_events.resize(4);
    for (auto& e : h->attn_events) CK(cudaEventCreate(&e));
    CK(cudaEventCreate(&h->win_begin));
    CK(cudaEventCreate(&h->win_end));
  }
  if (trace_enabled()) {
    // launch tracing synchronises after every kernel, which a stream capture
    // forbids: the traced engine launches each step's kernels directly
    release_graph(h);
    h->graph_batch = max_batch;
    h->graph_chunk = prefill_chunk;
  } else if (!h->graph_exec || h->graph_batch != max_batch || h->graph_chunk != prefill_chunk) {
    release_graph(h);
    // two step graphs: "M" may carry a prefill chunk (split-K projections),
    // "D" is decode-only (fused decode projections, no prefill attention)
    for (int mixed = 1; mixed >= 0; --mixed) {
      const EngineDev e = make_engine_dev(h, max_batch, prefill_chunk, mixed);
      cudaGraph_t g;
      CK(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
      h->record_attn_events = true;
      launch_schedule(e, h->stream);
      if (mixed)
        run_forward(h, nullptr, h->eng_arena.p);
      else
        run_forward(h, nullptr, h->eng_arena.p, true);
      h->record_attn_events = false;
      CK(cudaStreamEndCapture(h->stream, &g));
      {
        // kernels per replay of this graph (reported in fmd_stats)
        size_t n_nodes = 0;
        CK(cudaGraphGetNodes(g, nullptr, &n_nodes));
        std::vector<cudaGraphNode_t> nodes(n_nodes);
        CK(cudaGraphGetNodes(g, nodes.data(), &n_nodes));
        int64_t kernels = 0;
        for (cudaGraphNode_t nd : nodes) {
          cudaGraphNodeType ty;
          CK(cudaGraphNodeGetType(nd, &ty));
          kernels += ty == cudaGraphNodeTypeKernel;
        }
        (mixed ? h->graph_kernels_mixed : h->graph_kernels_decode) = kernels;
      }
      if (h->launch_refused) {
        cudaGraphDestroy(g);
        return sync_check(h);
      }
      cudaError_t ie = cudaGraphInstantiate(mixed ? &h->graph_exec : &h->graph_dec, g, 0);
      cudaGraphDestroy(g);
      if (ie != cudaSuccess) return fail(h, FMD_EIO, std::string("graph instantiate: ") + cudaGetErrorString(ie));
    }
    h->graph_batch = max_batch;
    h->graph_chunk = prefill_chunk;
  }
  h->first_block = true;
  h->watch = ProgressWatch(kEngineIdlePolls);
  h->engine_started = true;
  return FMD_OK;
}

int fmd_engine_step(fmd_handle* h, int64_t max_steps, fmd_stats* stats) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (!h->engine_started || (!trace_enabled() && (!h->graph_exec || !h->graph_dec)))
    return fail(h, FMD_EBUSY, "engine not started (fmd_engine_start)");
  if (max_steps < 0) return fail(h, FMD_EINVAL, "negative step count");
  CK(cudaSetDevice(h->device));
  const auto t0 = std::chrono::steady_clock::now();
  CK(cudaMemcpyAsync(h->h_ctr, h->eng_ctr, sizeof(EngineCounters), cudaMemcpyDeviceToHost, h->stream));
  if ((rc = sync_check(h))) return rc;
  const long long tokens0 = h->h_ctr->gen_tokens;
  bool finished = h->h_ctr->done >= h->eng_n_reqs;
  int64_t launched = 0;
  ProgressWatch& watch = h->watch;
  CK(cudaEventRecord(h->win_begin, h->stream));
  int64_t mixed_launched = 0;
  while (!finished && launched < max_steps) {
    const int64_t k = std::min<int64_t>(kEngineCheckEvery, max_steps - launched);
    // Steps that may carry a prefill chunk ("M") first, as many as the prompt
    // rows pending at the last poll need, then decode-only steps ("D").
    // Before the first poll everything admitted is still to be prefilled.
    int64_t n_m = k;
    if (!h->first_block)
      n_m = std::min<int64_t>(k, (h->h_ctr->pending_prefill + h->graph_chunk - 1) / h->graph_chunk);
    for (int64_t i = 0; i < k; ++i) {
      if (trace_enabled()) {
        const EngineDev e = make_engine_dev(h, h->graph_batch, h->graph_chunk, i < n_m ? 1 : 0);
        launch_schedule(e, h->stream);
        trace(h, "schedule", -1);
        run_forward(h, nullptr, h->eng_arena.p, i >= n_m);
      } else {
        CK(cudaGraphLaunch(i < n_m ? h->graph_exec : h->graph_dec, h->stream));
      }
    }
    launched += k;
    mixed_launched += n_m;
    h->first_block = false;
    CK(cudaMemcpyAsync(h->h_ctr, h->eng_ctr, sizeof(EngineCounters), cudaMemcpyDeviceToHost, h->stream));
    if ((rc = sync_check(h))) return rc;
    finished = h->h_ctr->done >= h->eng_n_reqs;
    // every live step emits a token or consumes prompt rows; a run of checks
    // without either means the queue cannot make progress
    const bool stalled = watch.stalled(h->h_ctr->gen_tokens, h->h_ctr->prefill_tokens, h->h_ctr->done);
    if (!finished && stalled)
      return fail(h, FMD_ETIMEDOUT, "engine made no progress for " +
                                        std::to_string(kEngineIdlePolls * kEngineCheckEvery) + " steps (requests done " +
                                        std::to_string(h->h_ctr->done) + ")");
  }
  // a consume-only scheduler pass books the samples of the last step run
  EngineDev e = make_engine_dev(h, h->graph_batch, h->graph_chunk);
  e.consume_only = 1;
  CK(cudaEventRecord(h->win_end, h->stream));
  const long long kv_last = h->h_ctr->last_kv_tokens, rows_last = h->h_ctr->last_decode_rows;
  const long long kv_lo_last = h->h_ctr->last_kv_tokens_lo, rows_lo_last = h->h_ctr->last_rows_lo;
  launch_schedule(e, h->stream);
  CK(cudaMemcpyAsync(h->h_ctr, h->eng_ctr, sizeof(EngineCounters), cudaMemcpyDeviceToHost, h->stream));
  if ((rc = sync_check(h))) return rc;
  // the consume-only pass leaves an empty plan; the next graph step re-plans
  // from the slot state, so the window boundary changes no result.
  float win_ms = 0.f;
  if (launched > 0) CK(cudaEventElapsedTime(&win_ms, h->win_begin, h->win_end));
  double attn_ms = 0.0, lm_ms = 0.0;
  if (launched > 0 && !trace_enabled()) {
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, h->attn_events[0], h->attn_events[1]));
    attn_ms = ms;
    CK(cudaEventElapsedTime(&ms, h->attn_events[2], h->attn_events[3]));
    lm_ms = ms;
  }
  const auto t1 = std::chrono::steady_clock::now();
  if (stats) {
    std::memset(stats, 0, sizeof(*stats));
    stats->steps = h->h_ctr->steps;
    stats->generated_tokens = h->h_ctr->gen_tokens;
    stats->prefill_tokens = h->h_ctr->prefill_tokens;
    stats->requests_done = h->h_ctr->done;
    stats->generate_seconds = std::chrono::duration<double>(t1 - t0).count();
    stats->device_status = h->h_ctr->status;
    stats->window_steps = launched;
    stats->window_tokens = h->h_ctr->gen_tokens - tokens0;
    stats->window_device_ms = win_ms;
    stats->attn_decode_ms = attn_ms;
    stats->lm_head_ms = lm_ms;
    // a split step's probe times the first half's attention
    stats->attn_kv_tokens = h->split_ok ? kv_lo_last : kv_last;
    stats->attn_rows = h->split_ok ? rows_lo_last : rows_last;
    stats->window_mixed_steps = mixed_launched;
    stats->graph_kernels_mixed = h->graph_kernels_mixed;
    stats->graph_kernels_decode = h->graph_kernels_decode;
  }
  return FMD_OK;
}

int fmd_engine_run(fmd_handle* h, int32_t max_batch, int32_t prefill_chunk, int64_t max_steps, fmd_stats* stats) {
  int rc = fmd_engine_start(h, max_batch, prefill_chunk);
  if (rc) return rc;
  return fmd_engine_step(h, max_steps, stats);
}

int fmd_engine_fetch(fmd_handle* h, int32_t* tokens, int32_t token_stride, fmd_result* results) {
  if (!h) return FMD_EINVAL;
  if (!h->eng_reqs.p) return fail(h, FMD_EBUSY, "no queue loaded");
  CK(cudaSetDevice(h->device));
  if (tokens) {
    if (token_stride < h->eng_tok_stride) return fail(h, FMD_EINVAL, "token_stride smaller than the max budget");
    CK(cudaMemcpy2D(tokens, (size_t)token_stride * 4, h->eng_tokens.p, (size_t)h->eng_tok_stride * 4,
                    (size_t)h->eng_tok_stride * 4, h->eng_n_reqs, cudaMemcpyDeviceToHost));
  }
  if (results) CK(cudaMemcpy(results, h->eng_results.p, sizeof(DevResult) * h->eng_n_reqs, cudaMemcpyDeviceToHost));
  return FMD_OK;
}

int fmd_generate(fmd_handle* h, const fmd_request* reqs, int32_t n_reqs, const void* embeds, int64_t embed_rows,
                 int32_t embeds_dtype, int32_t max_batch, int32_t prefill_chunk, int32_t* tokens, int32_t token_stride,
                 fmd_result* results, fmd_stats* stats) {
  int rc = fmd_engine_load(h, reqs, n_reqs, embeds, embed_rows, embeds_dtype);
  if (rc) return rc;
  if ((rc = fmd_engine_run(h, max_batch, prefill_chunk, INT64_MAX / 2, stats))) return rc;
  return fmd_engine_fetch(h, tokens, token_stride, results);
}

// ---- inspection ------------------------------------------------------------------------
int fmd_debug_weight(fmd_handle* h, int32_t layer, int32_t which, float* out, int64_t out_elems) {
  if (!h || !out) return FMD_EINVAL;
  if (!h->loaded) return fail(h, FMD_EBUSY, "no weights");
  const LinW* W = nullptr;
  if (which == 4) {
    W = &h->lm_head;
  } else {
    if (layer < 0 || layer >= (int)h->layers.size()) return fail(h, FMD_EINVAL, "bad layer");
    const LayerDev& L = h->layers[layer];
    W = which == 0 ? &L.qkv : which == 1 ? &L.o : which == 2 ? &L.gate_up : which == 3 ? &L.down : nullptr;
  }
  if (!W) return fail(h, FMD_EINVAL, "bad weight selector");
  const size_t n = (size_t)W->N * W->K;
  if (out_elems < (int64_t)n) return fail(h, FMD_EINVAL, "output too small");
  CK(cudaSetDevice(h->device));
  float* d;
  CK(cudaMalloc(&d, n * 4));
  launch_dequant(h->at, *W, d, h->stream);
  cudaError_t e = cudaMemcpyAsync(out, d, n * 4, cudaMemcpyDeviceToHost, h->stream);
  cudaError_t e2 = cudaStreamSynchronize(h->stream);
  cudaFree(d);
  if (e != cudaSuccess || e2 != cudaSuccess) return fail(h, FMD_EIO, "dequant copy failed");
  if (which == 2) {  // gate/up are stored interleaved in 32-row groups: restore [gate; up]
    std::vector<float> tmp(out, out + n);
    const int half = W->N / 2;
    for (int r = 0; r < W->N; ++r)
      std::memcpy(out + (size_t)r * W->K, tmp.data() + (size_t)((r / half) ? up_col(r % half) : gate_col(r % half)) * W->K,
                  sizeof(float) * W->K);
  }
  return FMD_OK;
}

int fmd_debug_kv(fmd_handle* h, int32_t slot, int32_t layer, int32_t pos, int32_t n, void* k_out, void* v_out) {
  if (!h || !k_out || !v_out) return FMD_EINVAL;
  if (!h->reserved || slot < 0 || slot >= h->max_slots || layer < 0 || layer >= h->cfg.num_hidden_layers || pos < 0 ||
      n < 0 || (int64_t)(pos + n) > (int64_t)h->slot_npages[slot] * kPageTokens)
    return fail(h, FMD_EINVAL, "bad kv range");
  CK(cudaSetDevice(h->device));
  const int Hkv = h->Hkv();
  const size_t rowb = kHeadDim * 2;
  for (int i = 0; i < n; ++i) {
    const int p = pos + i;
    const int page = h->h_page_table[(size_t)slot * h->max_pages_per_slot + p / kPageTokens];
    for (int kvi = 0; kvi < 2; ++kvi)
      for (int hh = 0; hh < Hkv; ++hh) {
        const char* src = (const char*)h->kv.base + (h->kv.elem_offset(layer, page, kvi, hh) + (size_t)(p % kPageTokens) * kHeadDim) * 2;
        char* dst = (char*)(kvi ? v_out : k_out) + ((size_t)i * Hkv + hh) * rowb;
        CK(cudaMemcpyAsync(dst, src, rowb, cudaMemcpyDeviceToHost, h->stream));
      }
  }
  return sync_check(h);
}

int fmd_debug_wait_timeout(fmd_handle* h, int32_t limit) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (limit < 1) return fail(h, FMD_EINVAL, "limit must be >= 1");
  CK(cudaSetDevice(h->device));
  launch_wait_probe((uint32_t)limit, h->d_status, h->stream);
  return sync_check(h);
}

int fmd_debug_mma_issue(fmd_handle* h, int32_t form, int32_t n, int32_t iters, double* cycles_per_mma) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (!cycles_per_mma || (form != 0 && form != 1) || n < 16 || n > 256 || n % 16 || iters < 8 || iters > (1 << 20) ||
      iters % 8)
    return fail(h, FMD_EINVAL, "form must be 0 or 1, n a multiple of 16 in [16, 256], iters a multiple of 8 in [8, 2^20]");
  CK(cudaSetDevice(h->device));
  long long* d = nullptr;
  CK(cudaMalloc((void**)&d, sizeof(long long)));
  long long c = -1;
  cudaError_t e = launch_mma_issue_probe(form, n, iters, d, h->d_status, h->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&c, d, sizeof(c), cudaMemcpyDeviceToHost, h->stream);
  rc = e != cudaSuccess ? fail(h, FMD_EIO, cudaGetErrorString(e)) : sync_check(h);
  cudaFree(d);
  if (rc) return rc;
  *cycles_per_mma = c < 0 ? -1.0 : (double)c / iters;
  return FMD_OK;
}

int fmd_debug_paths(const fmd_handle* h, int32_t* flags) {
  if (!h || !flags) return FMD_EINVAL;
  *flags = (h->chain_ok ? FMD_PATH_LAYER_TAIL : 0) | (h->tc_ready && h->proj_allowed ? FMD_PATH_PROJ_TC : 0) |
           (h->lm_tc_used ? FMD_PATH_LM_HEAD_TC : 0) |
           (h->pf_pp_allowed ? FMD_PATH_PREFILL_PP : 0) | (h->split_ok ? FMD_PATH_DECODE_SPLIT : 0);
  return FMD_OK;
}

int fmd_q8_0_quantize(const float* src, int64_t rows, int64_t cols, void* blocks) {
  if (!src || !blocks || rows < 0 || cols % 32) return FMD_EINVAL;
  std::vector<int8_t> qs((size_t)rows * cols);
  std::vector<uint16_t> d((size_t)rows * (cols / 32));
  quantize_rows(src, rows, cols, qs.data(), d.data());
  uint8_t* b = (uint8_t*)blocks;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t k = 0; k < cols / 32; ++k) {
      uint8_t* blk = b + (r * (cols / 32) + k) * 34;
      std::memcpy(blk, &d[r * (cols / 32) + k], 2);
      std::memcpy(blk + 2, &qs[r * cols + k * 32], 32);
    }
  return FMD_OK;
}

}  // extern "C"
