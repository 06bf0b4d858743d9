// Device-side data structures shared by the kernels, the scheduler and the
// host runtime, plus the launchers the runtime calls.
#pragma once

#include <utility>

#include <cuda.h>

#include "fmd_common.cuh"

namespace fmd {

// Counts of one forward pass ("step"). Written by the host (operator entry
// points) or by the device scheduler (continuous-batching engine).
struct PlanCounts {
  int n_rows;     // token rows in this pass
  int n_decode;   // rows [0, n_decode) are one-token decode rows
  int n_sample;   // rows whose logits / greedy id are wanted
  int n_pblocks;  // prefill attention blocks (<= 32 consecutive rows of one slot)
  int n_ditems;   // decode attention split items
  int finished;   // engine: every request is done
  int pad0, pad1;
};

// Per-pass token plan. All arrays live in one device buffer (`PlanLayout`).
struct Plan {
  PlanCounts* counts;
  int* row_slot;     // [R] sequence slot of each row
  int* row_pos;      // [R] absolute position (= KV index the row writes)
  int* row_tok;      // [R] token id, or -1: take the row from the embedding arena
  int* row_emb;      // [R] arena row when row_tok < 0
  int* sample_row;   // [B] rows that produce logits, in output order
  int* sample_slot;  // [B] their slots (engine bookkeeping)
  int* pb_row0;      // [PB] first row of a prefill attention block
  int* pb_n;         // [PB] rows in the block (1..32)
  int* di_row;       // [DI] decode row of a split item
  int* di_start;     // [DI] first key position of the item
  int* di_end;       // [DI] one past the last key position
  int* drow_item0;   // [R]  first split item of a decode row
  int* drow_nitems;  // [R]  split items of a decode row
};

// Sizes of the plan arrays and their offsets (in ints) inside one buffer.
struct PlanLayout {
  int R, B, PB, DI;
  size_t off_counts, off_row_slot, off_row_pos, off_row_tok, off_row_emb, off_sample_row, off_sample_slot,
      off_pb_row0, off_pb_n, off_di_row, off_di_start, off_di_end, off_drow_item0, off_drow_nitems, total;
  void init(int r, int b, int pb, int di) {
    R = r; B = b; PB = pb; DI = di;
    size_t o = 0;
    off_counts = o; o += sizeof(PlanCounts) / sizeof(int);
    off_row_slot = o; o += R;
    off_row_pos = o; o += R;
    off_row_tok = o; o += R;
    off_row_emb = o; o += R;
    off_sample_row = o; o += B;
    off_sample_slot = o; o += B;
    off_pb_row0 = o; o += PB;
    off_pb_n = o; o += PB;
    off_di_row = o; o += DI;
    off_di_start = o; o += DI;
    off_di_end = o; o += DI;
    off_drow_item0 = o; o += R;
    off_drow_nitems = o; o += R;
    total = o;
  }
  Plan bind(int* base) const {
    Plan p;
    p.counts = reinterpret_cast<PlanCounts*>(base + off_counts);
    p.row_slot = base + off_row_slot;
    p.row_pos = base + off_row_pos;
    p.row_tok = base + off_row_tok;
    p.row_emb = base + off_row_emb;
    p.sample_row = base + off_sample_row;
    p.sample_slot = base + off_sample_slot;
    p.pb_row0 = base + off_pb_row0;
    p.pb_n = base + off_pb_n;
    p.di_row = base + off_di_row;
    p.di_start = base + off_di_start;
    p.di_end = base + off_di_end;
    p.drow_item0 = base + off_drow_item0;
    p.drow_nitems = base + off_drow_nitems;
    return p;
  }
};

constexpr int kMaxPrefillBlocks = 1024;  // prefill attention blocks one pass may carry
constexpr int kRowsPerPBlock = 64;   // query rows per prefill attention block (x 2 heads = one 128-row MMA tile)
constexpr int kDecodeItemTokens = 256;  // keys per decode attention split item

// Paged KV pool: [layer][page][k|v][kv_head][kPageTokens][kHeadDim], act dtype.
struct KvView {
  void* base;
  const int* page_table;  // [max_slots][max_pages_per_slot]
  int n_pages;
  int max_pages_per_slot;
  int kv_heads;
  __host__ __device__ size_t elem_offset(int layer, int page, int kv, int head) const {
    return ((((size_t)layer * n_pages + page) * 2 + kv) * kv_heads + head) * (size_t)(kPageTokens * kHeadDim);
  }
};

// A projection stored on the device: Q8_0 as int8 [N][K] + f16 scales
// [N][K/32], or dense activation-dtype [N][K].
struct LinW {
  int N = 0, K = 0;
  bool q8 = false;
  const int8_t* qs = nullptr;
  const uint16_t* d = nullptr;
  const void* w = nullptr;
  int split = 1;  // K splits used when a pass has <= 64 rows
  const uint8_t* pk = nullptr;  // decode-packed tiles of the decode-step GEMV
};

// gate/up projections are stored with their rows interleaved in 32-row
// groups ([g0..g31, u0..u31, g32..g63, u32..u63, ...]) so a 64-row tile holds
// matching gate and up features; output column of gate / up feature i:
__host__ __device__ inline int gate_col(int i) { return (i >> 5) * 64 + (i & 31); }
__host__ __device__ inline int up_col(int i) { return gate_col(i) + 32; }

// Epilogue selector and arguments of the decode-step GEMV (fmd_gemv.cu).
enum GemvEpiKind { kGemvQkv = 0, kGemvResid = 1, kGemvSwiglu = 2, kGemvLogits = 3 };
struct GemvEpi {
  // normalised input (NORM variants): xn = x * rsqrt(sum(ssq[row]) / K + eps) * norm_w
  const float* ssq = nullptr;  // [rows][ssq_tiles] per-tile sums of squares of x
  const void* norm_w = nullptr;
  int ssq_tiles = 0;
  float eps = 0.f;
  void* x = nullptr;         // kGemvResid: residual stream [rows][N], updated in place
  float* ssq_out = nullptr;  // kGemvResid: [rows][N / 64] sums of squares of the new x
  void* h = nullptr;         // kGemvSwiglu: [rows][I]
  int I = 0;
  Plan plan{};               // kGemvQkv
  const void* qn_w = nullptr;
  const void* kn_w = nullptr;
  const void* cos = nullptr;
  const void* sin = nullptr;
  void* q_out = nullptr;
  KvView kv{};
  int layer = 0, Hq = 0, Hkv = 0;
  float* logits = nullptr;    // kGemvLogits: optional f32 logits [rows][N]
  float* best_val = nullptr;  // kGemvLogits: per-tile (max, index) per row
  int* best_idx = nullptr;
};

// The persistent tail of a decode layer (fmd_chain.cu): o_proj (+ residual)
// -> gate/up (post-attention RMSNorm, SwiGLU) -> down (+ residual) -> the next
// layer's qkv (its input RMSNorm, q/k norm, RoPE, KV write) in one launch of
// 8-CTA clusters. A phase is one projection in the decode-packed Q8_0 layout
// of the GEMV: `ft`-feature tiles split `S` (= 8) ways along K.
struct ChainPhase {
  const uint8_t* pk = nullptr;
  int N = 0, K = 0, ft = 0, S = 0;
};
constexpr int kChainMaxRows = 32;  // decode rows the layer tail serves
constexpr int kChainSyncInts = 4;  // per layer: the 3 grid-barrier counters (+1 spare), zero at launch
struct ChainArgs {
  ChainPhase ph[4];            // o, gate_up, down, next layer's qkv
  int n_phases = 4;            // 3 for the last layer (no qkv)
  const int* n_rows_ptr = nullptr;
  const void* ctx = nullptr;   // [rows][Hq x 128] attention output
  void* x = nullptr;           // [rows][H] residual stream
  void* h = nullptr;           // [rows][I] SwiGLU output
  float* ssq = nullptr;        // [rows][ssq_tiles] per-64-feature sums of squares of x
  int ssq_tiles = 0;
  float eps = 0.f;
  const void* post_norm = nullptr;  // this layer's post-attention norm
  const void* in_norm = nullptr;    // the next layer's input norm, q_norm, k_norm
  const void* qn_w = nullptr;
  const void* kn_w = nullptr;
  const void* cos = nullptr;
  const void* sin = nullptr;
  void* q_out = nullptr;
  KvView kv{};
  Plan plan{};
  int layer = 0;               // the next layer (its KV cache is written)
  int Hq = 0, Hkv = 0, H = 0, I = 0;
  int* sync = nullptr;         // this layer's kChainSyncInts counters, zero at launch
  int* status = nullptr;
};

// Epilogue of the persistent mixed-step projection GEMM (fmd_proj_tc.cu).
enum ProjEpiKind { kProjF32 = 0, kProjQkv = 1, kProjSwiglu = 2 };
struct ProjEpi {
  float* out = nullptr;  // kProjF32: [rows][N]
  Plan plan{};           // kProjQkv: row positions / slots, KV pages, norms, RoPE tables
  KvView kv{};
  const void* qn_w = nullptr;
  const void* kn_w = nullptr;
  const void* cos = nullptr;
  const void* sin = nullptr;
  void* q_out = nullptr;
  int layer = 0, Hq = 0, Hkv = 0;
  float eps = 0.f;
  void* h = nullptr;     // kProjSwiglu: [rows][I]
  int I = 0;
};

// Device-side K split actually used for a pass with `n_rows` rows.
__host__ __device__ inline int effective_split(int split, int n_rows) { return n_rows <= 64 ? split : 1; }

// How many K-split partials a projection left in the f32 buffer, by pass
// size: k_linear splits only passes of <= 64 rows (effective_split), the
// tensor-core GEMM splits every pass.
struct PartSplit {
  int small = 1;  // passes of <= 64 rows
  int large = 1;  // larger passes
  __host__ __device__ int at(int n_rows) const { return n_rows <= 64 ? small : large; }
};
inline PartSplit linear_split(int split) { return PartSplit{split, 1}; }

enum ActType { kBF16 = 0, kF16 = 1 };

// Launch with programmatic stream serialisation, so that inside a step (and
// its CUDA graph) a kernel's launch overlaps the tail of its predecessor.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---- launchers (fmd_kernels.cu) -------------------------------------------------
// also writes ssq[row][0] = sum of squares of the row, ssq[row][1..tiles) = 0, when ssq != nullptr
void launch_embed_norm(ActType at, const Plan& p, int R, const void* table, const void* arena, void* x, const void* w,
                       void* xn, int H, float eps, float* ssq, int ssq_tiles, cudaStream_t s,
                       int* zero = nullptr, int zero_n = 0);
// `decode_only`: every pass through this launch has <= 64 rows, so the K
// split is known before the plan is read and weights are prefetched early.
void launch_linear(ActType at, const LinW& W, const void* x, int ldx, const int* row_map, const int* n_rows_ptr,
                   int max_rows, float* out, size_t split_stride, bool decode_only, cudaStream_t s);
void launch_qkv_epilogue(ActType at, const Plan& p, int R, const float* part, PartSplit split, size_t split_stride,
                         int Hq, int Hkv, const void* qn_w, const void* kn_w, const void* cos, const void* sin,
                         void* q_out, const KvView& kv, int layer, float eps, cudaStream_t s);
// fmd_attn_prefill.cu: chunked-prefill flash attention on tcgen05; `q_tmap`
// views the query buffer as [rows][Hq x 128]. With persistent_ctas > 0,
// that many persistent CTAs (k_attn_prefill_pp, two query tiles per CTA),
// else one CTA per (prefill block, kv head) (k_attn_prefill_tc).
cudaError_t init_attn_prefill();
void launch_attn_prefill_tc(ActType at, const void* kv_tmap, const void* q_tmap, const Plan& p, int PB, int Hq,
                            int Hkv, const KvView& kv, int layer, float scale, void* ctx, int* status,
                            cudaStream_t s, int persistent_ctas = 0);
void launch_residual_norm(ActType at, const int* n_rows_ptr, int R, void* x, const float* part, PartSplit split,
                          size_t split_stride, const void* w, void* xn, int H, float eps, cudaStream_t s);
void launch_silu_mul(ActType at, const int* n_rows_ptr, int R, const float* part, PartSplit split, size_t split_stride,
                     int I, void* h, cudaStream_t s);
void launch_logits_argmax(ActType at, const int* n_sample_ptr, int B, const float* part, int V, float* logits,
                          int* next_ids, cudaStream_t s);
void launch_dequant(ActType at, const LinW& W, float* out, cudaStream_t s);
// fmd_chain.cu: the cluster count and shared-memory bytes of the layer tail
// for up to `max_rows` rows on `n_sm` SMs (false when it cannot run; sets the
// kernels' shared-memory limit), and its launch.
bool chain_plan(ActType at, const ChainArgs& a, int n_sm, int max_rows, int* n_clusters, size_t* smem, char* why,
                size_t why_len);
void launch_layer_tail(ActType at, const ChainArgs& a, int n_clusters, size_t smem, cudaStream_t s);
// halves[0] / halves[1]: the row counts of rows [0, split) / [split, n) of
// a decode-only pass (a step split over two streams).
void launch_half_counts(const PlanCounts* full, PlanCounts* halves, int split, cudaStream_t s);
// One bounded wait that runs out after `limit` tries and sets *status to
// FMD_ETIMEDOUT (the failure path of every ring kernel's waits).
void launch_wait_probe(uint32_t limit, int* status, cudaStream_t s);
// tcgen05.mma issue cost probe (fmd_debug_mma_issue): one CTA, `iters` MMAs
// of M 128 x N n x K 16 issued in `form` 0 (lone thread of a diverged warp)
// or 1 (converged warp, elected lane); cycles[0] = SM cycles for all of them.
cudaError_t launch_mma_issue_probe(int form, int n, int iters, long long* cycles, int* status, cudaStream_t s);
// fmd_splice.cu: prompt rows from vocabulary ids (src >= 0) or audio rows
// (src = -row - 1), H a multiple of 8, every pointer 16-byte aligned.
void launch_splice(ActType at, const int* src, long long n, const void* table, const void* audio, bool audio_f32,
                   int H, void* out, cudaStream_t s);

// fmd_gemv.cu: decode-step projections (cluster split-K, fused epilogues/norms).
cudaError_t init_gemv();
int gemv_split(int epi, int K);
int gemv_tile_features(int epi);
// Decode-packed copy of a projection for the GEMV of epilogue `epi`: q8 takes
// qs [N][K] + d [N][K/32] (f16 bits), else w [N][K] 16-bit (host side).
size_t gemv_packed_bytes(int epi, int N, int K, bool q8);
void gemv_pack(int epi, int N, int K, bool q8, const int8_t* qs, const uint16_t* d, const uint16_t* w,
               uint8_t* out);
// false (nothing launched) if the projection has no packed tiles or no valid
// K split for this epilogue.
bool launch_gemv(ActType at, int epi, bool norm, const LinW& W, const void* x, int ldx, const int* row_map,
                 const int* n_rows_ptr, int max_rows, const GemvEpi& ep, int* status, cudaStream_t s);
// lm_head of the decode step: Q8_0 weights and up to 64 rows on the tensor
// cores (k_lm_head_tc, when `tc`), else the persistent mma.sync kernel (f16
// operands for Q8_0 with bf16 rows when `f16ops`), else the cluster GEMV when
// the activation tile does not fit. Returns the candidates per row it writes
// into ep.best_val / best_idx (0: nothing launched).
int launch_lm_head(ActType at, const LinW& W, const void* x, int ldx, const int* row_map, const int* n_rows_ptr,
                   int max_rows, const GemvEpi& ep, int* status, cudaStream_t s, bool tc = true,
                   bool f16ops = true, bool* used_tc = nullptr);
// fmd_lm_head_tc.cu: the tensor-core lm_head (0 when it cannot serve the shapes).
int launch_lm_head_tc(ActType at, const LinW& W, const void* x, int ldx, const int* row_map, const int* n_rows_ptr,
                      int max_rows, const GemvEpi& ep, int* status, cudaStream_t s);
// next_ids[r] = the lowest-index maximum of row r; a row without a finite
// candidate gets 0 and sets *status to FMD_EIO
void launch_pick_reduce(const int* n_sample_ptr, int B, const float* best_val, const int* best_idx, int n_parts,
                        int* next_ids, int vocab, int* status, cudaStream_t s);

// fmd_attn_decode.cu: TMA-fed decode attention with the split-KV merge fused in.
// `tmap` points at a CUtensorMap over the KV pool viewed as 2D
// [layers*pages*2*kv_heads*64 rows][128 dims], box 64x64, 128B swizzle.
size_t attn_decode_smem_bytes();
// floats of the split-segment partials of a decode-attention grid of `grid`
// CTAs (two slots per CTA, both query heads of a kv head, acc + m + l)
size_t attn_decode_partial_floats(int grid);
cudaError_t init_attn_decode();
void launch_attn_decode_tma(ActType at, const void* tmap, const Plan& p, int grid, int Hq, int Hkv, const void* q,
                            const KvView& kv, int layer, float scale, float* part_acc, float* part_ml, int* counters,
                            void* ctx, int* status, cudaStream_t s);

// ---- tensor-core projections of mixed steps (fmd_gemm_tc.cu) ----
// W [N][K] 16-bit behind a TMA map with box {64, bn} and the 128-byte
// swizzle; the output goes to out[split][rows][N] (f32).
struct TcLinear {
  alignas(64) CUtensorMap wmap;  // 16-bit [N][K] weights, or (q8) the int8 [N][K] Q8_0 quants
  int N = 0, K = 0, bn = 0, split = 1;
  bool ok = false;
  bool q8 = false;
  const uint16_t* d = nullptr;   // q8: f16 scales [N][K / 32]
};
cudaError_t init_gemm_tc();
// Tile width and K split for an N x K projection (false: not supported).
bool tc_plan(int N, int K, int* bn, int* split);
// 2D map over a row-major int8 [outer][inner] matrix, box {64, box_outer}, no swizzle.
bool tc_make_map_i8(void* encode_fn, CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
                    uint32_t box_outer);
// 2D map over a row-major [outer][inner] 16-bit matrix, box {64, box_outer}.
bool tc_make_map(void* encode_fn, CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
                 uint32_t box_outer);
// false (nothing launched) if W has no tensor-core plan.
bool launch_gemm_tc(ActType at, const CUtensorMap& amap, const TcLinear& W, const int* n_rows_ptr, int max_rows,
                    float* out, size_t split_stride, int* status, cudaStream_t s);
cudaError_t init_proj_tc();
// false (nothing launched) if the projection's tensor-core plan does not fit
// the epilogue (qkv / gate-up: 256-feature tiles, f32 rows: 128).
bool launch_proj_tc(ActType at, int epi, const CUtensorMap& amap, const TcLinear& W, const int* n_rows_ptr,
                    int max_rows, const ProjEpi& ep, int n_sm, int* status, cudaStream_t s);


}  // namespace fmd
