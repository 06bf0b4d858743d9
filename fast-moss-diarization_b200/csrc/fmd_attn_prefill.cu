// Chunked-prefill flash attention over the paged KV cache on the
// 5th-generation tensor cores.
//
// Computes `Attention::forward` of crates/fmd-core/src/model/qwen3.rs:229-257
// for the prompt rows of a step (`Qwen3::prefill`, qwen3.rs:475-496): causal
// scores of each query row against every cached key up to its own position,
// softmax, weighted sum of the values, for the two query heads that share a kv
// head (GQA 16/8, qwen3.rs:237-241).
//
// One CTA per (prefill block of <= 64 consecutive rows of one sequence, kv
// head h). The block's rows of query heads 2h and 2h+1 are stacked into one
// 128-row MMA tile (rows 0-63 head 2h, 64-127 head 2h+1), so every K/V page
// tile is read once for both heads. CTAs take the blocks longest history
// first (rank by kv length), so the longest blocks do not start last:
//  * warp 0 (one lane): TMA loads of the query tile (four 64x64 boxes,
//    128-byte swizzle) and of each key page's K and V tiles (2 x 16 KB) into a
//    3-stage full/empty mbarrier ring;
//  * warp 1 (the whole warp, one elected lane issuing): tcgen05.mma, f32 accumulators in tensor memory:
//    S_j = Q K_j^T (M 128, N 64 keys, K 128 dims; S double-buffered), then
//    O += P_j V_j (M 128, N 128 dims, K 64 keys; V read MN-major straight from
//    the page tile; O stays in tensor memory for the whole block);
//  * warps 2-5 (one thread per tile row = tensor-memory lane): the online
//    softmax in the exp2 domain with a lazily updated reference maximum: P_j =
//    exp2(S_j - m_ref) goes as 16-bit values into a double-buffered
//    128-byte-swizzled shared tile (the A operand of the PV MMA); m_ref only
//    moves when a row maximum exceeds it by more than 2^8, and only then is
//    the row of O in tensor memory rescaled (load, scale, store). At the end
//    each thread divides its row of O by the row sum and stores ctx.
// Every wait is bounded; a timeout sets the status word, stops issuing work,
// waits (bounded) for copies and MMAs in flight and frees tensor memory.
#include <cuda.h>
#include <float.h>
#include <math.h>

#include <algorithm>

#include "fmd_kernels.cuh"

namespace fmd {

namespace {

constexpr int kPfStages = 3;
constexpr int kPfQBytes = 32768;   // 128 rows x 128 dims x 2 bytes
constexpr int kPfKvBytes = 32768;  // K (16 KB) + V (16 KB) of one 64-position page
constexpr int kPfPBytes = 16384;   // one P buffer: 128 rows x 64 keys x 2 bytes (two buffers)
constexpr int kPfBox = 8192;       // one 64 x 64 TMA box
constexpr uint32_t kPfWaitLimit = 1u << 24;
constexpr int kPfTmemCols = 256;   // S0 [0, 64), S1 [64, 128), O [128, 256)
constexpr float kPfRescale = 8.f;  // log2 headroom before the reference maximum moves

// Shared-memory descriptor of an MN-major operand with the 128-byte swizzle:
// 64 contiguous elements of the MN dimension per 128-byte row, one row per K
// index, 8-row atoms 1024 bytes apart along K (stride byte offset), 64-element
// MN blocks `mn_block_bytes` apart (leading byte offset).
FMD_DEV uint64_t umma_desc_sw128_mn(uint32_t saddr, uint32_t mn_block_bytes) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((mn_block_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

FMD_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// Softmax arithmetic of one tile row (64 raw scores), shared by both prefill
// kernels so that they compute the same values. Keys past the row's position
// become -inf (only a tile that reaches it is checked); the maximum is taken
// over the raw scores (the scale is positive, and rounding is monotonic, so
// max(s) * scale = max(s * scale)) in 8 independent chains.
FMD_DEV float pf_row_max(float (&s)[64], int key0, int qpos, float scale_log2) {
  if (key0 + 63 > qpos) {
#pragma unroll
    for (int c = 0; c < 64; ++c) s[c] = key0 + c <= qpos ? s[c] : -INFINITY;
  }
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = s[i];
#pragma unroll
  for (int c = 8; c < 64; ++c) m[c & 7] = fmaxf(m[c & 7], s[c]);
#pragma unroll
  for (int i = 1; i < 8; ++i) m[0] = fmaxf(m[0], m[i]);
  return m[0] * scale_log2;
}
// p = 2^(s * scale - m_ref) in place (one rounding of the argument); returns
// the row sum of the tile, added in 8 independent chains.
// 2^x by the hardware approximation (PTX ex2.approx.ftz.f32: relative error
// about 2^-22, results below 2^-126 flushed to zero). The probabilities are
// rounded to the 16-bit operand type right after, so its error is far below
// what reaches the PV product.
FMD_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Two f32 lanes at once (PTX fma.rn.f32x2 / add.rn.f32x2, sm_100): each lane
// rounds exactly as the scalar instruction, so the results are those of two
// scalar FMAs or adds, in half the instructions.
FMD_DEV float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)),
        "l"(*reinterpret_cast<unsigned long long*>(&c)));
  return *reinterpret_cast<float2*>(&d);
}
FMD_DEV float2 fadd2(float2 a, float2 b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)));
  return *reinterpret_cast<float2*>(&d);
}
// p = 2^(s * scale - m_ref) in place, and the row sum: eight partial sums
// (key c into sum c % 8, two per packed lane pair), added in a fixed tree.
FMD_DEV float pf_row_exp(float (&s)[64], float scale_log2, float m_ref) {
  float2 a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = make_float2(0.f, 0.f);
  const float2 sc = make_float2(scale_log2, scale_log2), nm = make_float2(-m_ref, -m_ref);
#pragma unroll
  for (int c = 0; c < 64; c += 2) {
    float2 v = ffma2(make_float2(s[c], s[c + 1]), sc, nm);
    v.x = ex2_approx(v.x);
    v.y = ex2_approx(v.y);
    s[c] = v.x;
    s[c + 1] = v.y;
    a[(c >> 1) & 3] = fadd2(a[(c >> 1) & 3], v);
  }
  return ((a[0].x + a[0].y) + (a[1].x + a[1].y)) + ((a[2].x + a[2].y) + (a[3].x + a[3].y));
}

template <typename T>
__global__ void __launch_bounds__(192, 1)
    k_attn_prefill_tc(const __grid_constant__ CUtensorMap kvmap, const __grid_constant__ CUtensorMap qmap, Plan p,
                      int Hq, int Hkv, KvView kv, int layer, float scale_log2, T* __restrict__ ctx,
                      int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, kv_full[kPfStages], kv_empty[kPfStages], s_full[2], s_empty[2],
      p_full[2], p_empty[2], o_full, o_final, mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s, block_s;
  __shared__ int klen_s[kMaxPrefillBlocks];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzle atoms need 1024-byte alignment
  uint8_t* base_p = smem_raw + (base - raw);
  const uint32_t q_s = base, p_s = base + kPfQBytes, kv_s = p_s + 2 * kPfPBytes;
  uint8_t* p_sp = base_p + kPfQBytes;

  griddep_wait();  // q, the KV rows of this step and the plan come from earlier kernels
  griddep_launch();  // only after the wait: see griddep_launch
  const int n_blocks = min(p.counts->n_pblocks, kMaxPrefillBlocks);
  if ((int)blockIdx.x >= n_blocks) return;  // whole CTA, before any barrier or tensor memory exists
  // CTA x takes the block of rank x by kv length (longest first, ties by index)
  for (int i = threadIdx.x; i < n_blocks; i += blockDim.x) klen_s[i] = p.row_pos[p.pb_row0[i]] + p.pb_n[i];
  __syncthreads();
  for (int i = threadIdx.x; i < n_blocks; i += blockDim.x) {
    const int ki = klen_s[i];
    int rank = 0;
    for (int k = 0; k < n_blocks; ++k) {
      const int kk = klen_s[k];
      rank += (kk > ki) || (kk == ki && k < i);
    }
    if (rank == (int)blockIdx.x) block_s = i;
  }
  __syncthreads();
  const int b = block_s, h = blockIdx.y;
  const int r0 = p.pb_row0[b], n = p.pb_n[b];
  const int slot = p.row_slot[r0], pos0 = p.row_pos[r0];
  const int kv_len = pos0 + n;
  const int T_tiles = (kv_len + kPageTokens - 1) / kPageTokens;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 128);
      mbar_init(&p_full[s], 128);
      mbar_init(&p_empty[s], 1);
    }
    mbar_init(&o_full, 1);
    mbar_init(&o_final, 1);
    mbar_init(&mma_done, 1);
    abort_s = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, kPfTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  volatile int* abort_v = &abort_s;

  // Parity waits never alias: each waits for a phase whose successor needs
  // work that the waiting role itself releases later, and whose predecessor
  // has completed (MMAs of one thread complete in issue order, and s_full(j)
  // fires only after PV_{j-2}); the final O has a barrier of its own.
  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tmap(&kvmap);
      prefetch_tmap(&qmap);
      mbar_arrive_expect_tx(&q_full, kPfQBytes);
      const int xq0 = 2 * h * kHeadDim, xq1 = (2 * h + 1) * kHeadDim;
      tma_load_2d(base_p + 0 * kPfBox, &qmap, xq0, r0, &q_full);        // rows 0-63: head 2h, dims 0-63
      tma_load_2d(base_p + 1 * kPfBox, &qmap, xq1, r0, &q_full);        // rows 64-127: head 2h+1, dims 0-63
      tma_load_2d(base_p + 2 * kPfBox, &qmap, xq0 + 64, r0, &q_full);   // dims 64-127
      tma_load_2d(base_p + 3 * kPfBox, &qmap, xq1 + 64, r0, &q_full);
      const int* ptab = kv.page_table + (size_t)slot * kv.max_pages_per_slot;
      int issued = 0;
      for (int j = 0; j < T_tiles; ++j) {
        const int st = j % kPfStages;
        if (j >= kPfStages &&
            (*abort_v || !mbar_wait_bounded(&kv_empty[st], ((j / kPfStages) - 1) & 1, kPfWaitLimit))) {
          *abort_v = 1;
          break;
        }
        const int page = ptab[j];
        const int yk = (int)(((((size_t)layer * kv.n_pages + page) * 2 + 0) * Hkv + h) * kPageTokens);
        const int yv = yk + Hkv * kPageTokens;
        uint8_t* dst = base_p + kPfQBytes + 2 * kPfPBytes + st * kPfKvBytes;
        mbar_arrive_expect_tx(&kv_full[st], kPfKvBytes);
        tma_load_2d(dst, &kvmap, 0, yk, &kv_full[st]);
        tma_load_2d(dst + kPfBox, &kvmap, 64, yk, &kv_full[st]);
        tma_load_2d(dst + 2 * kPfBox, &kvmap, 0, yv, &kv_full[st]);
        tma_load_2d(dst + 3 * kPfBox, &kvmap, 64, yv, &kv_full[st]);
        issued = j + 1;
      }
      // copies still in flight must land before the CTA can retire (bounded)
      mbar_wait_bounded(&q_full, 0, kPfWaitLimit);
      for (int j = issued > kPfStages ? issued - kPfStages : 0; j < issued; ++j)
        mbar_wait_bounded(&kv_full[j % kPfStages], (j / kPfStages) & 1, kPfWaitLimit);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the whole warp runs the loop, the elected lane issues ----------------
    {
      constexpr bool kBf = Act<T>::kIsBf16;
      constexpr uint32_t idesc_s = umma_idesc_f16(kBf, 128, 64);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBf, 128, 128) | (1u << 16);  // B (V) MN-major
      const uint32_t o_tmem = tmem + 128;
      auto pv = [&](int i) -> bool {
        const int pb = i & 1;
        if (*abort_v || !mbar_wait_warp(&p_full[pb], (i >> 1) & 1, kPfWaitLimit)) return false;
        tc_fence_after();
        const uint32_t v = kv_s + (i % kPfStages) * kPfKvBytes + 2 * kPfBox;
        const uint32_t pa = p_s + pb * kPfPBytes;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(o_tmem, umma_desc_sw128(pa + kk * 32), umma_desc_sw128_mn(v + kk * 2048, kPfBox), idesc_o,
                     (i | kk) != 0);
          umma_commit(&o_full);
          umma_commit(&p_empty[pb]);
          umma_commit(&kv_empty[i % kPfStages]);
        }
        __syncwarp();
        return true;
      };
      bool ok = !*abort_v && mbar_wait_warp(&q_full, 0, kPfWaitLimit);
      for (int j = 0; ok && j < T_tiles; ++j) {
        const int st = j % kPfStages, sb = j & 1;
        if (*abort_v || !mbar_wait_warp(&kv_full[st], (j / kPfStages) & 1, kPfWaitLimit) ||
            (j >= 2 && !mbar_wait_warp(&s_empty[sb], ((j >> 1) - 1) & 1, kPfWaitLimit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k = kv_s + st * kPfKvBytes;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t a = q_s + (kk < 4 ? kk * 32 : 2 * kPfBox + (kk - 4) * 32);
            const uint32_t bk = k + (kk < 4 ? kk * 32 : kPfBox + (kk - 4) * 32);
            umma_f16(tmem + sb * 64, umma_desc_sw128(a), umma_desc_sw128(bk), idesc_s, kk != 0);
          }
          umma_commit(&s_full[sb]);
        }
        __syncwarp();
        if (j >= 1 && !pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) ok = pv(T_tiles - 1);
      if (ok && elect_one()) umma_commit(&o_final);  // a phase of its own: the last o_full phase could alias
      __syncwarp();
      if (!ok) *abort_v = 1;
      if (elect_one()) umma_commit(&mma_done);  // every MMA issued so far has completed when this fires
      __syncwarp();
      mbar_wait_warp(&mma_done, 0, kPfWaitLimit);
    }
  } else {
    // ---------------- softmax + output: one thread per tile row ----------------
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const int hs = row >> 6, ri = row & 63;
    const int qpos = pos0 + ri;
    const uint32_t lane_addr = tmem + ((uint32_t)(q4 * 32) << 16);
    const uint32_t o_addr = lane_addr + 128;
    float m_ref = -INFINITY, l = 0.f;
    // tcgen05.ld / st are warp-wide (.sync.aligned): every branch around them
    // is taken by the whole warp. A wait counts as passed only when it passed
    // for all 32 lanes, so no lane goes on to a tensor-memory access alone.
    auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
      const bool mine = !*abort_v && mbar_wait_bounded(bar, parity, kPfWaitLimit);
      return __all_sync(0xffffffffu, mine);
    };
    bool ok = true;
    for (int j = 0; j < T_tiles && ok; ++j) {
      const int sb = j & 1;
      if (!wwait(&s_full[sb], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(lane_addr + sb * 64 + c * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i2 = 0; i2 < 32; ++i2) s[c * 32 + i2] = __uint_as_float(v[i2]);
      }
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      const float mx = pf_row_max(s, j * kPageTokens, qpos, scale_log2);
      // a row moves its reference maximum when its new maximum exceeds it by
      // more than 2^8; its O (all PVs so far) and l then scale by
      // 2^(m_ref - mx). The rescale reads and writes O in tensor memory, a
      // warp-wide operation: the warp does it when any of its rows moves,
      // and the rows that do not move scale by 1 (their O is unchanged).
      bool moves = false;
      if (j == 0)
        m_ref = mx;  // finite: key 0 <= qpos
      else
        moves = mx > m_ref + kPfRescale;
      if (__any_sync(0xffffffffu, moves)) {
        if (!wwait(&o_full, (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float f = moves ? exp2f(m_ref - mx) : 1.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(o_addr + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i2 = 0; i2 < 32; ++i2) v[i2] = __float_as_uint(__uint_as_float(v[i2]) * f);
          tmem_st32(o_addr + c * 32, v);
        }
        tmem_st_wait();
        if (moves) {
          l *= f;
          m_ref = mx;
        }
      }
      l += pf_row_exp(s, scale_log2, m_ref);
      // P buffer j&1 was last read by PV_{j-2}
      if (j >= 2 && !wwait(&p_empty[sb], ((j - 2) >> 1) & 1)) {
        ok = false;
        break;
      }
      // P_j -> the 128-byte-swizzled A tile: row `row`, 16-byte chunk c holds keys 8c .. 8c+7
      uint8_t* prow = p_sp + sb * kPfPBytes + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 u;
        u.x = Act<T>::pack2(s[8 * c + 0], s[8 * c + 1]);
        u.y = Act<T>::pack2(s[8 * c + 2], s[8 * c + 3]);
        u.z = Act<T>::pack2(s[8 * c + 4], s[8 * c + 5]);
        u.w = Act<T>::pack2(s[8 * c + 6], s[8 * c + 7]);
        *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    if (ok && !wwait(&o_final, 0)) ok = false;
    if (!ok) *abort_v = 1;
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l;
      T* dst = ctx + (size_t)(r0 + ri) * Hq * kHeadDim + (2 * h + hs) * kHeadDim;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(o_addr + c * 32, v);
        tmem_ld_wait();
        if (ri < n) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint4 u;
            u.x = Act<T>::pack2(__uint_as_float(v[8 * q8 + 0]) * inv, __uint_as_float(v[8 * q8 + 1]) * inv);
            u.y = Act<T>::pack2(__uint_as_float(v[8 * q8 + 2]) * inv, __uint_as_float(v[8 * q8 + 3]) * inv);
            u.z = Act<T>::pack2(__uint_as_float(v[8 * q8 + 4]) * inv, __uint_as_float(v[8 * q8 + 5]) * inv);
            u.w = Act<T>::pack2(__uint_as_float(v[8 * q8 + 6]) * inv, __uint_as_float(v[8 * q8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + 8 * q8) = u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && abort_s) report_timeout(status, kSiteAttnPrefill);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPfTmemCols);
  }
}

// ---- persistent, two query tiles per CTA ------------------------------------
// The same arithmetic as k_attn_prefill_tc, scheduled for the tensor cores:
//  * a work item is a pair of 64-row blocks of one sequence (A earlier, B
//    later) for one kv head: both tiles read the same key pages up to A's
//    history, so each such K/V page tile is read once for both. A sequence's
//    run of n blocks pairs block i with block n - 1 - i, which evens out the
//    items' key-tile counts; the middle block of an odd run is an item alone;
//  * items are ranked by key tiles (longest first), work w = (item w / Hkv,
//    head w % Hkv); CTA c of G takes works c, 2G - 1 - c, 2G + c, ... (snake
//    order), so the long items are spread over the CTAs and the short ones
//    even out their totals;
//  * warp 0: TMA of both query tiles and of the page tiles (3-stage ring);
//    warp 1: tcgen05.mma for both tiles, S_A(j), S_B(j), then PV_A(j - 1),
//    PV_B(j - 1): while one softmax group works on its scores the tensor core
//    runs the other tile's MMAs;
//  * warps 2-5 / 6-9: the online softmax of tile A / B, one thread per tile
//    row, as in k_attn_prefill_tc; P goes through one shared buffer per tile
//    (the PV that read the previous P has completed before it is rewritten);
//    O of each tile stays in tensor memory for the whole item (512 columns:
//    per tile two S buffers and O).
// Ring positions, S buffers, P and PV counts continue across a CTA's items;
// each barrier is waited on in use order by one role, which has already
// seen the previous use of the same slot complete, so no parity wait aliases.
constexpr int kPpThreads = 320;
constexpr int kPpTmemCols = 512;

size_t attn_pp_smem_bytes() {
  return 1024 + 2 * kPfQBytes + 2 * kPfPBytes + kPfStages * kPfKvBytes + (size_t)4 * kMaxPrefillBlocks * 4;
}

template <typename T>
__global__ void __launch_bounds__(kPpThreads, 1)
    k_attn_prefill_pp(const __grid_constant__ CUtensorMap kvmap, const __grid_constant__ CUtensorMap qmap, Plan p,
                      int Hq, int Hkv, KvView kv, int layer, float scale_log2, T* __restrict__ ctx,
                      int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, q_empty, kv_full[kPfStages], kv_empty[kPfStages], s_full[2][2],
      s_empty[2][2], p_full[2], pv_done[2], o_final[2], o_empty[2], mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s, n_items_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzle atoms need 1024-byte alignment
  uint8_t* base_p = smem_raw + (base - raw);
  // Q_A | Q_B | P_A | P_B | K/V stages | block slots | item costs | item order
  const uint32_t q_s = base, p_s = base + 2 * kPfQBytes, kv_s = p_s + 2 * kPfPBytes;
  uint8_t* p_sp = base_p + 2 * kPfQBytes;
  int* s_slot = reinterpret_cast<int*>(base_p + 2 * kPfQBytes + 2 * kPfPBytes + kPfStages * kPfKvBytes);
  int* s_cost = s_slot + kMaxPrefillBlocks;
  int* s_order = s_cost + kMaxPrefillBlocks;
  int* s_partner = s_order + kMaxPrefillBlocks;  // tile B of the item a block starts (-1: none)

  griddep_wait();  // q, the KV rows of this step and the plan come from earlier kernels
  griddep_launch();  // only after the wait: see griddep_launch
  const int n_blocks = min(p.counts->n_pblocks, kMaxPrefillBlocks);
  if (n_blocks == 0) return;  // whole CTA, before any barrier or tensor memory exists
  auto tiles_of = [&](int b) { return (p.row_pos[p.pb_row0[b]] + p.pb_n[b] + kPageTokens - 1) / kPageTokens; };
  // ---- items: the run of n blocks of one sequence pairs its block i with
  // block n - 1 - i (the shortest history with the longest, so that every
  // item needs about the same number of key tiles); the middle block of an
  // odd run is an item of its own
  if (threadIdx.x == 0) n_items_s = 0;
  for (int b = threadIdx.x; b < n_blocks; b += kPpThreads) s_slot[b] = p.row_slot[p.pb_row0[b]];
  __syncthreads();
  for (int b = threadIdx.x; b < n_blocks; b += kPpThreads) {
    int j = 0, after = 0;
    while (b - j - 1 >= 0 && s_slot[b - j - 1] == s_slot[b]) ++j;
    while (b + after + 1 < n_blocks && s_slot[b + after + 1] == s_slot[b]) ++after;
    const int n = j + 1 + after;  // the run's length; b is its block j
    int cost = 0, partner = -1;
    if (2 * j + 1 <= n) {
      partner = 2 * j + 1 < n ? b + (n - 1 - 2 * j) : -1;  // block n - 1 - j of the run
      cost = tiles_of(b) + (partner >= 0 ? tiles_of(partner) : 0);
      atomicAdd(&n_items_s, 1);
    }
    s_cost[b] = cost;  // 0: not an item start (every item has >= 1 tile)
    s_partner[b] = partner;
  }
  __syncthreads();
  for (int b = threadIdx.x; b < n_blocks; b += kPpThreads) {
    const int cb = s_cost[b];
    if (cb == 0) continue;
    int rank = 0;
    for (int k = 0; k < n_blocks; ++k) {
      const int ck = s_cost[k];
      rank += (ck > cb) || (ck == cb && k < b);
    }
    s_order[rank] = b;
  }
  __syncthreads();
  const int G = gridDim.x, c = blockIdx.x;
  const int n_works = n_items_s * Hkv;
  if (c >= n_works) return;  // whole CTA, before any barrier or tensor memory exists
  auto work_at = [&](int r) -> int { return r * G + ((r & 1) ? G - 1 - c : c); };

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      for (int s = 0; s < 2; ++s) {
        mbar_init(&s_full[x][s], 1);
        mbar_init(&s_empty[x][s], 128);
      }
      mbar_init(&p_full[x], 128);
      mbar_init(&pv_done[x], 1);
      mbar_init(&o_final[x], 1);
      mbar_init(&o_empty[x], 128);
    }
    mbar_init(&mma_done, 1);
    abort_s = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, kPpTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  volatile int* abort_v = &abort_s;

  // the work of round r: tiles A, B (B = -1 for a lone block) and kv head h
  struct Work {
    int a, b, h;
  };
  auto work = [&](int r, Work& w) -> bool {
    const int wi = work_at(r);
    if (wi >= n_works) return false;
    w.a = s_order[wi / Hkv];
    w.h = wi % Hkv;
    w.b = s_partner[w.a];
    return true;
  };

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tmap(&kvmap);
      prefetch_tmap(&qmap);
      int g = 0, k = 0;  // page tiles and query loads issued
      bool ok = true;
      Work w;
      for (int r = 0; ok && work(r, w); ++r) {
        if (k >= 1 && (*abort_v || !mbar_wait_bounded(&q_empty, (k - 1) & 1, kPfWaitLimit))) {
          ok = false;
          break;
        }
        const int nq = w.b >= 0 ? 2 : 1;
        mbar_arrive_expect_tx(&q_full, nq * kPfQBytes);
        ++k;
        for (int x = 0; x < nq; ++x) {
          const int r0 = p.pb_row0[x ? w.b : w.a];
          const int xq0 = 2 * w.h * kHeadDim, xq1 = (2 * w.h + 1) * kHeadDim;
          uint8_t* qd = base_p + x * kPfQBytes;
          tma_load_2d(qd + 0 * kPfBox, &qmap, xq0, r0, &q_full);       // rows 0-63: head 2h, dims 0-63
          tma_load_2d(qd + 1 * kPfBox, &qmap, xq1, r0, &q_full);       // rows 64-127: head 2h+1, dims 0-63
          tma_load_2d(qd + 2 * kPfBox, &qmap, xq0 + 64, r0, &q_full);  // dims 64-127
          tma_load_2d(qd + 3 * kPfBox, &qmap, xq1 + 64, r0, &q_full);
        }
        const int slot = s_slot[w.a];
        const int* ptab = kv.page_table + (size_t)slot * kv.max_pages_per_slot;
        const int T = tiles_of(w.b >= 0 ? w.b : w.a);
        for (int j = 0; j < T; ++j, ++g) {
          const int st = g % kPfStages;
          if (g >= kPfStages &&
              (*abort_v || !mbar_wait_bounded(&kv_empty[st], ((g / kPfStages) + 1) & 1, kPfWaitLimit))) {
            ok = false;
            break;
          }
          const int page = ptab[j];
          const int yk = (int)(((((size_t)layer * kv.n_pages + page) * 2 + 0) * Hkv + w.h) * kPageTokens);
          const int yv = yk + Hkv * kPageTokens;
          uint8_t* dst = base_p + 2 * kPfQBytes + 2 * kPfPBytes + st * kPfKvBytes;
          mbar_arrive_expect_tx(&kv_full[st], kPfKvBytes);
          tma_load_2d(dst, &kvmap, 0, yk, &kv_full[st]);
          tma_load_2d(dst + kPfBox, &kvmap, 64, yk, &kv_full[st]);
          tma_load_2d(dst + 2 * kPfBox, &kvmap, 0, yv, &kv_full[st]);
          tma_load_2d(dst + 3 * kPfBox, &kvmap, 64, yv, &kv_full[st]);
        }
      }
      if (!ok) *abort_v = 1;
      // copies still in flight must land before the CTA can retire (bounded)
      if (k >= 1) mbar_wait_bounded(&q_full, (k - 1) & 1, kPfWaitLimit);
      for (int j = g > kPfStages ? g - kPfStages : 0; j < g; ++j)
        mbar_wait_bounded(&kv_full[j % kPfStages], (j / kPfStages) & 1, kPfWaitLimit);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the whole warp runs the loop, the elected lane issues ----------------
    {
      constexpr bool kBf = Act<T>::kIsBf16;
      constexpr uint32_t idesc_s = umma_idesc_f16(kBf, 128, 64);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBf, 128, 128) | (1u << 16);  // B (V) MN-major
      int g = 0, k = 0;
      int sn[2] = {0, 0}, pn[2] = {0, 0}, wn[2] = {0, 0};  // S tiles, PVs, items per tile role
      bool ok = true;
      // O_x += P_x V for key tile i of the item (first of the item: O_x = P_x V)
      auto pv = [&](int x, int i, int st) -> bool {
        if (i == 0 && wn[x] >= 1 &&
            (*abort_v || !mbar_wait_warp(&o_empty[x], (wn[x] - 1) & 1, kPfWaitLimit)))
          return false;
        if (*abort_v || !mbar_wait_warp(&p_full[x], pn[x] & 1, kPfWaitLimit)) return false;
        tc_fence_after();
        const uint32_t v = kv_s + st * kPfKvBytes + 2 * kPfBox;
        const uint32_t pa = p_s + x * kPfPBytes;
        const uint32_t o_tmem = tmem + x * 256 + 128;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(o_tmem, umma_desc_sw128(pa + kk * 32), umma_desc_sw128_mn(v + kk * 2048, kPfBox), idesc_o,
                     (i | kk) != 0);
          umma_commit(&pv_done[x]);  // P_x is free and O_x holds this PV when it fires
        }
        __syncwarp();
        ++pn[x];
        return true;
      };
      Work w;
      for (int r = 0; ok && work(r, w); ++r, ++k) {
        const int Tx[2] = {tiles_of(w.a), w.b >= 0 ? tiles_of(w.b) : 0};
        const int T = w.b >= 0 ? Tx[1] : Tx[0];
        if (*abort_v || !mbar_wait_warp(&q_full, k & 1, kPfWaitLimit)) {
          ok = false;
          break;
        }
        const int g0 = g;
        for (int j = 0; ok && j <= T; ++j) {
          if (j < T) {
            const int st = (g0 + j) % kPfStages;
            if (*abort_v || !mbar_wait_warp(&kv_full[st], ((g0 + j) / kPfStages) & 1, kPfWaitLimit)) {
              ok = false;
              break;
            }
            const uint32_t kt = kv_s + st * kPfKvBytes;
            for (int x = 0; x < 2; ++x) {
              if (j >= Tx[x]) continue;
              const int n = sn[x], sb = n & 1;
              if (n >= 2 && (*abort_v || !mbar_wait_warp(&s_empty[x][sb], ((n >> 1) + 1) & 1, kPfWaitLimit))) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t qa = q_s + x * kPfQBytes;
              if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                  const uint32_t a = qa + (kk < 4 ? kk * 32 : 2 * kPfBox + (kk - 4) * 32);
                  const uint32_t bk = kt + (kk < 4 ? kk * 32 : kPfBox + (kk - 4) * 32);
                  umma_f16(tmem + x * 256 + sb * 64, umma_desc_sw128(a), umma_desc_sw128(bk), idesc_s, kk != 0);
                }
                umma_commit(&s_full[x][sb]);
              }
              __syncwarp();
              ++sn[x];
            }
            if (!ok) break;
            if (j == T - 1 && elect_one()) umma_commit(&q_empty);  // the item's last score MMAs have read Q
            __syncwarp();
          }
          if (j >= 1) {
            const int i = j - 1, st = (g0 + i) % kPfStages;
            for (int x = 0; x < 2 && ok; ++x)
              if (i < Tx[x]) ok = pv(x, i, st);
            if (!ok) break;
            if (elect_one()) umma_commit(&kv_empty[st]);  // the page tile is free once its MMAs have read it
            __syncwarp();
          }
        }
        if (!ok) break;
        g = g0 + T;
        for (int x = 0; x < 2; ++x)
          if (Tx[x] > 0) {
            if (elect_one()) umma_commit(&o_final[x]);  // the item's O_x is complete when this fires
            __syncwarp();
            ++wn[x];
          }
      }
      if (!ok) *abort_v = 1;
      if (elect_one()) umma_commit(&mma_done);  // every MMA issued so far has completed when this fires
      __syncwarp();
      mbar_wait_warp(&mma_done, 0, kPfWaitLimit);
    }
  } else {
    // ---------------- softmax + output of tile x: one thread per tile row ----------------
    const int x = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const int hs = row >> 6, ri = row & 63;
    const uint32_t lane_addr = tmem + ((uint32_t)(q4 * 32) << 16) + x * 256;
    const uint32_t o_addr = lane_addr + 128;
    // tcgen05.ld / st are warp-wide (.sync.aligned): every branch around them
    // is taken by the whole warp. A wait counts as passed only when it passed
    // for all 32 lanes, so no lane goes on to a tensor-memory access alone.
    auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
      const bool mine = !*abort_v && mbar_wait_bounded(bar, parity, kPfWaitLimit);
      return __all_sync(0xffffffffu, mine);
    };
    int sn = 0, pn = 0, wn = 0;
    bool ok = true;
    Work w;
    for (int r = 0; ok && work(r, w); ++r) {
      const int blk = x ? w.b : w.a;
      if (blk < 0) continue;  // a lone block: no tile B
      const int r0 = p.pb_row0[blk], n = p.pb_n[blk];
      const int pos0 = p.row_pos[r0];
      const int qpos = pos0 + ri;
      const int Tt = tiles_of(blk);
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < Tt && ok; ++j) {
        const int sb = sn & 1;
        if (!wwait(&s_full[x][sb], (sn >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[64];
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t v[32];
          tmem_ld32(lane_addr + sb * 64 + c2 * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i2 = 0; i2 < 32; ++i2) s[c2 * 32 + i2] = __uint_as_float(v[i2]);
        }
        tc_fence_before();
        mbar_arrive(&s_empty[x][sb]);
        ++sn;
        const float mx = pf_row_max(s, j * kPageTokens, qpos, scale_log2);
        // lazy rescale (as k_attn_prefill_tc): the warp reads and writes O
        // when any of its rows moves its reference maximum; the previous PV
        // of this tile (the pn - 1-th) must have completed
        bool moves = false;
        if (j == 0)
          m_ref = mx;  // finite: key 0 <= qpos
        else
          moves = mx > m_ref + kPfRescale;
        if (__any_sync(0xffffffffu, moves)) {
          if (!wwait(&pv_done[x], (pn - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float f = moves ? exp2f(m_ref - mx) : 1.f;
#pragma unroll
          for (int c2 = 0; c2 < 4; ++c2) {
            uint32_t v[32];
            tmem_ld32(o_addr + c2 * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int i2 = 0; i2 < 32; ++i2) v[i2] = __float_as_uint(__uint_as_float(v[i2]) * f);
            tmem_st32(o_addr + c2 * 32, v);
          }
          tmem_st_wait();
          if (moves) {
            l *= f;
            m_ref = mx;
          }
        }
        l += pf_row_exp(s, scale_log2, m_ref);
        // the P buffer was last read by the previous PV of this tile role
        if (pn >= 1 && !wwait(&pv_done[x], (pn - 1) & 1)) {
          ok = false;
          break;
        }
        // P -> the 128-byte-swizzled A tile: row `row`, 16-byte chunk c holds keys 8c .. 8c+7
        uint8_t* prow = p_sp + x * kPfPBytes + row * 128;
#pragma unroll
        for (int c2 = 0; c2 < 8; ++c2) {
          uint4 u;
          u.x = Act<T>::pack2(s[8 * c2 + 0], s[8 * c2 + 1]);
          u.y = Act<T>::pack2(s[8 * c2 + 2], s[8 * c2 + 3]);
          u.z = Act<T>::pack2(s[8 * c2 + 4], s[8 * c2 + 5]);
          u.w = Act<T>::pack2(s[8 * c2 + 6], s[8 * c2 + 7]);
          *reinterpret_cast<uint4*>(prow + ((c2 ^ (row & 7)) << 4)) = u;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&p_full[x]);
        ++pn;
      }
      if (!ok) break;
      if (!wwait(&o_final[x], wn & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = 1.f / l;
      T* dst = ctx + (size_t)(r0 + ri) * Hq * kHeadDim + (2 * w.h + hs) * kHeadDim;
#pragma unroll
      for (int c2 = 0; c2 < 4; ++c2) {
        uint32_t v[32];
        tmem_ld32(o_addr + c2 * 32, v);
        tmem_ld_wait();
        if (ri < n) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint4 u;
            u.x = Act<T>::pack2(__uint_as_float(v[8 * q8 + 0]) * inv, __uint_as_float(v[8 * q8 + 1]) * inv);
            u.y = Act<T>::pack2(__uint_as_float(v[8 * q8 + 2]) * inv, __uint_as_float(v[8 * q8 + 3]) * inv);
            u.z = Act<T>::pack2(__uint_as_float(v[8 * q8 + 4]) * inv, __uint_as_float(v[8 * q8 + 5]) * inv);
            u.w = Act<T>::pack2(__uint_as_float(v[8 * q8 + 6]) * inv, __uint_as_float(v[8 * q8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c2 * 32 + 8 * q8) = u;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&o_empty[x]);  // O_x may be overwritten by the next item's first PV
      ++wn;
    }
    if (!ok) *abort_v = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && abort_s) report_timeout(status, kSiteAttnPrefill);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPpTmemCols);
  }
}

size_t attn_prefill_smem_bytes() { return 1024 + kPfQBytes + 2 * kPfPBytes + kPfStages * kPfKvBytes; }

}  // namespace

cudaError_t init_attn_prefill() {
  const int bytes = (int)attn_prefill_smem_bytes(), pp = (int)attn_pp_smem_bytes();
  for (cudaError_t e :
       {cudaFuncSetAttribute(k_attn_prefill_tc<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
        cudaFuncSetAttribute(k_attn_prefill_tc<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
        cudaFuncSetAttribute(k_attn_prefill_pp<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, pp),
        cudaFuncSetAttribute(k_attn_prefill_pp<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, pp)})
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

void launch_attn_prefill_tc(ActType at, const void* kv_tmap, const void* q_tmap, const Plan& p, int PB, int Hq,
                            int Hkv, const KvView& kv, int layer, float scale, void* ctx, int* status,
                            cudaStream_t s, int persistent_ctas) {
  const float scale_log2 = scale * 1.4426950408889634f;
  const CUtensorMap& km = *reinterpret_cast<const CUtensorMap*>(kv_tmap);
  const CUtensorMap& qm = *reinterpret_cast<const CUtensorMap*>(q_tmap);
  if (persistent_ctas > 0) {
    // at most one work per CTA is never idle: PB * Hkv bounds the works
    const int grid = std::min(persistent_ctas, PB * Hkv);
    const size_t smem = attn_pp_smem_bytes();
    if (at == kBF16)
      launch_pdl(k_attn_prefill_pp<__nv_bfloat16>, dim3(grid), dim3(kPpThreads), smem, s, km, qm, p, Hq, Hkv, kv,
                 layer, scale_log2, (__nv_bfloat16*)ctx, status);
    else
      launch_pdl(k_attn_prefill_pp<__half>, dim3(grid), dim3(kPpThreads), smem, s, km, qm, p, Hq, Hkv, kv, layer,
                 scale_log2, (__half*)ctx, status);
    return;
  }
  const size_t smem = attn_prefill_smem_bytes();
  if (at == kBF16)
    launch_pdl(k_attn_prefill_tc<__nv_bfloat16>, dim3(PB, Hkv), dim3(192), smem, s, km, qm, p, Hq, Hkv, kv, layer,
               scale_log2, (__nv_bfloat16*)ctx, status);
  else
    launch_pdl(k_attn_prefill_tc<__half>, dim3(PB, Hkv), dim3(192), smem, s, km, qm, p, Hq, Hkv, kv, layer,
               scale_log2, (__half*)ctx, status);
}

}  // namespace fmd
