// lm_head + greedy candidates of a decode step on the 5th-generation tensor
// cores (qwen3.rs:459-463, engine.rs:550-559), for Q8_0 weights and up to 64
// sampled rows.
//
// The reference dequantises each Q8_0 block (q * d, linear.rs:179-265) and
// multiplies in f32. Here the int8 values themselves go through the MMA as
// f16 (exact), every 32-wide block into its own f32 accumulator in tensor
// memory, and the block's f16 scale is applied in f32 on the way out:
// y = sum_b d_b * (sum_{k in b} q_k x_k), the reference's sum up to the f32
// summation order, as the mma.sync kernel (k_lm_head) computes it. The
// operands are f16 for both activation types (int8 -> f16 takes half the
// instructions of int8 -> bf16): bf16 rows are scaled by a power of two that
// puts their largest value in [2^14, 2^15), which leaves every value within
// 2^28 of the row's largest exact in f16 (smaller ones weigh less than the
// f32 rounding of the sum), and the logits are scaled back exactly.
//
// One CTA per SM walks 128-feature tiles (tile blockIdx.x + i * gridDim.x);
// a tile's k-blocks of 64 are stages:
//  * warp 0 (one lane): TMA bulk copies of the decode-packed stages (8 units
//    of 16 features x 64 k, 8.5 KB, the k_lm_head layout) into a ring of RAW
//    stages. Weights depend on no earlier kernel, so the ring fills before
//    the dependency wait;
//  * warps 2 .. 1 + CONVW (converters): one group of four warps, or two
//    taking alternate stages (32 rows); warp w of a group takes units w and
//    w + 4 of its stages, turns their int8 values into f16 operands and
//    writes them as 16 rows each of the stage's A tile (128 features x 64
//    k, K-major, 128-byte swizzle) in a ring of CONV slots, releasing the raw
//    stage as soon as its fragments are in registers;
//  * warp 1 (the whole warp, one elected lane issuing): tcgen05.mma M = 128
//    (features) x N = NR (rows) x K = 16, two per Q8_0 block, each block into
//    the next of 512 / NR accumulators, two stages per pass; per pass one
//    tcgen05.commit frees its A slots for the converters and one hands its
//    accumulators to the epilogue;
//  * the last 8 warps (epilogue): before the loop they stage the rows (final
//    RMSNorm applied) as the B operand, resident for the whole launch. Warp
//    w reads tensor-memory lanes 32 (w % 4) .. (the thread's feature) x NR
//    columns (the rows); the first four take the even stages of a tile, the
//    other four the odd ones, so two accumulator reads of a lane quarter are in
//    flight at once. Per stage a warp loads both blocks' accumulators behind
//    one wait, frees both with one arrival and adds d0 x block 0, then d1 x
//    block 1, in f32.
//    After a tile, the even-stage sum plus the odd-stage sum is scaled back,
//    rounded to the activation type (as the reference's lm_head output is)
//    and reduced per row to the best (value, lowest index) through shared
//    memory.
// Each CTA writes one candidate per row; k_pick_reduce finishes the pick.
// Every wait is bounded; a timeout sets the status word, each role stops,
// and the CTA waits (bounded) for its copies and MMAs in flight before it
// frees its tensor memory.
#include <cuda_runtime.h>
#include <math.h>

#include <cstdio>

#include "fmd_gemv.cuh"
#include "fmd_kernels.cuh"

namespace fmd {

namespace {

constexpr int kLhFeat = 128;                       // features of a tile = MMA M = tensor-memory lanes
constexpr int kLhUnits = kLhFeat / 16;             // 16-feature units of a stage
constexpr uint32_t kLhRaw = kLhUnits * kUnitQ8;    // packed stage: 8704 bytes
constexpr uint32_t kLhConv = kLhFeat * 128;        // converted A tile: 128 rows x 64 k x 2 bytes
constexpr int kLhEpiWarps = 8;                     // two per tensor-memory lane quarter: even / odd stages
constexpr int kLhTmemCols = 512;  // all of tensor memory: accumulator slack over a tile's end
constexpr int kLhLgStride = 132;                   // row stride (floats) of the rounded-logit tile
constexpr uint32_t kLhWaitLimit = 1u << 24;
constexpr int kScaleAhead = 8;                     // stages of block scales in flight per epilogue thread

// The weight stream needs ~100 KB in flight per SM to run at the HBM rate
// (bytes in flight = bandwidth x loaded latency), so most of the shared
// memory goes to packed stages; two converted slots keep the MMAs fed.
// Converters: groups of four warps (two units of a stage each). A stage is
// a chain of dependent steps for its group (slot and data waits, loads,
// conversion, stores, proxy fence, arrival), longer than the MMAs of a stage,
// so with 32 rows two groups take alternate stages; with 64 rows the
// epilogue's registers leave room for one group.
template <int NR>
struct LhCfg {
  static constexpr int RAW = NR == 32 ? 8 : 4;   // packed stages in flight
  static constexpr int CONV = NR == 32 ? 4 : 2;  // converted A slots
  static constexpr int ACC = kLhTmemCols / NR;   // block accumulators
  static constexpr int AP = ACC / 4;              // accumulator sets of a pass (two stages, four blocks)
  static constexpr int CP = CONV / 2;             // A slot pairs (one pass each)
  static constexpr int NG = NR == 32 ? 2 : 1;    // converter groups (stage g: group g % NG)
  static constexpr int CONVW = 4 * NG;           // converter warps
  static constexpr int THREADS = (2 + CONVW + kLhEpiWarps) * 32;
  static_assert(RAW % NG == 0 && CONV % NG == 0, "a group's stages keep to its own ring slots");
};

// Dynamic shared memory: B (rows, K-major, swizzled) | CONV A slots | RAW
// packed stages | rounded logits of 32 rows x 128 features; 1024-byte
// aligned for the swizzle atoms.
template <int NR>
size_t lh_smem(int K) {
  using C = LhCfg<NR>;
  return 1024 + (size_t)NR * K * 2 + (size_t)C::CONV * kLhConv + (size_t)C::RAW * kLhRaw +
         (size_t)32 * kLhLgStride * 4;
}

template <typename T, int NR>
__global__ void __launch_bounds__(LhCfg<NR>::THREADS, 1)
    k_lm_head_tc(const T* __restrict__ x, int ldx, const int* __restrict__ row_map, const int* __restrict__ n_rows_ptr,
                 LinW W, GemvEpi ep, int* __restrict__ status) {
  using C = LhCfg<NR>;
  constexpr int RAW = C::RAW, CONV = C::CONV, ACC = C::ACC, AP = C::AP, CP = C::CP;
  extern __shared__ uint8_t smem_raw[];
  // The MMA warp works in passes of two stages (p = g / 2; n_stages is even
  // since K % 128 == 0), with one tcgen05.commit per pass on each of:
  //  * conv_free[p % CP]: the pass's MMAs have read its two A slots;
  //  * acc_full[p % AP]: its four block accumulators hold their sums;
  // and the epilogue's eight warps release a pass's accumulators on
  // acc_empty[p % AP]. With all 512 tensor-memory columns there are AP
  // passes of accumulators, so the MMAs and the converters run on through
  // the epilogue's end-of-tile work (logits, rounding, per-row best).
  __shared__ __align__(8) uint64_t full[RAW], empty[RAW], conv_full[CONV], conv_free[CP], acc_full[AP],
      acc_empty[AP], mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ float rs_s[NR];
  __shared__ uint32_t xmax_s[NR];  // largest |value| of each staged row (f32 bits)
  __shared__ int src_s[NR];        // source row of each staged row (-1: padding)
  __shared__ float inv_s[NR];      // 1 / the row's power-of-two operand scale
  __shared__ uint32_t sc_ring[2][kScaleAhead][kLhFeat];
  __shared__ int abort_s, stop_s;

  const int K = W.K, nkb = K / 64;
  const int n_tiles = W.N / kLhFeat;
  const int my_tiles = n_tiles > (int)blockIdx.x ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int n_stages = my_tiles * nkb;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t raw_u = smem_u32(smem_raw);
  const uint32_t base = (raw_u + 1023u) & ~1023u;
  uint8_t* base_p = smem_raw + (base - raw_u);
  const uint32_t xs = base;                                    // B: nkb blocks of NR rows x 128 bytes
  const uint32_t cv = xs + (uint32_t)NR * K * 2;               // A slots
  uint8_t* xs_p = base_p;
  uint8_t* cv_p = base_p + (size_t)NR * K * 2;
  uint8_t* rw_p = cv_p + (size_t)CONV * kLhConv;               // packed stages
  float* lg = reinterpret_cast<float*>(rw_p + (size_t)RAW * kLhRaw);  // [32][kLhLgStride]

  if (threadIdx.x == 0) {
    for (int i = 0; i < RAW; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);  // the four warps of the stage's converter group
    }
    for (int i = 0; i < CONV; ++i) {
      mbar_init(&conv_full[i], 4);
    }
    for (int i = 0; i < CP; ++i) mbar_init(&conv_free[i], 1);  // tcgen05.commit after the pass's MMAs
    for (int i = 0; i < AP; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kLhEpiWarps);  // both stage parities' four warps
    }
    mbar_init(&mma_done, 1);
    abort_s = 0;
    stop_s = 0;
    fence_barrier_init();
  }
  __syncthreads();
  volatile int* abort_v = &abort_s;

  // Parity waits never alias: each ring is waited on in use order by one
  // role, which has already seen the previous use of the same slot complete.
  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int tile = blockIdx.x + i * gridDim.x;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % RAW;
          if (g >= RAW && (*abort_v || !mbar_wait_bounded(&empty[s], ((g / RAW) + 1) & 1, kLhWaitLimit))) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kLhRaw);
          bulk_load(rw_p + (size_t)s * kLhRaw, W.pk + ((size_t)tile * nkb + kb) * kLhRaw, kLhRaw, &full[s]);
        }
      }
      if (!ok) *abort_v = 1;
      // copies still in flight land before the CTA retires (bounded)
      for (int j = g - RAW > 0 ? g - RAW : 0; j < g; ++j)
        mbar_wait_bounded(&full[j % RAW], (j / RAW) & 1, kLhWaitLimit);
    }
  } else if (warp == 1) {
    // tensor memory only after the dependency wait: the previous kernel has
    // then finished, so none of its CTAs can wait for these columns
    griddep_wait();
    griddep_launch();  // only after the wait: see griddep_launch
    tmem_alloc(&tmem_base_s, kLhTmemCols);
    tmem_relinquish();
    tc_fence_before();
    named_sync(2, (1 + kLhEpiWarps) * 32);  // with the epilogue: rows staged, columns allocated
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    {
      // the whole warp runs the loop; the elected lane issues (elect_one)
      constexpr uint32_t idesc = umma_idesc_f16(false, kLhFeat, NR);  // f16 operands
      bool ok = true;
      // two stages per pass, which halves this warp's loop and wait
      // instructions per stage; it shares its scheduler with converter and
      // epilogue warps, so its instruction count, not the MMAs, sets the pace
      for (int g = 0; ok && g < n_stages; g += 2) {
        const int p = g >> 1;
        if (*abort_v || !mbar_wait_warp(&conv_full[g % CONV], (g / CONV) & 1, kLhWaitLimit) ||
            !mbar_wait_warp(&conv_full[(g + 1) % CONV], ((g + 1) / CONV) & 1, kLhWaitLimit) ||
            (p >= AP && !mbar_wait_warp(&acc_empty[p % AP], ((p / AP) + 1) & 1, kLhWaitLimit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int gh = g + h, c = gh % CONV, kb = gh % nkb;
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              const uint32_t acc = tmem + (uint32_t)(((2 * gh + b) % ACC) * NR);
              const uint32_t at = cv + (uint32_t)c * kLhConv + b * 64, bt = xs + (uint32_t)kb * NR * 128 + b * 64;
              umma_f16(acc, umma_desc_sw128(at), umma_desc_sw128(bt), idesc, false);
              umma_f16(acc, umma_desc_sw128(at + 32), umma_desc_sw128(bt + 32), idesc, true);
            }
          }
          umma_commit(&conv_free[p % CP]);  // the pass's A slots are read once these MMAs complete
          umma_commit(&acc_full[p % AP]);   // and its accumulators hold the sums
        }
        __syncwarp();
      }
      if (!ok && lane == 0) *abort_v = 1;
      if (elect_one()) umma_commit(&mma_done);  // every MMA issued so far has completed when this fires
      __syncwarp();
      mbar_wait_warp(&mma_done, 0, kLhWaitLimit);
    }
    __syncwarp();
  } else if (warp < 2 + C::CONVW) {
    // ---- converters: group grp takes stages grp, grp + NG, ...; its warp cw
    // units cw and cw + 4 of each -> rows 16u .. 16u + 15 of the A tile
    const int grp = (warp - 2) >> 2, cw = (warp - 2) & 3, gq = lane >> 2, t = lane & 3;
    bool ok = true;
    for (int g = grp; ok && g < n_stages; g += C::NG) {
      const int s = g % RAW, c = g % CONV;
      // slot c is free once the MMAs of pass g / 2 - CP have completed
      const int p = g >> 1;
      if (p >= CP && (*abort_v || !mbar_wait_bounded(&conv_free[p % CP], ((p / CP) + 1) & 1, kLhWaitLimit))) {
        ok = false;
        break;
      }
      if (*abort_v || !mbar_wait_bounded(&full[s], (g / RAW) & 1, kLhWaitLimit)) {
        ok = false;
        break;
      }
      int4 qv[4];  // (unit cw, cw + 4) x (feature gq, gq + 8)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint8_t* un = rw_p + (size_t)s * kLhRaw + (size_t)(cw + 4 * (k >> 1)) * kUnitQ8;
        qv[k] = *reinterpret_cast<const int4*>(un + (k & 1) * 512 + lane * 16);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      // lane (gq, t) holds k [8t, 8t + 8) of block 0 and [32 + 8t, +8) of
      // block 1: 16-byte chunks t and 4 + t of the row. Odd rows store their
      // block-1 chunk first, so each quarter-warp store covers all 32 banks.
      uint8_t* tile = cv_p + (size_t)c * kLhConv;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int4 q = qv[k];
        const int r = (cw + 4 * (k >> 1)) * 16 + gq + 8 * (k & 1);
        uint32_t o[8];
        i8x4_to_act<__half>((uint32_t)q.x, o[0], o[1]);
        i8x4_to_act<__half>((uint32_t)q.y, o[2], o[3]);
        i8x4_to_act<__half>((uint32_t)q.z, o[4], o[5]);
        i8x4_to_act<__half>((uint32_t)q.w, o[6], o[7]);
        const int4 c0 = make_int4(o[0], o[1], o[2], o[3]), c1 = make_int4(o[4], o[5], o[6], o[7]);
        uint8_t* rowp = tile + r * 128;
        const int j0 = t ^ (r & 7), j1 = (4 + t) ^ (r & 7);
        if (r & 1) {
          *reinterpret_cast<int4*>(rowp + (j1 << 4)) = c1;
          *reinterpret_cast<int4*>(rowp + (j0 << 4)) = c0;
        } else {
          *reinterpret_cast<int4*>(rowp + (j0 << 4)) = c0;
          *reinterpret_cast<int4*>(rowp + (j1 << 4)) = c1;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // visible to tcgen05.mma
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv_full[c]);
    }
    if (!ok) *abort_v = 1;
  } else {
    // ---- epilogue warps: stage the rows, then the accumulators
    constexpr int NE = kLhEpiWarps * 32;
    const int et = threadIdx.x - (2 + C::CONVW) * 32;
    griddep_wait();
    griddep_launch();  // only after the wait: see griddep_launch
    const int rows = min(*n_rows_ptr, NR);
    const bool norm = ep.ssq != nullptr;  // else the rows are already normalised
    const int cpr = K >> 3;
    // the source row of each staged row first: the copies below need it
    for (int r = et; r < NR; r += NE) {
      xmax_s[r] = 0u;
      src_s[r] = r < rows ? (row_map ? row_map[r] : r) : -1;
    }
    named_sync(1, NE);
    // every 16-byte chunk of the rows in one round of copies (zeros past the
    // last row): chunk ch of row r is chunk ch % 8 of k-block ch / 8, stored
    // swizzled (chunk j of row r at j ^ (r % 8))
    for (int idx = et; idx < NR * cpr; idx += NE) {
      const int r = idx / cpr, ch = idx - r * cpr, sr = src_s[r];
      cp_async16(xs_p + (size_t)(ch >> 3) * NR * 128 + r * 128 + (((ch & 7) ^ (r & 7)) << 4),
                 sr >= 0 ? (const void*)(x + (size_t)sr * ldx + ch * 8) : (const void*)x, sr >= 0 ? 16 : 0);
    }
    cp_async_commit();
    if (norm) {  // the row norms, while the copies are in flight
      for (int r = et; r < rows; r += NE) {
        const float* sp = ep.ssq + (size_t)src_s[r] * ep.ssq_tiles;
        float ss = 0.f;
        for (int i0 = 0; i0 < ep.ssq_tiles; i0 += 16) {
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = i0 + i < ep.ssq_tiles ? sp[i0 + i] : 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) ss += v[i];
        }
        rs_s[r] = rsqrtf(ss / K + ep.eps);
      }
    }
    cp_async_wait<0>();
    named_sync(1, NE);
    if (norm || Act<T>::kIsBf16) {
      // RMSNorm in place (rounded to the activation type) and, for bf16 rows,
      // each row's largest |value|
      const T* nw = reinterpret_cast<const T*>(ep.norm_w);
      for (int idx = et; idx < rows * cpr; idx += NE) {
        const int r = idx / cpr, ch = idx - r * cpr;
        int4* pv = reinterpret_cast<int4*>(xs_p + (size_t)(ch >> 3) * NR * 128 + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
        int4 v = *pv;
        uint32_t* uv = reinterpret_cast<uint32_t*>(&v);
        if (norm) {
          const int4 wv = *reinterpret_cast<const int4*>(nw + ch * 8);
          const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv);
          const float rsr = rs_s[r];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Act<T>::unpack2(uv[e]);
            const float2 gw = Act<T>::unpack2(uw[e]);
            uv[e] = Act<T>::pack2(f.x * rsr * gw.x, f.y * rsr * gw.y);
          }
          *pv = v;
        }
        if constexpr (Act<T>::kIsBf16) {
          float m = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Act<T>::unpack2(uv[e]);
            m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
          }
          if (m > 0.f) atomicMax(&xmax_s[r], __float_as_uint(m));
        }
      }
    }
    named_sync(1, NE);
    if constexpr (Act<T>::kIsBf16) {
      // f16 operands: row r scaled by 2^(14 - e), e the exponent of its
      // largest |value|; the rounded bf16 values scale and convert exactly
      for (int r = et; r < NR; r += NE) {
        const uint32_t mb = xmax_s[r];
        const int e = (int)((mb >> 23) & 0xffu) - 127;
        const int sh = mb == 0u || e > 127 ? 0 : max(-126, min(126, 14 - e));  // 2^-sh stays a normal f32
        inv_s[r] = __uint_as_float((uint32_t)(127 - sh) << 23);
        rs_s[r] = __uint_as_float((uint32_t)(127 + sh) << 23);  // the staging's row scales are dead: reuse
      }
      named_sync(1, NE);
      const int cpr = K >> 3;
      for (int idx = et; idx < NR * cpr; idx += NE) {
        const int r = idx / cpr, ch = idx - r * cpr, kb = ch >> 3, jj = ch & 7;
        int4* pv = reinterpret_cast<int4*>(xs_p + (size_t)kb * NR * 128 + r * 128 + ((jj ^ (r & 7)) << 4));
        int4 v = *pv;
        uint32_t* uv = reinterpret_cast<uint32_t*>(&v);
        const float sc = rs_s[r];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = Act<T>::unpack2(uv[e]);
          uv[e] = Act<__half>::pack2(f.x * sc, f.y * sc);
        }
        *pv = v;
      }
    } else {
      for (int r = et; r < NR; r += NE) inv_s[r] = 1.f;
    }
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // the rows, visible to tcgen05.mma
    named_sync(2, (1 + kLhEpiWarps) * 32);
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    const int q = warp & 3, fl = q * 32 + lane;  // this thread's feature of a tile
    const int par = (et >> 7) & 1;               // warps 0-3 take the even stages, 4-7 the odd ones
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    // running best of rows j (+ 32) over this CTA's tiles: thread 8 j + fq
    // scans features [16 fq, 16 fq + 16) of row j of each tile
    const int jr = et >> 3, fq = et & 7;
    float rb_v[NR / 32];
    int rb_i[NR / 32];
#pragma unroll
    for (int h = 0; h < NR / 32; ++h) rb_v[h] = -INFINITY, rb_i[h] = 0x7fffffff;
    bool ok = true;  // this warp's waits all passed
    // scale words (block 0 | block 1 f16) of this feature for this warp's
    // stages: each thread copies its own word of its stage n + kScaleAhead - 1
    // (n counting the stages of its parity) into a private ring slot with
    // cp.async, one group per stage, far enough ahead to hide the L2 latency
    const int my_stages = (n_stages - par + 1) / 2;
    auto scale_fetch = [&](int n) {
      if (n < my_stages) {
        const int gs = 2 * n + par;
        const int tile = blockIdx.x + (gs / nkb) * gridDim.x, kb = gs % nkb;
        const uint8_t* un = W.pk + ((size_t)tile * nkb + kb) * kLhRaw + (size_t)(fl >> 4) * kUnitQ8 + 1024;
        cp_async4(&sc_ring[par][n % kScaleAhead][fl], reinterpret_cast<const uint32_t*>(un) + (fl & 15));
      }
      cp_async_commit();  // an empty group past the end keeps the group count per stage
    };
    for (int n = 0; n < kScaleAhead - 1; ++n) scale_fetch(n);
    // The eight warps take every tile's named barriers together whatever
    // their waits did: a warp whose wait gave up skips its tensor-memory
    // work, and all stop after the tile on a flag read between barriers.
    int n = 0;  // this warp's stages so far
    for (int i = 0; i < my_tiles; ++i) {
      const int tile = blockIdx.x + i * gridDim.x;
      float acc[NR];
#pragma unroll
      for (int j = 0; j < NR; ++j) acc[j] = 0.f;
      for (int kb = par; kb < nkb && ok; kb += 2, ++n) {
        const int g = i * nkb + kb;
        scale_fetch(n + kScaleAhead - 1);
        cp_async_wait<kScaleAhead - 1>();  // this stage's group has landed
        const uint32_t sc = sc_ring[par][n % kScaleAhead][fl];
        const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc));
        const int a0 = (2 * g) % ACC, a1 = (2 * g + 1) % ACC;
        // the tensor-memory loads are warp-wide: the warp goes on only if
        // the waits passed for all of its lanes
        const bool got = !*abort_v && mbar_wait_bounded(&acc_full[(g >> 1) % AP], ((g >> 1) / AP) & 1, kLhWaitLimit);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          *abort_v = 1;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < NR; c0 += 32) {
          // both blocks of the stage behind one wait; block 0 is added first
          uint32_t r0[32], r1[32];
          tmem_ld32(lane_base + (uint32_t)(a0 * NR + c0), r0);
          tmem_ld32(lane_base + (uint32_t)(a1 * NR + c0), r1);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            acc[c0 + j] = fmaf(d.y, __uint_as_float(r1[j]), fmaf(d.x, __uint_as_float(r0[j]), acc[c0 + j]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[(g >> 1) % AP]);
      }
      // the tile's logits: even-stage sum + odd-stage sum, scaled back and
      // rounded; per row the best (value, lowest index) of the tile
      const int f0 = tile * kLhFeat;
#pragma unroll
      for (int h = 0; h < NR / 32; ++h) {
        named_sync(1, NE);  // the previous half's reads are done
        // each parity hands the other its partial sums of half the rows
        // (odd: rows 0-15, even: rows 16-31), then completes the other half:
        // even sum + odd sum, scaled back, rounded
        // (register indices stay compile-time: the parity selects values)
        const int mine = par == 0 ? 0 : 16, theirs = 16 - mine;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          lg[(theirs + j) * kLhLgStride + fl] = par == 0 ? acc[h * 32 + 16 + j] : acc[h * 32 + j];
        named_sync(1, NE);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int r = mine + j;
          const float o = lg[r * kLhLgStride + fl];
          const float a = par == 0 ? acc[h * 32 + j] : acc[h * 32 + 16 + j];
          // the even stages' sum first, as a fixed order for both halves
          const float v = rnd<T>((par == 0 ? a + o : o + a) * inv_s[h * 32 + r]);
          lg[r * kLhLgStride + fl] = v;
          if (ep.logits && h * 32 + r < rows) ep.logits[(size_t)(h * 32 + r) * W.N + f0 + fl] = v;
        }
        named_sync(1, NE);
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        const float* lr = lg + jr * kLhLgStride + fq * 16;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int kk = (k + (fq >> 1)) & 15;  // the 32 lanes of a warp on 32 distinct banks
          const float v = lr[kk];
          const int ix = f0 + fq * 16 + kk;
          if (v > bv || (v == bv && ix < bi)) bv = v, bi = ix;
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
        }
        if (bv > rb_v[h] || (bv == rb_v[h] && bi < rb_i[h])) rb_v[h] = bv, rb_i[h] = bi;
      }
      named_sync(1, NE);
      if (et == 0) stop_s = *abort_v;
      named_sync(1, NE);
      if (stop_s) break;
    }
    if (!ok) *abort_v = 1;
    cp_async_wait<0>();  // no scale copy may land after the CTA retires
    if (fq == 0) {
#pragma unroll
      for (int h = 0; h < NR / 32; ++h) {
        const int r = h * 32 + jr;
        if (r < rows) {
          ep.best_val[(size_t)r * gridDim.x + blockIdx.x] = rb_v[h];
          ep.best_idx[(size_t)r * gridDim.x + blockIdx.x] = rb_i[h];
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort_v) report_timeout(status, kSiteLmHead);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base_s, kLhTmemCols);
  }
}

template <typename T, int NR>
int launch_t(const LinW& W, const void* x, int ldx, const int* row_map, const int* n_rows_ptr, const GemvEpi& ep,
             int* status, int n_sm, cudaStream_t s) {
  const size_t smem = lh_smem<NR>(W.K);
  // the opt-in limit covers dynamic plus static shared memory
  static size_t attr_set = 0;
  if (attr_set < smem) {
    const cudaError_t e = cudaFuncSetAttribute(k_lm_head_tc<T, NR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem);
    if (e != cudaSuccess) {
      cudaGetLastError();
      static bool told = false;
      if (!told)
        std::fprintf(stderr, "[fmd] tensor-core lm_head unavailable (%zu bytes of shared memory: %s); "
                             "the mma.sync kernel runs instead\n", smem, cudaGetErrorString(e));
      told = true;
      return 0;
    }
    attr_set = smem;
  }
  const int n_tiles = W.N / kLhFeat;
  const int grid = n_tiles < n_sm ? n_tiles : n_sm;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(LhCfg<NR>::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k_lm_head_tc<T, NR>, (const T*)x, ldx, row_map, n_rows_ptr, W, ep, status);
  return grid;
}

}  // namespace

int launch_lm_head_tc(ActType at, const LinW& W, const void* x, int ldx, const int* row_map, const int* n_rows_ptr,
                      int max_rows, const GemvEpi& ep, int* status, cudaStream_t s) {
  if (!W.q8 || W.pk == nullptr || max_rows > 64 || max_rows < 1 ||
      W.N % kLhFeat != 0 || W.K % 128 != 0 || ep.best_val == nullptr || ep.best_idx == nullptr)
    return 0;
  static int n_sm = 0;
  if (n_sm == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (n_sm <= 0) n_sm = 148;
  }
  if (at == kBF16)
    return max_rows <= 32 ? launch_t<__nv_bfloat16, 32>(W, x, ldx, row_map, n_rows_ptr, ep, status, n_sm, s)
                          : launch_t<__nv_bfloat16, 64>(W, x, ldx, row_map, n_rows_ptr, ep, status, n_sm, s);
  return max_rows <= 32 ? launch_t<__half, 32>(W, x, ldx, row_map, n_rows_ptr, ep, status, n_sm, s)
                        : launch_t<__half, 64>(W, x, ldx, row_map, n_rows_ptr, ep, status, n_sm, s);
}

}  // namespace fmd
