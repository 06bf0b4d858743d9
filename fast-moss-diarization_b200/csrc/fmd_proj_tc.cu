// Projections of a mixed (prefill-carrying) step as persistent tcgen05 GEMMs
// with the elementwise work that follows each one fused into the epilogue:
//  * qkv     -> per-head q/k RMSNorm, RoPE at each row's position, q to the
//               query buffer and k, v to the paged KV cache (qwen3.rs:211-227);
//  * gate/up -> SwiGLU, h = rnd(rnd(silu(rnd(g))) * rnd(u)) (qwen3.rs:288-292);
//  * o, down -> f32 rows for the residual add + RMSNorm kernel.
// The reference runs each projection as one candle matmul over the chunk's
// rows followed by separate elementwise ops (linear.rs:29-65 through
// qwen3.rs:211-338).
//
// One CTA per SM walks 128 x BN output tiles (tile t: row block t % m_tiles,
// feature block t / m_tiles, so the CTAs in flight share weight tiles in L2;
// the row count is read on the device, the plan of the step decides it):
//  * warp 0 (one lane) streams the k-blocks of the activations (16-bit,
//    128-byte swizzle) and of the weights by TMA through a STAGES-deep
//    full/empty mbarrier ring that runs on across tiles. Dense weights arrive
//    as the swizzled 16-bit tile the MMA reads; Q8_0 weights as their int8
//    tile (64-byte rows);
//  * Q8_0 only, warps 10-17: converters. Each k-block's BN x 64 int8 values
//    and their f16 block scales become q * d rounded to the activation type,
//    written in the swizzled layout, then a proxy fence and an arrival on the
//    stage's `conv` barrier;
//  * warp 1 allocates two BN-column f32 accumulators in tensor memory and,
//    the whole warp running the loop, its elected lane issues tcgen05.mma
//    (M = 128, N = BN, K = 16; four per k-block) into
//    accumulator i % 2, releasing each stage with tcgen05.commit;
//  * warps 2-9: the epilogue. Warp w owns tensor-memory lanes 32 (w % 4) ...
//    (32 rows of the tile) and half (w - 2) / 4 of its columns; with BN = 256
//    a half is one 128-wide head (qkv) or two gate/up groups (SwiGLU), so each
//    thread holds everything its row needs. The epilogue of tile i runs while
//    the MMAs of tile i + 1 fill the other accumulator.
// Every wait is bounded; a timeout sets the status word, every role stops,
// and the CTA waits (bounded) for its copies and MMAs in flight and frees its
// tensor memory before leaving.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "fmd_kernels.cuh"

namespace fmd {

namespace {

constexpr int kPBM = 128;
constexpr int kPBK = 64;
constexpr uint32_t kPWaitLimit = 1u << 24;

template <int BN, bool Q8>
constexpr int proj_stages() {
  return Q8 ? (BN == 256 ? 3 : 5) : (BN == 256 ? 4 : 6);
}
template <int BN, bool Q8>
constexpr size_t proj_smem() {
  return (size_t)proj_stages<BN, Q8>() * (kPBM * kPBK * 2 + BN * kPBK * 2 + (Q8 ? BN * kPBK : 0)) + 1024;
}
// Q8_0: 8 converter warps (warps 10-17); the dequantisation of a stage's
// int8 tile, not the MMAs, paces the Q8_0 k-loop, so it is split over as many
// warps as the registers allow (112 per thread at 576 threads)
constexpr int kPConvWarps = 8;
template <bool Q8>
constexpr int proj_threads() {
  return Q8 ? (10 + kPConvWarps) * 32 : 320;
}

// 16 int8 weights (one lane's 16 bytes) times their block scale, rounded to
// the activation type: 8 packed words in k order.
template <typename T>
FMD_DEV void dequant16(const int4 q, float d, uint32_t (&o)[8]) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&q);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t v = w[j] ^ 0x80808080u;  // biased bytes q + 128
    float f[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = (__int_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | i)) - 8388736.f) * d;
    o[2 * j] = Act<T>::pack2(f[0], f[1]);
    o[2 * j + 1] = Act<T>::pack2(f[2], f[3]);
  }
}

template <typename T>
FMD_DEV void store_row16(T* dst, const float (&v)[16]) {
  uint4 a, b;
  a.x = Act<T>::pack2(v[0], v[1]), a.y = Act<T>::pack2(v[2], v[3]);
  a.z = Act<T>::pack2(v[4], v[5]), a.w = Act<T>::pack2(v[6], v[7]);
  b.x = Act<T>::pack2(v[8], v[9]), b.y = Act<T>::pack2(v[10], v[11]);
  b.z = Act<T>::pack2(v[12], v[13]), b.w = Act<T>::pack2(v[14], v[15]);
  reinterpret_cast<uint4*>(dst)[0] = a;
  reinterpret_cast<uint4*>(dst)[1] = b;
}

template <typename T>
FMD_DEV void load_act16(const T* src, float (&v)[16]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(src)), b = __ldg(reinterpret_cast<const uint4*>(src) + 1);
  const uint32_t u[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 f = Act<T>::unpack2(u[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// qkv epilogue of one row and one 128-wide head held in tensor memory at
// `ta` (the row's lane, the head's first column).
template <typename T>
FMD_DEV void epi_qkv(uint32_t ta, int row, bool live, int hh, const ProjEpi& ep) {
  const int Hq = ep.Hq, Hkv = ep.Hkv;
  int pos = 0, page = 0;
  if (live) {
    pos = ep.plan.row_pos[row];
    if (hh >= Hq) {
      const int slot = ep.plan.row_slot[row];
      page = ep.kv.page_table[(size_t)slot * ep.kv.max_pages_per_slot + pos / kPageTokens];
    }
  }
  T* kvb = reinterpret_cast<T*>(ep.kv.base);
  T* dst;
  if (hh < Hq)
    dst = reinterpret_cast<T*>(ep.q_out) + (size_t)row * Hq * kHeadDim + hh * kHeadDim;
  else if (hh < Hq + Hkv)
    dst = kvb + ep.kv.elem_offset(ep.layer, page, 0, hh - Hq) + (size_t)(pos % kPageTokens) * kHeadDim;
  else
    dst = kvb + ep.kv.elem_offset(ep.layer, page, 1, hh - Hq - Hkv) + (size_t)(pos % kPageTokens) * kHeadDim;
  if (hh >= Hq + Hkv) {
    // v: the rounded projection as is
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      uint32_t r[16];
      tmem_ld16(ta + c * 16, r);
      tmem_ld_wait();
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
      if (live) store_row16<T>(dst + c * 16, v);
    }
    return;
  }
  // q / k: RMSNorm over the head of the rounded projection, then RoPE
  float ss = 0.f;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld32(ta + c * 32, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float v = rnd<T>(__uint_as_float(r[i]));
      ss += v * v;
    }
  }
  const float inv = rsqrtf(ss / kHeadDim + ep.eps);
  const T* nw = reinterpret_cast<const T*>(hh < Hq ? ep.qn_w : ep.kn_w);
  const T* cos_t = reinterpret_cast<const T*>(ep.cos) + (size_t)pos * (kHeadDim / 2);
  const T* sin_t = reinterpret_cast<const T*>(ep.sin) + (size_t)pos * (kHeadDim / 2);
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t rl[16], rh[16];
    tmem_ld16(ta + c * 16, rl);       // dims 16c ..
    tmem_ld16(ta + 64 + c * 16, rh);  // dims 64 + 16c .. (the RoPE partners)
    tmem_ld_wait();
    float wl[16], wh[16], cs[16], sn[16];
    load_act16<T>(nw + c * 16, wl);
    load_act16<T>(nw + 64 + c * 16, wh);
    load_act16<T>(cos_t + c * 16, cs);
    load_act16<T>(sin_t + c * 16, sn);
    float ol[16], oh[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float yl = rnd<T>(rnd<T>(__uint_as_float(rl[i])) * inv * wl[i]);
      const float yh = rnd<T>(rnd<T>(__uint_as_float(rh[i])) * inv * wh[i]);
      ol[i] = yl * cs[i] - yh * sn[i];
      oh[i] = yh * cs[i] + yl * sn[i];
    }
    if (live) {
      store_row16<T>(dst + c * 16, ol);
      store_row16<T>(dst + 64 + c * 16, oh);
    }
  }
}

// SwiGLU epilogue of one row: two interleaved groups (32 gate + 32 up
// features each) held in tensor memory at `ta`; group g of the tile is
// intermediate features [32 (col0 / 64 + g), + 32).
template <typename T>
FMD_DEV void epi_swiglu(uint32_t ta, int row, bool live, int col0, const ProjEpi& ep) {
#pragma unroll 1
  for (int j = 0; j < 2; ++j) {
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t rg[16], ru[16];
      tmem_ld16(ta + 64 * j + 16 * c, rg);
      tmem_ld16(ta + 64 * j + 32 + 16 * c, ru);
      tmem_ld_wait();
      float o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float gr = rnd<T>(__uint_as_float(rg[i]));
        const float sg = rnd<T>(gr / (1.f + expf(-gr)));
        o[i] = sg * rnd<T>(__uint_as_float(ru[i]));
      }
      if (live)
        store_row16<T>(reinterpret_cast<T*>(ep.h) + (size_t)row * ep.I + (col0 / 64 + j) * 32 + 16 * c, o);
    }
  }
}

template <typename T, int BN, int STAGES, bool Q8, int EPI>
__global__ void __launch_bounds__(proj_threads<Q8>(), 1)
    k_proj_tc(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
              const int* __restrict__ n_rows_ptr, int K, int N, const uint16_t* __restrict__ wd, ProjEpi ep,
              int* __restrict__ status) {
  constexpr uint32_t A_BYTES = kPBM * kPBK * 2;
  constexpr uint32_t B_BYTES = BN * kPBK * 2;
  constexpr uint32_t Q_BYTES = Q8 ? BN * kPBK : 0;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES + Q_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], conv[STAGES], acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t tiles = (raw + 1023u) & ~1023u;  // swizzle atoms need 1024-byte alignment
  uint8_t* tiles_p = smem_raw + (tiles - raw);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], kPConvWarps);  // Q8_0: one arrival per converter warp
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one arrival per epilogue warp
    }
    mbar_init(&mma_done, 1);
    abort_s = 0;
    fence_barrier_init();
  }
  // Tensor memory is allocated only after the dependency wait: the previous
  // kernel has then finished, so no CTA of it can be left waiting for the
  // columns this CTA holds.
  griddep_wait();  // the activations and the row count come from earlier kernels
  griddep_launch();  // only after the wait: see griddep_launch
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  volatile int* abort_v = &abort_s;

  const int n_rows = *n_rows_ptr;
  const int m_tiles = (n_rows + kPBM - 1) / kPBM;
  const int n_tiles = m_tiles * (N / BN);
  const int nk = K / kPBK;

  // Parity waits never alias: the ring and the two accumulators are each
  // waited on in use order by one role, which has already seen the previous
  // use of the same slot complete.
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&amap);
      prefetch_tmap(&bmap);
      int g = 0;  // k-block position in the ring across tiles
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
        const int row0 = (t % m_tiles) * kPBM, n0 = (t / m_tiles) * BN;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int st = g % STAGES;
          if (g >= STAGES &&
              (*abort_v || !mbar_wait_bounded(&empty[st], ((g / STAGES) + 1) & 1, kPWaitLimit))) {
            ok = false;
            break;
          }
          uint8_t* a = tiles_p + st * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[st], A_BYTES + (Q8 ? Q_BYTES : B_BYTES));
          tma_load_2d(a, &amap, kb * kPBK, row0, &full[st]);
          tma_load_2d(a + A_BYTES + (Q8 ? B_BYTES : 0), &bmap, kb * kPBK, n0, &full[st]);
        }
      }
      if (!ok) *abort_v = 1;
      // copies still in flight land before the CTA retires (bounded)
      for (int j = g - STAGES > 0 ? g - STAGES : 0; j < g; ++j)
        mbar_wait_bounded(&full[j % STAGES], (j / STAGES) & 1, kPWaitLimit);
    }
  } else if (warp == 1) {
    {
      // the whole warp runs the loop; the elected lane issues (elect_one)
      constexpr uint32_t idesc = umma_idesc_f16(Act<T>::kIsBf16, kPBM, BN);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (i >= 2 && (*abort_v || !mbar_wait_warp(&acc_empty[buf], ((i >> 1) - 1) & 1, kPWaitLimit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int st = g % STAGES;
          if (*abort_v || !mbar_wait_warp(&full[st], (g / STAGES) & 1, kPWaitLimit) ||
              (Q8 && !mbar_wait_warp(&conv[st], (g / STAGES) & 1, kPWaitLimit))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = tiles + st * STAGE_BYTES, b = a + A_BYTES;
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < kPBK / 16; ++j)
              umma_f16(acc, umma_desc_sw128(a + j * 32), umma_desc_sw128(b + j * 32), idesc, (kb | j) != 0);
            umma_commit(&empty[st]);  // the stage is free once these MMAs have read it
          }
          __syncwarp();
        }
        if (ok && elect_one()) umma_commit(&acc_full[buf]);
        __syncwarp();
      }
      if (!ok) *abort_v = 1;
      if (elect_one()) umma_commit(&mma_done);  // every MMA issued so far has completed when this fires
      __syncwarp();
      mbar_wait_warp(&mma_done, 0, kPWaitLimit);
    }
  } else if (warp >= 10) {
    if constexpr (Q8) {
      // converters: warp cw turns rows (cw % 4)*8 + 32*i + (lane >> 2), for the
      // 32-row bands i of parity cw / 4, of each stage's int8 tile into the
      // swizzled 16-bit B tile; lane & 3 picks 16 consecutive k (half a Q8_0
      // block), so a lane needs one scale. The stage's previous B tile is
      // free: the new copy landed only after the MMAs that read the old one
      // completed (the producer waited on empty).
      const int cw = (warp - 10) & 3, band = (warp - 10) >> 2, c = lane & 3;
      const int KB = K / 32;
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
        const int n0 = (t / m_tiles) * BN;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int st = g % STAGES;
          float dsc[BN / 64];  // the scales first: their latency overlaps the copy's
#pragma unroll
          for (int ii = 0; ii < BN / 64; ++ii) {
            const int r = cw * 8 + 32 * (2 * ii + band) + (lane >> 2);
            dsc[ii] = h2f_bits(__ldg(wd + (size_t)(n0 + r) * KB + kb * 2 + (c >> 1)));
          }
          if (*abort_v || !mbar_wait_bounded(&full[st], (g / STAGES) & 1, kPWaitLimit)) {
            ok = false;
            break;
          }
          const uint8_t* qt = tiles_p + st * STAGE_BYTES + A_BYTES + B_BYTES;
          uint8_t* bt = tiles_p + st * STAGE_BYTES + A_BYTES;
#pragma unroll
          for (int ii = 0; ii < BN / 64; ++ii) {
            const int r = cw * 8 + 32 * (2 * ii + band) + (lane >> 2);
            const int4 qv = *reinterpret_cast<const int4*>(qt + r * kPBK + c * 16);
            uint32_t o[8];
            dequant16<T>(qv, dsc[ii], o);
            // 16-byte chunk j of row r sits at chunk j ^ (r % 8) (128-byte swizzle)
            uint8_t* rowp = bt + r * 128;
            *reinterpret_cast<int4*>(rowp + (((2 * c) ^ (r & 7)) << 4)) = make_int4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<int4*>(rowp + (((2 * c + 1) ^ (r & 7)) << 4)) = make_int4(o[4], o[5], o[6], o[7]);
          }
          asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // visible to tcgen05.mma
          __syncwarp();
          if (lane == 0) mbar_arrive(&conv[st]);
        }
      }
      if (!ok) *abort_v = 1;
    }
  } else {
    // epilogue warps 2-9
    const int q = warp & 3, half = (warp - 2) >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    int i = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
      const int buf = i & 1;
      // the tensor-memory loads below are warp-wide: the warp goes on only
      // if the wait passed for all of its lanes
      const bool got = !*abort_v && mbar_wait_bounded(&acc_full[buf], (i >> 1) & 1, kPWaitLimit);
      if (!__all_sync(0xffffffffu, got)) {
        *abort_v = 1;
        break;
      }
      tc_fence_after();
      const int row = (t % m_tiles) * kPBM + q * 32 + lane;
      const bool live = row < n_rows;
      const int col0 = (t / m_tiles) * BN + half * (BN / 2);
      const uint32_t ta = lane_base + (uint32_t)(buf * BN + half * (BN / 2));
      if constexpr (EPI == kProjQkv) {
        epi_qkv<T>(ta, row, live, col0 / kHeadDim, ep);
      } else if constexpr (EPI == kProjSwiglu) {
        epi_swiglu<T>(ta, row, live, col0, ep);
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t r[32];
          tmem_ld32(ta + c * 32, r);
          tmem_ld_wait();
          if (live) {
            float4* o4 = reinterpret_cast<float4*>(ep.out + (size_t)row * N + col0 + c * 32);
#pragma unroll
            for (int k = 0; k < 8; ++k)
              o4[k] = make_float4(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1]),
                                  __uint_as_float(r[4 * k + 2]), __uint_as_float(r[4 * k + 3]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && abort_s) report_timeout(status, kSiteProjTc);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <typename T, int BN, bool Q8, int EPI>
void launch_t(const CUtensorMap& amap, const TcLinear& W, const int* n_rows_ptr, int max_rows, const ProjEpi& ep,
              int n_sm, int* status, cudaStream_t s) {
  const int max_tiles = (max_rows + kPBM - 1) / kPBM * (W.N / BN);
  launch_pdl(k_proj_tc<T, BN, proj_stages<BN, Q8>(), Q8, EPI>, dim3(max_tiles < n_sm ? max_tiles : n_sm),
             dim3(proj_threads<Q8>()), proj_smem<BN, Q8>(), s, amap, W.wmap, n_rows_ptr, W.K, W.N, W.d, ep, status);
}

template <typename T, int BN, bool Q8, int EPI>
cudaError_t set_smem() {
  return cudaFuncSetAttribute(k_proj_tc<T, BN, proj_stages<BN, Q8>(), Q8, EPI>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, (int)proj_smem<BN, Q8>());
}

template <typename T, bool Q8>
cudaError_t init_t() {
  for (cudaError_t e : {set_smem<T, 256, Q8, kProjQkv>(), set_smem<T, 256, Q8, kProjSwiglu>(),
                        set_smem<T, 128, Q8, kProjF32>()})
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

}  // namespace

cudaError_t init_proj_tc() {
  for (cudaError_t e : {init_t<__nv_bfloat16, false>(), init_t<__nv_bfloat16, true>(), init_t<__half, false>(),
                        init_t<__half, true>()})
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

// qkv and gate/up need 256-feature tiles (one head per epilogue half, two
// gate/up groups per half); o and down use 128-feature tiles. False (nothing
// launched) when the projection's plan does not fit.
bool launch_proj_tc(ActType at, int epi, const CUtensorMap& amap, const TcLinear& W, const int* n_rows_ptr,
                    int max_rows, const ProjEpi& ep, int n_sm, int* status, cudaStream_t s) {
  const int bn = epi == kProjF32 ? 128 : 256;
  if (!W.ok || W.bn != bn || W.N % bn || W.K % kPBK || (W.q8 && W.d == nullptr) || n_sm < 1) return false;
  if (epi == kProjQkv && (ep.Hq + 2 * ep.Hkv) * kHeadDim != W.N) return false;
  if (epi == kProjSwiglu && W.N != 2 * ep.I) return false;
#define FMD_P(T, Q8)                                                                                              \
  switch (epi) {                                                                                                  \
    case kProjQkv: launch_t<T, 256, Q8, kProjQkv>(amap, W, n_rows_ptr, max_rows, ep, n_sm, status, s); break;     \
    case kProjSwiglu: launch_t<T, 256, Q8, kProjSwiglu>(amap, W, n_rows_ptr, max_rows, ep, n_sm, status, s); break; \
    default: launch_t<T, 128, Q8, kProjF32>(amap, W, n_rows_ptr, max_rows, ep, n_sm, status, s); break;          \
  }
  if (at == kBF16) {
    if (W.q8) { FMD_P(__nv_bfloat16, true) } else { FMD_P(__nv_bfloat16, false) }
  } else {
    if (W.q8) { FMD_P(__half, true) } else { FMD_P(__half, false) }
  }
#undef FMD_P
  return true;
}

}  // namespace fmd
