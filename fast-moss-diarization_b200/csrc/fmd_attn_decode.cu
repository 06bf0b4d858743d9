// Split-KV GQA decode attention over the paged KV cache, B200 style.
//
// Computes `Attention::forward` of crates/fmd-core/src/model/qwen3.rs:229-257
// for one query token per sequence (decode): scores over every cached key,
// softmax, weighted sum of values, for the two query heads that share each kv
// head (GQA 16/8, qwen3.rs:237-241).
//
// Design:
//  * work unit = (split item of <= 256 positions of one sequence, kv head);
//    a persistent grid (2 CTAs per SM) strides over all units.
//  * warp-specialised: a producer warp streams every 64-position page tile of
//    K and V (2 x 16 KB) by TMA (cp.async.bulk.tensor.2d, 128B swizzle, no
//    multicast), plus the unit's two query rows by 1D bulk copy, into a
//    3-stage shared-memory ring with full/empty mbarriers; it runs ahead across
//    work-unit boundaries, so the ring never drains while there is work.
//  * each of the 4 consumer warps takes 16 positions of a tile: S = Q K^T and O += P V
//    on the tensor cores (mma.sync m16n8k16, rows 0/1 = the two query heads),
//    operands read with ldmatrix from the swizzled tiles (conflict-free);
//    online softmax in the exp2 domain per warp, merged across warps at the
//    end of the unit.
//  * split units of one sequence merge without a second kernel: each writes
//    (m, l, acc) partials, and the last unit to finish (atomic counter per
//    (row, kv head), reset by that unit) merges them and writes ctx.
//  * every mbarrier wait is bounded; on timeout the kernel records
//    FMD_ETIMEDOUT in a status word, drains its outstanding copies (bounded)
//    and returns.
#include <cuda.h>
#include <float.h>
#include <math.h>

#include "fmd_kernels.cuh"

namespace fmd {

namespace {

constexpr int kStages = 3;
constexpr int kTileBytes = 32768;  // K (16 KB) + V (16 KB) of one page of one kv head
constexpr int kBoxBytes = 8192;    // 64 positions x 64 dims x 2 bytes
constexpr int kRedStride = 130;    // 128 dims + m + l
constexpr int kQBytes = 512;       // query rows of the two heads of a kv head (2 x 128 x 2 bytes)
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr int kStatusTimeout = -110;

FMD_DEV uint32_t swz(int row, int chunk) {
  // byte offset of 16-byte `chunk` (0..15) of tile row `row` under the TMA
  // 128B swizzle, with the 128 dims split into two 64-dim boxes
  return (uint32_t)((chunk >> 3) * kBoxBytes + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

template <typename T>
__global__ void __launch_bounds__(160, 2)
    k_attn_decode_tma(const __grid_constant__ CUtensorMap tmap, Plan p, int Hq, int Hkv, const T* __restrict__ q,
                      KvView kv, int layer, float scale_log2, float* __restrict__ part_acc,
                      float* __restrict__ part_ml, int* __restrict__ counters, T* __restrict__ ctx,
                      int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;                                        // [kStages][K 16 KB | V 16 KB]
  uint8_t* qbuf = smem + kStages * kTileBytes;                   // [kStages][2 heads x 256 B]
  float* red = reinterpret_cast<float*>(qbuf + kStages * kQBytes);  // [4 warps][2 heads][130]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 4 * 2 * kRedStride);
  uint64_t* empty = full + kStages;
  __shared__ int s_last;

  griddep_launch();
  griddep_wait();
  const int n_work = p.counts->n_ditems * Hkv;
  if ((int)blockIdx.x >= n_work) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_barrier_init();
    prefetch_tmap(&tmap);
  }
  __syncthreads();

  if (warp == 4) {
    // ---------------- producer warp: TMA tiles + query rows, runs ahead ----------------
    uint32_t j = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
      const int it = w / Hkv, hh = w % Hkv;
      const int r = p.di_row[it];
      const int slot = p.row_slot[r];
      const int k0 = p.di_start[it], k1 = p.di_end[it];
      const int nt = (k1 - k0 + 63) >> 6;  // <= 4: a unit spans at most kDecodeItemTokens positions
      const int my_page = lane < nt ? kv.page_table[(size_t)slot * kv.max_pages_per_slot + (k0 >> 6) + lane] : 0;
      const T* qsrc = q + (size_t)r * Hq * kHeadDim + 2 * hh * kHeadDim;
      for (int tile = 0; tile < nt; ++tile, ++j) {
        const int page = __shfl_sync(0xffffffffu, my_page, tile);
        const int s = j % kStages;
        if (j >= (uint32_t)kStages && !mbar_wait_bounded(&empty[s], ((j / kStages) - 1) & 1, kWaitLimit)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const int yk = (int)(((((size_t)layer * kv.n_pages + page) * 2 + 0) * Hkv + hh) * kPageTokens);
          const int yv = yk + Hkv * kPageTokens;
          uint8_t* dst = stages + s * kTileBytes;
          mbar_arrive_expect_tx(&full[s], kTileBytes + (tile == 0 ? kQBytes : 0));
          tma_load_2d(dst, &tmap, 0, yk, &full[s]);
          tma_load_2d(dst + kBoxBytes, &tmap, 64, yk, &full[s]);
          tma_load_2d(dst + 2 * kBoxBytes, &tmap, 0, yv, &full[s]);
          tma_load_2d(dst + 3 * kBoxBytes, &tmap, 64, yv, &full[s]);
          if (tile == 0) bulk_load(qbuf + s * kQBytes, qsrc, kQBytes, &full[s]);
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      atomicExch(status, kStatusTimeout);
      // let the copies already issued land before the CTA can retire (bounded)
      for (uint32_t i = j > (uint32_t)kStages ? j - kStages : 0; i < j; ++i)
        mbar_wait_bounded(&full[i % kStages], (i / kStages) & 1, kWaitLimit);
    }
    return;
  }

  // ---------------- consumer warps 0..3: 16 positions of every tile each ----------------
  uint32_t j = 0;
  bool aborted = false;
  for (int w = blockIdx.x; w < n_work; w += gridDim.x) {
    const int it = w / Hkv, h = w % Hkv;
    const int r = p.di_row[it], k0 = p.di_start[it], k1 = p.di_end[it];
    const int ntiles = (k1 - k0 + 63) >> 6;
    uint32_t qf[8][2];
    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m = -INFINITY, l = 0.f;

    for (int tile = 0; tile < ntiles; ++tile, ++j) {
      const int s = j % kStages;
      if (!aborted && !mbar_wait_bounded(&full[s], (j / kStages) & 1, kWaitLimit)) aborted = true;
      if (tile == 0) {
        // A-fragment rows 0/1 = query heads 2h, 2h+1 (staged with the unit's first tile); rows 2..15 zero
        const uint32_t* qrow = reinterpret_cast<const uint32_t*>(qbuf + s * kQBytes + (g & 1) * 256);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          qf[ks][0] = g < 2 ? qrow[ks * 8 + t] : 0u;
          qf[ks][1] = g < 2 ? qrow[ks * 8 + 4 + t] : 0u;
        }
      }
      const int nvalid = min(64, k1 - (k0 + tile * 64));
      if (!aborted && warp * 16 < nvalid) {
        const uint32_t kb = smem_u32(stages + s * kTileBytes);
        const uint32_t vb = kb + 2 * kBoxBytes;
        const int mi = lane >> 3;
        float sc[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.f;
        {
          const int tok = warp * 16 + (mi >> 1) * 8 + (lane & 7);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            uint32_t rr[4];
            ldmatrix_x4(rr, kb + swz(tok, 2 * ks + (mi & 1)));
            const uint32_t a[4] = {qf[ks][0], 0u, qf[ks][1], 0u};
            mma16816<T>(sc[0], a, rr[0], rr[1]);
            mma16816<T>(sc[1], a, rr[2], rr[3]);
          }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int tok = warp * 16 + nt * 8 + 2 * t + e;
            sc[nt][e] = tok < nvalid ? sc[nt][e] * scale_log2 : -INFINITY;
            mx = fmaxf(mx, sc[nt][e]);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m, mx);  // finite: position warp*16 is valid
        const float corr = exp2f(m - mn);
        float ps = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            sc[nt][e] = exp2f(sc[nt][e] - mn);
            ps += sc[nt][e];
          }
        l = l * corr + ps;
        m = mn;
#pragma unroll
        for (int dn = 0; dn < 16; ++dn) {
          o[dn][0] *= corr;
          o[dn][1] *= corr;
        }
        const uint32_t pa[4] = {Act<T>::pack2(sc[0][0], sc[0][1]), 0u, Act<T>::pack2(sc[1][0], sc[1][1]), 0u};
        const int tok = warp * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {
          uint32_t rr[4];
          ldmatrix_x4_trans(rr, vb + swz(tok, 2 * dp + (mi >> 1)));
          mma16816<T>(o[2 * dp], pa, rr[0], rr[1]);
          mma16816<T>(o[2 * dp + 1], pa, rr[2], rr[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with stage s
    }

    // ---- merge the 4 consumer warps of this unit ----
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (g < 2) {
      float* rw = red + (warp * 2 + g) * kRedStride;
#pragma unroll
      for (int dn = 0; dn < 16; ++dn) {
        rw[dn * 8 + 2 * t] = o[dn][0];
        rw[dn * 8 + 2 * t + 1] = o[dn][1];
      }
      if (t == 0) {
        rw[128] = m;
        rw[129] = l;
      }
    }
    named_sync(1, 128);
    const int hd = tid >> 6, d0 = (tid & 63) * 2;
    float M = -INFINITY;
#pragma unroll
    for (int w4 = 0; w4 < 4; ++w4) M = fmaxf(M, red[(w4 * 2 + hd) * kRedStride + 128]);
    float L = 0.f, A0 = 0.f, A1 = 0.f;
#pragma unroll
    for (int w4 = 0; w4 < 4; ++w4) {
      const float* rw = red + (w4 * 2 + hd) * kRedStride;
      const float wgt = exp2f(rw[128] - M);  // a warp with no valid position: exp2(-inf) = 0
      L = fmaf(rw[129], wgt, L);
      A0 = fmaf(rw[d0], wgt, A0);
      A1 = fmaf(rw[d0 + 1], wgt, A1);
    }
    const int nit = p.drow_nitems[r];
    T* cdst = ctx + (size_t)r * Hq * kHeadDim + (2 * h + hd) * kHeadDim + d0;
    if (nit == 1) {
      if (!aborted) *reinterpret_cast<uint32_t*>(cdst) = Act<T>::pack2(A0 / L, A1 / L);
    } else {
      const size_t e = (size_t)it * Hq + 2 * h + hd;
      part_acc[e * kHeadDim + d0] = A0;
      part_acc[e * kHeadDim + d0 + 1] = A1;
      if (d0 == 0) {
        part_ml[e * 2] = M;
        part_ml[e * 2 + 1] = L;
      }
      __threadfence();
      named_sync(1, 128);
      if (tid == 0) s_last = atomicAdd(&counters[r * Hkv + h], 1) == nit - 1;
      named_sync(1, 128);
      if (s_last) {
        __threadfence();
        const int i0 = p.drow_item0[r];
        float MM = -INFINITY;
        for (int i = 0; i < nit; ++i) MM = fmaxf(MM, __ldcg(&part_ml[((size_t)(i0 + i) * Hq + 2 * h + hd) * 2]));
        float LL = 0.f, B0 = 0.f, B1 = 0.f;
        for (int i = 0; i < nit; ++i) {
          const size_t e2 = (size_t)(i0 + i) * Hq + 2 * h + hd;
          const float wgt = exp2f(__ldcg(&part_ml[e2 * 2]) - MM);
          LL = fmaf(__ldcg(&part_ml[e2 * 2 + 1]), wgt, LL);
          B0 = fmaf(__ldcg(&part_acc[e2 * kHeadDim + d0]), wgt, B0);
          B1 = fmaf(__ldcg(&part_acc[e2 * kHeadDim + d0 + 1]), wgt, B1);
        }
        if (!aborted) *reinterpret_cast<uint32_t*>(cdst) = Act<T>::pack2(B0 / LL, B1 / LL);
        if (tid == 0) counters[r * Hkv + h] = 0;
      }
    }
    named_sync(1, 128);  // `red` is reused by the next unit
  }
  if (aborted && tid == 0) atomicExch(status, kStatusTimeout);
}

}  // namespace

size_t attn_decode_smem_bytes() {
  return 1024 + kStages * (kTileBytes + kQBytes) + 4 * 2 * kRedStride * 4 + 2 * kStages * 8;
}

cudaError_t init_attn_decode() {
  const int bytes = (int)attn_decode_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(k_attn_decode_tma<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       bytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_attn_decode_tma<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

void launch_attn_decode_tma(ActType at, const void* tmap, const Plan& p, int grid, int Hq, int Hkv, const void* q,
                            const KvView& kv, int layer, float scale, float* part_acc, float* part_ml, int* counters,
                            void* ctx, int* status, cudaStream_t s) {
  const float scale_log2 = scale * 1.4426950408889634f;
  const CUtensorMap& m = *reinterpret_cast<const CUtensorMap*>(tmap);
  const size_t smem = attn_decode_smem_bytes();
  if (at == kBF16)
    launch_pdl(k_attn_decode_tma<__nv_bfloat16>, dim3(grid), dim3(160), smem, s, m, p, Hq, Hkv, (const __nv_bfloat16*)q, kv, layer,
                                                             scale_log2, part_acc, part_ml, counters,
                                                             (__nv_bfloat16*)ctx, status);
  else
    launch_pdl(k_attn_decode_tma<__half>, dim3(grid), dim3(160), smem, s, m, p, Hq, Hkv, (const __half*)q, kv, layer, scale_log2,
                                                      part_acc, part_ml, counters, (__half*)ctx, status);
}

}  // namespace fmd
