// Split-KV GQA decode attention over the paged KV cache, B200 style.
//
// Computes `Attention::forward` of crates/fmd-core/src/model/qwen3.rs:229-257
// for one query token per sequence (decode): scores over every cached key,
// softmax, weighted sum of values, for the two query heads that share each kv
// head (GQA 16/8, qwen3.rs:237-241).
//
// Design:
//  * balanced ("stream-K") split: every (decode row, kv head) is a segment of
//    ceil(len / 64) page tiles; the segments, row-major then head, form one
//    sequence of T tiles, and CTA c of G owns tiles [c T / G, (c + 1) T / G).
//    Every CTA streams the same number of bytes whatever the context lengths.
//    A CTA derives the row prefix of tile counts itself (the rows' positions
//    and slots go to shared memory, one warp scans them).
//  * warp-specialised: a producer warp looks up the page ids of 32 tiles at
//    a time (one per lane), then streams each 64-position page tile of K and V
//    (2 x 16 KB) by TMA (cp.async.bulk.tensor.2d, 128B swizzle, no multicast),
//    plus a segment's two query rows (1D bulk copy) with its first tile, into a
//    3-stage shared-memory ring with full/empty mbarriers.
//  * each of the 4 consumer warps takes 16 positions of a tile: S = Q K^T and
//    O += P V on the tensor cores (mma.sync m16n8k16, rows 0/1 = the two query
//    heads), operands read with ldmatrix from the swizzled tiles
//    (conflict-free); online softmax in the exp2 domain per warp, merged across
//    warps at the end of the CTA's piece of a segment. The consumers walk the
//    tile sequence themselves, so every warp agrees on where pieces end.
//  * a segment that lies inside one CTA writes ctx directly. A segment cut by
//    CTA boundaries leaves (m, l, acc) partials in two slots per CTA (its first
//    and its last piece); the last of the segment's CTAs to finish (atomic
//    counter per (row, kv head), reset by that CTA) merges them and writes ctx.
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
constexpr int kMaxRows = 256;      // decode rows per pass (the slot limit)
constexpr uint32_t kWaitLimit = 1u << 22;

FMD_DEV uint32_t swz(int row, int chunk) {
  // byte offset of 16-byte `chunk` (0..15) of tile row `row` under the TMA
  // 128B swizzle, with the 128 dims split into two 64-dim boxes
  return (uint32_t)((chunk >> 3) * kBoxBytes + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// CTA whose range [c T / G, (c + 1) T / G) holds flattened tile x.
FMD_DEV int cta_of(long long x, long long T, int G) { return (int)(((x + 1) * G - 1) / T); }

template <typename T>
__global__ void __launch_bounds__(160, 2)
    k_attn_decode_tma(const __grid_constant__ CUtensorMap tmap, Plan p, int Hq, int Hkv, const T* __restrict__ q,
                      KvView kv, int layer, float scale_log2, float* __restrict__ part_acc,
                      float* __restrict__ part_ml, int* __restrict__ counters, T* __restrict__ ctx,
                      int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;                                           // [kStages][K 16 KB | V 16 KB]
  uint8_t* qbuf = smem + kStages * kTileBytes;                      // [kStages][2 heads x 256 B]
  float* red = reinterpret_cast<float*>(qbuf + kStages * kQBytes);  // [4 warps][2 heads][130]
  int* s_prefix = reinterpret_cast<int*>(red + 4 * 2 * kRedStride);  // [kMaxRows + 1] tiles before row r
  int* s_len = s_prefix + kMaxRows + 1;                              // [kMaxRows] kv length of row r
  int* s_slot = s_len + kMaxRows;                                    // [kMaxRows]
  uint64_t* full = reinterpret_cast<uint64_t*>(s_slot + kMaxRows + 1);  // 8-byte aligned (2 * 257 + 256 ints)
  uint64_t* empty = full + kStages;
  __shared__ int s_last;

  // The plan, the page table and the KV rows of earlier steps come from
  // grids that completed before this one started (griddep_launch): the
  // prologue and the first page tiles go ahead of the dependency wait. The
  // query rows and each row's newest K/V (the last tile of its segment) come
  // from the kernel right before: the producer waits before those copies.
  const int nd = min(p.counts->n_decode, kMaxRows);
  if (nd == 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_barrier_init();
    prefetch_tmap(&tmap);
  }
  for (int r = tid; r < nd; r += blockDim.x) {
    s_len[r] = p.row_pos[r] + 1;  // positions 0 .. pos, the row's own key included
    s_slot[r] = p.row_slot[r];
  }
  __syncthreads();
  if (warp == 0) {
    // tiles per row -> exclusive prefix (lane l holds rows 8l .. 8l+7)
    int loc[8], sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = lane * 8 + k;
      loc[k] = r < nd ? (s_len[r] + 63) >> 6 : 0;
      sum += loc[k];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - sum;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = lane * 8 + k;
      if (r < nd) s_prefix[r] = run;
      run += loc[k];
    }
    if (lane == 31) s_prefix[nd] = incl;  // total tiles per kv head
  }
  __syncthreads();
  const long long Tt = (long long)Hkv * s_prefix[nd];
  // with fewer tiles than CTAs only the first Tt take part, so that every
  // participating CTA owns at least one tile (the merge counts on it)
  const int G = (int)min((long long)gridDim.x, Tt), c = blockIdx.x;
  if (c >= G) return;
  const long long x0 = (long long)c * Tt / G, x1 = (long long)(c + 1) * Tt / G;
  const int ntl = (int)(x1 - x0);
  // (row, head, tile) of flattened tile x: the last row whose first tile is <= x
  auto locate = [&](long long x, int& r, int& h, int& j) {
    int lo = 0, hi = nd - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((long long)Hkv * s_prefix[mid] <= x) lo = mid;
      else hi = mid - 1;
    }
    r = lo;
    const int tr = s_prefix[r + 1] - s_prefix[r];
    const long long off = x - (long long)Hkv * s_prefix[r];
    h = (int)(off / tr);
    j = (int)(off - (long long)h * tr);
  };

  if (warp == 4) {
    // ---------------- producer warp: TMA tiles + query rows, runs ahead ----------------
    bool ok = true, waited = false;
    int issued = 0;
    // copies held back until the dependency wait: stage s's query rows
    // (row, head) and its newest K/V page
    int held_q[kStages], held_kv[kStages], held_y[kStages];
    for (int b0 = 0; b0 < ntl && ok; b0 += 32) {
      // lane i looks up tile b0 + i: its row, head, tile index and page
      int lr = 0, lh = 0, lj = 0, lpage = 0;
      if (b0 + lane < ntl) {
        locate(x0 + b0 + lane, lr, lh, lj);
        lpage = kv.page_table[(size_t)s_slot[lr] * kv.max_pages_per_slot + lj];
      }
      const int cnt = min(32, ntl - b0);
      for (int i = 0; i < cnt; ++i) {
        const int r = __shfl_sync(0xffffffffu, lr, i), h = __shfl_sync(0xffffffffu, lh, i);
        const int j = __shfl_sync(0xffffffffu, lj, i), page = __shfl_sync(0xffffffffu, lpage, i);
        const int tt = b0 + i, s = tt % kStages;
        if (!waited && tt >= kStages) {
          // the ring is full: wait for the kernel before, then issue what was held back
          griddep_wait();
          griddep_launch();  // only after the wait: see griddep_launch
          waited = true;
          if (lane == 0)
            for (int k = 0; k < kStages; ++k) {
              uint8_t* dst = stages + k * kTileBytes;
              if (held_kv[k]) {
                tma_load_2d(dst, &tmap, 0, held_y[k], &full[k]);
                tma_load_2d(dst + kBoxBytes, &tmap, 64, held_y[k], &full[k]);
                tma_load_2d(dst + 2 * kBoxBytes, &tmap, 0, held_y[k] + Hkv * kPageTokens, &full[k]);
                tma_load_2d(dst + 3 * kBoxBytes, &tmap, 64, held_y[k] + Hkv * kPageTokens, &full[k]);
              }
              if (held_q[k] >= 0) bulk_load(qbuf + k * kQBytes, q + (size_t)held_q[k], kQBytes, &full[k]);
            }
          __syncwarp();
        }
        if (tt >= kStages && !mbar_wait_bounded(&empty[s], ((tt / kStages) - 1) & 1, kWaitLimit)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const bool first = tt == 0 || j == 0;
          const bool newest = j == ((s_len[r] + 63) >> 6) - 1;  // holds the row's own (new) position
          const int yk = (int)(((((size_t)layer * kv.n_pages + page) * 2 + 0) * Hkv + h) * kPageTokens);
          const int yv = yk + Hkv * kPageTokens;
          uint8_t* dst = stages + s * kTileBytes;
          const int qoff = r * Hq * kHeadDim + 2 * h * kHeadDim;
          mbar_arrive_expect_tx(&full[s], kTileBytes + (first ? kQBytes : 0));
          if (waited || !newest) {
            tma_load_2d(dst, &tmap, 0, yk, &full[s]);
            tma_load_2d(dst + kBoxBytes, &tmap, 64, yk, &full[s]);
            tma_load_2d(dst + 2 * kBoxBytes, &tmap, 0, yv, &full[s]);
            tma_load_2d(dst + 3 * kBoxBytes, &tmap, 64, yv, &full[s]);
          }
          if (first && waited) bulk_load(qbuf + s * kQBytes, q + (size_t)qoff, kQBytes, &full[s]);
          if (!waited) {
            held_kv[s] = newest;
            held_y[s] = yk;
            held_q[s] = first ? qoff : -1;
          }
        }
        __syncwarp();
        issued = tt + 1;
      }
    }
    if (!waited) {
      // fewer tiles than stages: everything held back goes out now
      griddep_wait();
      griddep_launch();  // only after the wait: see griddep_launch
      waited = true;
      if (lane == 0 && ok)
        for (int k = 0; k < kStages && k < issued; ++k) {
          uint8_t* dst = stages + k * kTileBytes;
          if (held_kv[k]) {
            tma_load_2d(dst, &tmap, 0, held_y[k], &full[k]);
            tma_load_2d(dst + kBoxBytes, &tmap, 64, held_y[k], &full[k]);
            tma_load_2d(dst + 2 * kBoxBytes, &tmap, 0, held_y[k] + Hkv * kPageTokens, &full[k]);
            tma_load_2d(dst + 3 * kBoxBytes, &tmap, 64, held_y[k] + Hkv * kPageTokens, &full[k]);
          }
          if (held_q[k] >= 0) bulk_load(qbuf + k * kQBytes, q + (size_t)held_q[k], kQBytes, &full[k]);
        }
      __syncwarp();
    }
    if (!ok && lane == 0) {
      report_timeout(status, kSiteAttnDecode);
      // let the copies already issued land before the CTA can retire (bounded)
      for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
        mbar_wait_bounded(&full[i % kStages], (i / kStages) & 1, kWaitLimit);
    }
    return;
  }

  // ---------------- consumer warps 0..3: 16 positions of every tile each ----------------
  // ctx, the split partials and the merge counters are written only after
  // the kernel before has completed (it may still read ctx of the layer
  // before); the first tile's query rows arrive only after that anyway
  griddep_wait();
  bool aborted = false;
  int cr, ch, cj;  // the tile being consumed, walked forward from x0
  locate(x0, cr, ch, cj);
  int ctr = s_prefix[cr + 1] - s_prefix[cr];
  int pj0 = cj;    // first tile of the current piece
  uint32_t qf[8][2];
  float o[16][4];
  float m = -INFINITY, l = 0.f;
  for (int tt = 0; tt < ntl; ++tt) {
    const int s = tt % kStages;
    if (!aborted && !mbar_wait_bounded(&full[s], (tt / kStages) & 1, kWaitLimit)) aborted = true;
    const bool first = tt == 0 || cj == 0, last = tt == ntl - 1 || cj == ctr - 1;
    if (first) {
      pj0 = cj;
      m = -INFINITY;
      l = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      // A-fragment rows 0/1 = query heads 2h, 2h+1 (staged with the piece's first tile); rows 2..15 zero
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(qbuf + s * kQBytes + (g & 1) * 256);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qf[ks][0] = g < 2 ? qrow[ks * 8 + t] : 0u;
        qf[ks][1] = g < 2 ? qrow[ks * 8 + 4 + t] : 0u;
      }
    }
      const int nvalid = min(64, s_len[cr] - cj * 64);
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

    if (last) {
      // ---- merge the 4 consumer warps over this piece ----
      float lw = l;
      lw += __shfl_xor_sync(0xffffffffu, lw, 1);
      lw += __shfl_xor_sync(0xffffffffu, lw, 2);
      if (g < 2) {
        float* rw = red + (warp * 2 + g) * kRedStride;
#pragma unroll
        for (int dn = 0; dn < 16; ++dn) {
          rw[dn * 8 + 2 * t] = o[dn][0];
          rw[dn * 8 + 2 * t + 1] = o[dn][1];
        }
        if (t == 0) {
          rw[128] = m;
          rw[129] = lw;
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
      T* cdst = ctx + (size_t)cr * Hq * kHeadDim + (2 * ch + hd) * kHeadDim + d0;
      if (pj0 == 0 && cj == ctr - 1) {
        // the whole segment lies in this CTA
        if (!aborted) *reinterpret_cast<uint32_t*>(cdst) = Act<T>::pack2(A0 / L, A1 / L);
      } else {
        const long long seg0 = (long long)Hkv * s_prefix[cr] + (long long)ch * ctr;
        // slot 2c holds a piece that began in an earlier CTA, 2c + 1 one that continues in a later one
        const int slot = 2 * c + (seg0 < x0 ? 0 : 1);
        const size_t e = (size_t)slot * 2 + hd;
        part_acc[e * kHeadDim + d0] = A0;
        part_acc[e * kHeadDim + d0 + 1] = A1;
        if (d0 == 0) {
          part_ml[e * 2] = M;
          part_ml[e * 2 + 1] = L;
        }
        const int cf = cta_of(seg0, Tt, G), cl = cta_of(seg0 + ctr - 1, Tt, G);
        // the barrier orders every consumer's partial stores before thread
        // 0's fence (cumulative); the merging CTA's reads are ordered after its
        // fenced atomic the same way
        named_sync(1, 128);
        if (tid == 0) {
          __threadfence();
          s_last = atomicAdd(&counters[cr * Hkv + ch], 1) == cl - cf;
          if (s_last) __threadfence();
        }
        named_sync(1, 128);
        if (s_last) {
          float MM = -INFINITY;
          for (int cc = cf; cc <= cl; ++cc)
            MM = fmaxf(MM, __ldcg(&part_ml[((size_t)(2 * cc + (cc == cf ? 1 : 0)) * 2 + hd) * 2]));
          float LL = 0.f, B0 = 0.f, B1 = 0.f;
          for (int cc = cf; cc <= cl; ++cc) {
            const size_t e2 = (size_t)(2 * cc + (cc == cf ? 1 : 0)) * 2 + hd;
            const float wgt = exp2f(__ldcg(&part_ml[e2 * 2]) - MM);
            LL = fmaf(__ldcg(&part_ml[e2 * 2 + 1]), wgt, LL);
            B0 = fmaf(__ldcg(&part_acc[e2 * kHeadDim + d0]), wgt, B0);
            B1 = fmaf(__ldcg(&part_acc[e2 * kHeadDim + d0 + 1]), wgt, B1);
          }
          if (!aborted) *reinterpret_cast<uint32_t*>(cdst) = Act<T>::pack2(B0 / LL, B1 / LL);
          if (tid == 0) counters[cr * Hkv + ch] = 0;
        }
      }
      named_sync(1, 128);  // `red` is reused by the next piece
    }
    // advance to the next tile of the sequence
    if (++cj == ctr) {
      cj = 0;
      if (++ch == Hkv) {
        ch = 0;
        if (++cr < nd) ctr = s_prefix[cr + 1] - s_prefix[cr];
      }
    }
  }
  if (aborted && tid == 0) report_timeout(status, kSiteAttnDecode);
}

}  // namespace

size_t attn_decode_partial_floats(int grid) { return (size_t)2 * grid * 2 * (kHeadDim + 2); }

size_t attn_decode_smem_bytes() {
  return 1024 + kStages * (kTileBytes + kQBytes) + 4 * 2 * kRedStride * 4 + (3 * kMaxRows + 2) * 4 +
         2 * kStages * 8;
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
