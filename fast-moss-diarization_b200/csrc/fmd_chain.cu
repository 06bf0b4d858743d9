// The tail of a decode layer as one persistent launch: o_proj (+ residual,
// qwen3.rs:333-334) -> gate/up (post-attention RMSNorm, SwiGLU, qwen3.rs:
// 288-292) -> down (+ residual, qwen3.rs:336-338) -> the next layer's fused
// qkv (input RMSNorm, per-head q/k RMSNorm, RoPE, KV-cache write, qwen3.rs:
// 211-227).
//
// Why: a decode step multiplies ~32 rows by each projection, so each of
// these four GEMVs moves 2-7 MB of Q8_0 weights, ~1 us at HBM speed, but as
// separate launches each costs ~10 us of launch, dependency and drain
// latency. Here the four run in one launch of thread-block clusters:
//  * every projection is in the decode-packed Q8_0 layout of the GEMV
//    (fmd_gemv.cuh): T feature tiles of `ft` features, each split 8 ways
//    along K into contiguous units. A cluster of 8 CTAs owns whole tiles
//    (tiles c, c + NC, ... of cluster c); CTA rank r computes split r of each,
//    so a CTA stages one activation slice per projection;
//  * before griddepcontrol.wait, one thread per CTA issues a TMA bulk copy
//    for each of its weight units of all four projections (~130 KB per SM:
//    the layer's 16.7 MB stream at full bandwidth while the previous kernel
//    drains);
//  * per projection: stage the slice (cp.async.cg: the inputs were written by
//    other clusters), normalise it for the normed projections, run the exact
//    Q8_0 MMAs of fmd_gemv.cuh per (tile, 16 features) warp task into f32
//    partial tiles in shared memory; a cluster barrier; rank r sums rows
//    r, r + 8, ... over the 8 CTAs' partials through distributed shared
//    memory in the fixed order 0..7 and applies the projection's epilogue
//    with the reference's rounding points;
//  * a grid barrier separates the projections: a cluster barrier, one
//    release-add per cluster on a global counter that rank 0 then polls
//    (acquire), and a cluster barrier again.
// The split-K reduction never leaves the cluster, so a projection costs one
// round trip through L2 for its inputs and two for the barrier.
// Every wait on global memory is bounded (iterations and 0.5 s of wall
// time); a wait that gives up sets the status word and the kernel runs on to
// its end (the results are then wrong, never a hang), draining its own
// weight copies before it exits. The counters are cleared by the step's
// first kernel (k_embed_norm). One CTA per SM and a grid of at most the
// clusters the GPU can hold at once (cudaOccupancyMaxActiveClusters) keep
// every CTA resident, which the grid barrier relies on.
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <cstdio>

#include "fmd_gemv.cuh"
#include "fmd_kernels.cuh"

namespace cg = cooperative_groups;

namespace fmd {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCS = 8;            // CTAs per cluster = the K split of every projection
constexpr int kMaxUnits = 16;     // weight units (bulk copies) one CTA may own over the four projections
constexpr int kTailRows = kChainMaxRows;  // rows served (4 MMA n-tiles)
static_assert(kTailRows == 32, "the MMA loops hold 4 n-tiles of 8 rows");
constexpr int kMaxRounds = 4;     // warp tasks (tile, 16 features) per warp and projection
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr uint32_t kSpinLimit = 1u << 17;

struct Geom {
  int T, S, ft, fw, klen, nkb;
  uint32_t ubytes;
};

FMD_HD Geom geom_of(const ChainPhase& p) {
  Geom g;
  g.ft = p.ft;
  g.fw = p.ft / 16;
  g.S = p.S;
  g.T = p.N / p.ft;
  g.klen = p.K / p.S;
  g.nkb = g.klen / 64;
  g.ubytes = (uint32_t)(g.nkb * g.fw * kUnitQ8);
  return g;
}

// One activation slice in shared memory: kTailRows rows of klen features
// (+ the GEMV's bank padding), 16-byte multiple.
FMD_HD uint32_t slice_bytes(const Geom& q) { return (uint32_t)kTailRows * (q.klen + x_pad<true>()) * 2; }

// Tiles of cluster c among NC clusters.
FMD_HD int tiles_of(int T, int c, int NC) { return T > c ? (T - 1 - c) / NC + 1 : 0; }

FMD_DEV int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
FMD_DEV void red_release(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

// All CTAs of the grid: each CTA fences its global writes at gpu scope, the
// cluster barrier gathers the cluster at rank 0, rank 0 counts the cluster on
// the global counter with release semantics and polls it with acquire until
// every cluster has arrived, and a second cluster barrier hands that on.
FMD_DEV void grid_barrier(cg::cluster_group& cluster, int* bar, int n_clusters, int* status) {
  __syncthreads();
  if (threadIdx.x == 0) __threadfence();  // the CTA's global writes, at gpu scope
  cluster.sync();
  if (cluster.block_rank() == 0 && threadIdx.x == 0) {
    red_release(bar, 1);
    const uint64_t t0 = globaltimer_ns();
    bool ok = false;
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
      if (ld_acquire(bar) >= n_clusters) {
        ok = true;
        break;
      }
      if ((i & 63) == 63 && globaltimer_ns() - t0 > kWaitNsCap) break;
      __nanosleep(32);
    }
    if (!ok) report_timeout(status, kSiteLayerTail);
  }
  cluster.sync();
}

template <typename T>
FMD_DEV float2 ldcg_act2(const T* p) {
  const uint32_t u = __ldcg(reinterpret_cast<const unsigned int*>(p));
  return Act<T>::unpack2(u);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_layer_tail(ChainArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t wbar[kMaxUnits];
  __shared__ float rs_s[kTailRows];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int NC = gridDim.x / kCS, cl = blockIdx.x / kCS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int np = a.n_phases;

  // ---- this CTA's weight units (split `rank` of each of its cluster's tiles)
  uint32_t woff[4];
  int ntl[4], bidx[4];
  uint32_t wtot = 0;
  int nunits = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    ntl[p] = 0;
    woff[p] = wtot;
    bidx[p] = nunits;
    if (p < np) {
      const Geom q = geom_of(a.ph[p]);
      ntl[p] = tiles_of(q.T, cl, NC);
      wtot += (uint32_t)ntl[p] * q.ubytes;
      nunits += ntl[p];
    }
  }
  // then the activation slice. After a projection's MMAs, its f32 partial
  // tiles [row][feature] (rows padded by 4 floats: the MMA fragment stores
  // hit 32 distinct banks) take the place of its weight units.
  uint8_t* act = smem + ((wtot + 127u) & ~127u);
  if (threadIdx.x == 0) {
    for (int i = 0; i < nunits; ++i) mbar_init(&wbar[i], 1);
    fence_barrier_init();
    // every weight unit of the layer tail: no dependency on earlier kernels
    for (int p = 0; p < np; ++p) {
      const Geom q = geom_of(a.ph[p]);
      for (int i = 0; i < ntl[p]; ++i) {
        const int tile = cl + i * NC;
        mbar_arrive_expect_tx(&wbar[bidx[p] + i], q.ubytes);
        bulk_load(smem + woff[p] + (uint32_t)i * q.ubytes, a.ph[p].pk + ((size_t)tile * q.S + rank) * q.ubytes,
                  q.ubytes, &wbar[bidx[p] + i]);
      }
    }
  }
  __syncthreads();  // barrier initialisation visible to every thread
  griddep_wait();   // ctx (attention) and every earlier write are visible
  griddep_launch();  // only after the wait: see griddep_launch

  const int n_rows = min(*a.n_rows_ptr, kTailRows);
  const int n_nt = (n_rows + 7) >> 3;
  bool ok = true;

  for (int p = 0; p < np; ++p) {
    const Geom q = geom_of(a.ph[p]);
    const int K = a.ph[p].K, nt = ntl[p];
    const int PS = q.ft + 4;  // partial row stride (floats)
    // inputs: o <- ctx, gate/up <- norm(x), down <- h, qkv <- norm(x)
    const T* in = reinterpret_cast<const T*>(p == 0 ? a.ctx : p == 2 ? a.h : a.x);
    const T* norm_w = reinterpret_cast<const T*>(p == 1 ? a.post_norm : p == 3 ? a.in_norm : nullptr);
    const int xstride = q.klen + x_pad<true>();
    const int kbeg = rank * q.klen;
    T* xs = reinterpret_cast<T*>(act);
    if (nt > 0 && n_rows > 0) {
      const int cpr = q.klen >> 3;
      for (int ci = threadIdx.x; ci < n_nt * 8 * cpr; ci += kThreads) {
        const int r = ci / cpr, ch = ci - r * cpr;
        const bool live = r < n_rows;
        cp_async16(xs + (size_t)r * xstride + ch * 8, live ? in + (size_t)r * K + kbeg + ch * 8 : in, live ? 16 : 0);
      }
      cp_async_commit();
      if (norm_w != nullptr) {
        // rsqrt(mean(x^2) + eps) from the per-64-feature sums of squares the
        // residual epilogues wrote: a row's partials in flight together
        for (int r = threadIdx.x; r < n_rows; r += kThreads) {
          const float* sp = a.ssq + (size_t)r * a.ssq_tiles;
          float ss = 0.f;
          for (int i0 = 0; i0 < a.ssq_tiles; i0 += 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = i0 + i < a.ssq_tiles ? __ldcg(sp + i0 + i) : 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) ss += v[i];
          }
          rs_s[r] = rsqrtf(ss / a.H + a.eps);
        }
      }
      cp_async_wait<0>();
      __syncthreads();
      if (norm_w != nullptr) {
        const T* nw = norm_w + kbeg;
        for (int ci = threadIdx.x; ci < n_rows * cpr; ci += kThreads) {
          const int r = ci / cpr, ch = ci - r * cpr;
          int4* pv = reinterpret_cast<int4*>(xs + (size_t)r * xstride + ch * 8);
          int4 v = *pv;
          const int4 wv = *reinterpret_cast<const int4*>(nw + ch * 8);
          uint32_t* u = reinterpret_cast<uint32_t*>(&v);
          const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv);
          const float rsr = rs_s[r];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Act<T>::unpack2(u[e]);
            const float2 gw = Act<T>::unpack2(uw[e]);
            u[e] = Act<T>::pack2(f.x * rsr * gw.x, f.y * rsr * gw.y);
          }
          *pv = v;
        }
        __syncthreads();
      }
      // warp tasks (tile, 16-feature slice), up to kMaxRounds per warp, held
      // in registers until every warp is done with the projection's weights:
      // tile i's f32 partials then overwrite tile i's weight unit
      const int n_tasks = nt * q.fw;
      float res[kMaxRounds][4][4];
#pragma unroll
      for (int rd = 0; rd < kMaxRounds; ++rd) {
#pragma unroll
        for (int i = 0; i < 4; ++i) res[rd][i][0] = res[rd][i][1] = res[rd][i][2] = res[rd][i][3] = 0.f;
        const int task = rd * kWarps + warp;
        if (task >= n_tasks) continue;
        const int ti = task / q.fw, f = task - ti * q.fw;
        if (!mbar_wait_bounded(&wbar[bidx[p] + ti], 0, kWaitLimit)) {
          ok = false;
          continue;
        }
        const uint8_t* wu = smem + woff[p] + (uint32_t)ti * q.ubytes;
#pragma unroll 1
        for (int kb = 0; kb < q.nkb; ++kb) {
          WRegs w;
          gemv_wload<true>(wu + (size_t)(kb * q.fw + f) * kUnitQ8, lane, w);
          uint32_t af[4][4];
          gemv_afrag<T, true>(w, af);
#pragma unroll
          for (int n8 = 0; n8 < 4; ++n8) {
            if (n8 < n_nt) {
              uint32_t xw[8];
              gemv_xfrag<T, true>(xs + (size_t)(n8 * 8 + g) * xstride + kb * 64, t, xw);
              gemv_kblock<T, true>(res[rd][n8], af, xw, w);
            }
          }
        }
      }
      __syncthreads();  // the projection's weight units are dead from here on
#pragma unroll
      for (int rd = 0; rd < kMaxRounds; ++rd) {
        const int task = rd * kWarps + warp;
        if (task >= n_tasks) continue;
        const int ti = task / q.fw, f = task - ti * q.fw;
        // D fragment: features f*16 + g (+8), rows n8*8 + 2t (+1)
        float* pt = reinterpret_cast<float*>(smem + woff[p] + (uint32_t)ti * q.ubytes);
        const int fl = f * 16 + g;
#pragma unroll
        for (int n8 = 0; n8 < 4; ++n8) {
          if (n8 < n_nt) {
            const int lr = n8 * 8 + 2 * t;
            pt[lr * PS + fl] = res[rd][n8][0];
            pt[(lr + 1) * PS + fl] = res[rd][n8][1];
            pt[lr * PS + fl + 8] = res[rd][n8][2];
            pt[(lr + 1) * PS + fl + 8] = res[rd][n8][3];
          }
        }
      }
    }
    cluster.sync();  // every CTA's partial tiles written (distributed shared memory)

    // ---- rank r finishes rows r, r + 8, ... of each tile of the cluster:
    // the 8 partials summed in the fixed order 0..7, then the epilogue
    const int rows_per = (n_rows + kCS - 1 - rank) / kCS;  // rows r = rank + kCS * j < n_rows
    const int n_work = nt * (rows_per > 0 ? rows_per : 0);
    for (int wi = warp; wi < n_work; wi += kWarps) {
      const int ti = wi / rows_per, r = rank + kCS * (wi - ti * rows_per);
      const int tile = cl + ti * NC;
      const int FPL = q.ft / 32;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      T* xr = reinterpret_cast<T*>(a.x) + (size_t)r * a.H + tile * 64 + lane * 2;
      float2 xo = make_float2(0.f, 0.f);
      if (p == 0 || p == 2) xo = ldcg_act2(xr);  // in flight with the peer reads
      const float* mine =
          reinterpret_cast<const float*>(smem + woff[p] + (uint32_t)ti * q.ubytes) + (size_t)r * PS + lane * FPL;
#pragma unroll
      for (int s = 0; s < kCS; ++s) {
        const float* peer = cluster.map_shared_rank(mine, s);
        if (FPL == 4) {
          const float4 z = *reinterpret_cast<const float4*>(peer);
          v[0] += z.x, v[1] += z.y, v[2] += z.z, v[3] += z.w;
        } else {
          const float2 z = *reinterpret_cast<const float2*>(peer);
          v[0] += z.x, v[1] += z.y;
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = rnd<T>(v[i]);
      if (p == 0 || p == 2) {
        // x <- rnd(x + rnd(y)) and the tile's sum of squares of the new x
        const float n0 = rnd<T>(xo.x + v[0]), n1 = rnd<T>(xo.y + v[1]);
        *reinterpret_cast<uint32_t*>(xr) = Act<T>::pack2(n0, n1);
        const float ss = warp_sum(n0 * n0 + n1 * n1);
        if (lane == 0) a.ssq[(size_t)r * a.ssq_tiles + tile] = ss;
      } else if (p == 1) {
        // features [0, 32) gate, [32, 64) up of intermediate index tile*32 + j
        const float g0 = __shfl_sync(0xffffffffu, v[0], lane >> 1), g1 = __shfl_sync(0xffffffffu, v[1], lane >> 1);
        const float u0v = __shfl_sync(0xffffffffu, v[0], 16 + (lane >> 1));
        const float u1v = __shfl_sync(0xffffffffu, v[1], 16 + (lane >> 1));
        const float gv = (lane & 1) ? g1 : g0, uv = (lane & 1) ? u1v : u0v;
        const float sg = rnd<T>(gv / (1.f + expf(-gv)));
        reinterpret_cast<T*>(a.h)[(size_t)r * a.I + tile * 32 + lane] = Act<T>::from_f(sg * uv);
      } else {
        // one head per tile: q/k RMSNorm, RoPE at the row's position, q to
        // the query buffer, k and v to the next layer's KV pages
        const int hh = tile, Hq = a.Hq, Hkv = a.Hkv;
        const int pos = a.plan.row_pos[r], slot = a.plan.row_slot[r];
        T* kvb = reinterpret_cast<T*>(a.kv.base);
        T* dst;
        if (hh < Hq + Hkv) {
          const T* nwh = reinterpret_cast<const T*>(hh < Hq ? a.qn_w : a.kn_w) + lane * 4;
          const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
          const float inv = rsqrtf(ss / kHeadDim + a.eps);
          float y[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) y[i] = rnd<T>(v[i] * inv * Act<T>::to_f(nwh[i]));
          const T* cos_t = reinterpret_cast<const T*>(a.cos) + (size_t)pos * (kHeadDim / 2) + (lane & 15) * 4;
          const T* sin_t = reinterpret_cast<const T*>(a.sin) + (size_t)pos * (kHeadDim / 2) + (lane & 15) * 4;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float pr2 = __shfl_xor_sync(0xffffffffu, y[i], 16);
            const float cs = Act<T>::to_f(cos_t[i]), sn = Act<T>::to_f(sin_t[i]);
            v[i] = lane < 16 ? y[i] * cs - pr2 * sn : pr2 * sn + y[i] * cs;
          }
          if (hh < Hq) {
            dst = reinterpret_cast<T*>(a.q_out) + (size_t)r * Hq * kHeadDim + hh * kHeadDim;
          } else {
            const int page = a.kv.page_table[(size_t)slot * a.kv.max_pages_per_slot + pos / kPageTokens];
            dst = kvb + a.kv.elem_offset(a.layer, page, 0, hh - Hq) + (size_t)(pos % kPageTokens) * kHeadDim;
          }
        } else {
          const int page = a.kv.page_table[(size_t)slot * a.kv.max_pages_per_slot + pos / kPageTokens];
          dst = kvb + a.kv.elem_offset(a.layer, page, 1, hh - Hq - Hkv) + (size_t)(pos % kPageTokens) * kHeadDim;
        }
        uint2 o;
        o.x = Act<T>::pack2(v[0], v[1]);
        o.y = Act<T>::pack2(v[2], v[3]);
        *reinterpret_cast<uint2*>(dst + lane * 4) = o;
      }
    }
    // the next projection overwrites the partial tiles that peers read above:
    // the grid barrier's first cluster barrier keeps them until every peer is
    // done; after the last projection a cluster barrier does the same before
    // the CTA (and its shared memory) goes away
    if (p + 1 < np)
      grid_barrier(cluster, a.sync + p, NC, a.status);
    else
      cluster.sync();
  }
  if (!ok && threadIdx.x == 0) report_timeout(a.status, kSiteLayerTail);
  // no copy may still be landing when the CTA's shared memory is released
  if (threadIdx.x == 0)
    for (int i = 0; i < nunits; ++i)
      if (!mbar_wait_bounded(&wbar[i], 0, kWaitLimit)) report_timeout(a.status, kSiteLayerTail);
}

// Shared memory of a CTA for `n_clusters` clusters: the weight units of the
// CTA holding the most, then the widest activation slice. 0 if the layer
// tail cannot serve the shapes (each partial tile must fit in its weight
// unit, and each warp holds at most kMaxRounds tasks of a projection).
size_t tail_smem(const ChainArgs& a, int n_clusters) {
  size_t wmax = 0, slice = 0;
  for (int c = 0; c < n_clusters; ++c) {
    size_t w = 0;
    int units = 0;
    for (int p = 0; p < a.n_phases; ++p) {
      const Geom q = geom_of(a.ph[p]);
      w += (size_t)tiles_of(q.T, c, n_clusters) * q.ubytes;
      units += tiles_of(q.T, c, n_clusters);
    }
    if (units > kMaxUnits) return 0;
    wmax = w > wmax ? w : wmax;
  }
  for (int p = 0; p < a.n_phases; ++p) {
    const Geom q = geom_of(a.ph[p]);
    if (q.S != kCS || q.klen % 64 != 0 || (q.ft != 64 && q.ft != 128) || q.T * q.ft != a.ph[p].N) return 0;
    if ((size_t)kTailRows * (q.ft + 4) * 4 > q.ubytes) return 0;
    if (tiles_of(q.T, 0, n_clusters) * q.fw > kMaxRounds * kWarps) return 0;
    slice = std::max(slice, (size_t)slice_bytes(q));
  }
  return ((wmax + 127) & ~(size_t)127) + slice;
}

template <typename T>
cudaError_t max_clusters(size_t smem, int* n) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCS * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaFuncSetAttribute(k_layer_tail<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveClusters(n, k_layer_tail<T>, &cfg);
}

}  // namespace

// The cluster count and shared memory of the layer tail for rows <= 32:
// as many clusters as the GPU holds at once (at most one per 8 SMs), fewer
// if the weights of the CTAs then no longer fit. False if it cannot run.
bool chain_plan(ActType at, const ChainArgs& a, int n_sm, int max_rows, int* n_clusters, size_t* smem, char* why,
                size_t why_len) {
  if (max_rows > kChainMaxRows || n_sm < kCS) {
    snprintf(why, why_len, "max_rows %d > %d or %d SMs", max_rows, kChainMaxRows, n_sm);
    return false;
  }
  int nc = n_sm / kCS;
  for (int iter = 0; iter < 8 && nc >= 1; ++iter) {
    const size_t b = tail_smem(a, nc);
    if (b == 0 || b > 226 * 1024) {
      snprintf(why, why_len, "%d clusters: shared memory %zu bytes (0 = shapes not served)", nc, b);
      return false;
    }
    int fit = 0;
    const cudaError_t e =
        at == kBF16 ? max_clusters<__nv_bfloat16>(b, &fit) : max_clusters<__half>(b, &fit);
    if (e != cudaSuccess) {
      snprintf(why, why_len, "%d clusters of %zu bytes: %s", nc, b, cudaGetErrorString(e));
      cudaGetLastError();
      return false;
    }
    if (fit >= nc) {
      *n_clusters = nc;
      *smem = b;
      return true;
    }
    snprintf(why, why_len, "%d clusters of %zu bytes requested, %d resident at once", nc, b, fit);
    nc = fit;
  }
  return false;
}

void launch_layer_tail(ActType at, const ChainArgs& a, int n_clusters, size_t smem, cudaStream_t s) {
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kCS;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCS * n_clusters);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (at == kBF16)
    cudaLaunchKernelEx(&cfg, k_layer_tail<__nv_bfloat16>, a);
  else
    cudaLaunchKernelEx(&cfg, k_layer_tail<__half>, a);
}

}  // namespace fmd
