// The tail of a decode layer as one persistent launch: o_proj (+ residual,
// qwen3.rs:333-334) -> gate/up (post-attention RMSNorm, SwiGLU, qwen3.rs:
// 288-292) -> down (+ residual, qwen3.rs:336-338) -> the next layer's fused
// qkv (input RMSNorm, per-head q/k RMSNorm, RoPE, KV-cache write, qwen3.rs:
// 211-227).
//
// Why: a decode step multiplies ~32 rows by each projection, so each of
// these four GEMVs moves 2-7 MB of Q8_0 weights, ~1 us at HBM speed, but as
// separate launches each costs ~10 us of launch, dependency and drain
// latency. Here one CTA per SM runs all four, with the dependencies between
// them (every feature of the previous output feeds every CTA) carried by
// grid barriers in global memory, and the whole layer's weights requested at
// kernel start:
//  * phase p is one projection in the decode-packed Q8_0 layout of the GEMV
//    (fmd_gemv.cuh): T feature tiles of `ft` features x S k-splits = T*S
//    units, each a contiguous block in HBM. CTA c owns a contiguous chunk
//    of the units in split-major order, so its units of a phase share one
//    or two activation slices. Before griddepcontrol.wait, one thread issues
//    a TMA bulk copy per unit for all four phases (about 113 KB per SM: the
//    16.7 MB of a layer stream at full bandwidth while the previous kernel
//    drains);
//  * per phase: stage the activation slices (through L2: cp.async.cg; the
//    inputs were written by other CTAs), normalise them for the normed
//    projections, run the exact Q8_0 MMAs of fmd_gemv.cuh per (unit, 16
//    features) warp task, and write f32 partials [s][row][feature] to
//    global memory; then count the unit on its tile's counter (release);
//  * the S CTAs of a tile each wait for the tile's count to reach S
//    (acquire) and reduce rows r = s (mod S) in the fixed order s' = 0..S-1
//    (deterministic), applying the phase's epilogue with the reference's
//    rounding points;
//  * a grid barrier separates the phases.
// Every wait is bounded: a wait that gives up sets the status word and the
// kernel runs on to its end (the results are then wrong, never a hang),
// draining its own weight copies before it exits. The counters are cleared
// by the step's first kernel (k_embed_norm). One CTA per SM (the shared
// memory footprint allows no second one) and a grid no larger than the SM
// count keep every CTA resident, which the grid barriers rely on.
#include <cuda_runtime.h>
#include <math.h>

#include "fmd_gemv.cuh"
#include "fmd_kernels.cuh"

namespace fmd {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxUnits = 16;  // weight units (bulk copies) one CTA may own over the four phases
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr uint32_t kSpinLimit = 1u << 17;  // polls of a global counter (each after a short sleep): ~0.1 s

struct Geom {
  int T, S, ft, fw, klen, nkb, U;
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
  g.U = g.T * g.S;
  g.ubytes = (uint32_t)(g.nkb * g.fw * kUnitQ8);
  return g;
}

// CTA c's units [u0, u1) of a phase with U units on G CTAs.
FMD_HD void unit_range(int U, int c, int G, int& u0, int& u1) {
  u0 = (int)((long long)U * c / G);
  u1 = (int)((long long)U * (c + 1) / G);
}

FMD_DEV int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Add with release semantics: every write this thread has observed (the
// CTA's writes, after a __syncthreads) is visible before the count.
FMD_DEV void red_release(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
FMD_DEV int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;\n" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Thread 0 polls *p until it reaches `target` (bounded); false if it gave up.
FMD_DEV bool spin_until(const int* p, int target) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (ld_acquire(p) >= target) return true;
    if ((i & 63) == 63 && globaltimer_ns() - t0 > kWaitNsCap) return false;
    __nanosleep(32);
  }
  return false;
}

// All CTAs of the grid: every write before it is visible to every CTA after.
// Two levels, so that no address takes more than ~16 atomics: CTA c counts
// on group counter c % 16; the last arrival of a group counts on the top
// counter, which every CTA then polls. `bar` holds 17 counters.
constexpr int kBarGroups = 16;
FMD_DEV void grid_barrier(int* bar, int* status) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const int grp = blockIdx.x % kBarGroups;
    const int members = ((int)gridDim.x - grp + kBarGroups - 1) / kBarGroups;
    const int groups = min((int)gridDim.x, kBarGroups);
    if (atom_add_acq_rel(bar + 1 + grp, 1) == members - 1) red_release(bar, 1);
    if (!spin_until(bar, groups)) report_timeout(status, kSiteLayerTail);
  }
  __syncthreads();
}

// L2-coherent loads of data other CTAs of this launch wrote.
FMD_DEV float2 ldcg_f2(const float* p) { return __ldcg(reinterpret_cast<const float2*>(p)); }
FMD_DEV float4 ldcg_f4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

template <typename T>
FMD_DEV float2 ldcg_act2(const T* p) {
  const uint32_t u = __ldcg(reinterpret_cast<const unsigned int*>(p));
  return Act<T>::unpack2(u);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_layer_tail(ChainArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t wbar[kMaxUnits];
  __shared__ float rs_s[kChainMaxRows];
  griddep_launch();
  const int G = gridDim.x, c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int np = a.n_phases;

  // ---- this CTA's units of every phase and where their weights go
  uint32_t woff[4];
  int ub[4], ue[4], bidx[4];
  uint32_t wtot = 0;
  int nunits = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    ub[p] = ue[p] = 0;
    woff[p] = wtot;
    bidx[p] = nunits;
    if (p < np) {
      const Geom q = geom_of(a.ph[p]);
      unit_range(q.U, c, G, ub[p], ue[p]);
      wtot += (uint32_t)(ue[p] - ub[p]) * q.ubytes;
      nunits += ue[p] - ub[p];
    }
  }
  uint8_t* act = smem + ((wtot + 127u) & ~127u);
  if (threadIdx.x == 0) {
    for (int i = 0; i < nunits; ++i) mbar_init(&wbar[i], 1);
    fence_barrier_init();
    // every weight unit of the layer tail: no dependency on earlier kernels
    for (int p = 0; p < np; ++p) {
      const Geom q = geom_of(a.ph[p]);
      for (int u = ub[p]; u < ue[p]; ++u) {
        const int tile = u % q.T, s = u / q.T, i = bidx[p] + u - ub[p];
        mbar_arrive_expect_tx(&wbar[i], q.ubytes);
        bulk_load(smem + woff[p] + (uint32_t)(u - ub[p]) * q.ubytes,
                  a.ph[p].pk + ((size_t)tile * q.S + s) * q.ubytes, q.ubytes, &wbar[i]);
      }
    }
  }
  __syncthreads();  // barrier initialisation visible to every thread
  griddep_wait();   // ctx (attention) and every earlier write are visible

  const int n_rows = min(*a.n_rows_ptr, kChainMaxRows);
  const int n_nt = (n_rows + 7) >> 3;
  bool ok = true;
  int* const bars = a.sync + 4 * kChainMaxTiles;  // 3 barriers of 1 + kBarGroups counters

  for (int p = 0; p < np; ++p) {
    const Geom q = geom_of(a.ph[p]);
    const int u0 = ub[p], u1 = ue[p];
    int* const ctr = a.sync + p * kChainMaxTiles;
    const int N = a.ph[p].N, K = a.ph[p].K;
    // inputs: o <- ctx, gate/up <- norm(x), down <- h, qkv <- norm(x)
    const T* in = reinterpret_cast<const T*>(p == 0 ? a.ctx : p == 2 ? a.h : a.x);
    const T* norm_w = reinterpret_cast<const T*>(p == 1 ? a.post_norm : p == 3 ? a.in_norm : nullptr);
    const int xstride = q.klen + x_pad<true>();
    const int slot_bytes = kChainMaxRows * xstride * 2;  // one activation slice, laid out for the most rows
    if (u1 > u0 && n_rows > 0) {
      const int s_lo = u0 / q.T, s_hi = (u1 - 1) / q.T;  // at most two slices
      const int cpr = q.klen >> 3;
      for (int j = 0; j <= s_hi - s_lo; ++j) {
        T* xs = reinterpret_cast<T*>(act + (size_t)j * slot_bytes);
        const int kbeg = (s_lo + j) * q.klen;
        for (int ci = threadIdx.x; ci < n_nt * 8 * cpr; ci += kThreads) {
          const int r = ci / cpr, ch = ci - r * cpr;
          const bool live = r < n_rows;
          cp_async16(xs + (size_t)r * xstride + ch * 8, live ? in + (size_t)r * K + kbeg + ch * 8 : in, live ? 16 : 0);
        }
      }
      cp_async_commit();
      if (norm_w != nullptr) {
        // rsqrt(mean(x^2) + eps) from the per-64-feature sums of squares the
        // residual epilogues wrote: a row's 16 partials in flight together,
        // summed in order
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
        for (int j = 0; j <= s_hi - s_lo; ++j) {
          T* xs = reinterpret_cast<T*>(act + (size_t)j * slot_bytes);
          const T* nw = norm_w + (s_lo + j) * q.klen;
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
        }
        __syncthreads();
      }
      // warp tasks: (unit, 16-feature slice)
      const int n_tasks = (u1 - u0) * q.fw;
      for (int task = warp; task < n_tasks; task += kWarps) {
        const int ui = task / q.fw, f = task - ui * q.fw, u = u0 + ui;
        const int tile = u % q.T, s = u / q.T;
        if (!mbar_wait_bounded(&wbar[bidx[p] + ui], 0, kWaitLimit)) {
          ok = false;
          continue;
        }
        const uint8_t* wu = smem + woff[p] + (uint32_t)ui * q.ubytes;
        const T* xs = reinterpret_cast<const T*>(act + (size_t)(s - s_lo) * slot_bytes);
        float acc[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll 1
        for (int kb = 0; kb < q.nkb; ++kb) {
          WRegs w;
          gemv_wload<true>(wu + (size_t)(kb * q.fw + f) * kUnitQ8, lane, w);
          uint32_t af[4][4];
          gemv_afrag<T, true>(w, af);
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) {
            if (nt < n_nt) {
              uint32_t xw[8];
              gemv_xfrag<T, true>(xs + (size_t)(nt * 8 + g) * xstride + kb * 64, t, xw);
              gemv_kblock<T, true>(acc[nt], af, xw, w);
            }
          }
        }
        // f32 partials [s][row][feature]
        float* pp = a.part + (size_t)s * kChainMaxRows * N + tile * q.ft + f * 16 + g;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          if (nt < n_nt) {
            const int r = nt * 8 + 2 * t;
            if (r < n_rows) {
              pp[(size_t)r * N] = acc[nt][0];
              pp[(size_t)r * N + 8] = acc[nt][2];
            }
            if (r + 1 < n_rows) {
              pp[(size_t)(r + 1) * N] = acc[nt][1];
              pp[(size_t)(r + 1) * N + 8] = acc[nt][3];
            }
          }
        }
      }
      __syncthreads();
      if (threadIdx.x == 0)  // the CTA's partials before the counts
        for (int u = u0; u < u1; ++u) red_release(ctr + u % q.T, 1);
    }

    // ---- reduction + epilogue: unit (tile, s) finishes rows r = s (mod S).
    // One poll over the tile counters of all of this CTA's units, then every
    // (unit, row) pair on its own warp, all in parallel.
    if (u1 > u0 && n_rows > 0) {
      __shared__ int wait_ok;
      if (threadIdx.x == 0) {
        bool all = true;
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t it = 0;; ++it) {
          all = true;
          for (int u = u0; u < u1; ++u) all &= ld_acquire(ctr + u % q.T) >= q.S;
          if (all || it >= kSpinLimit || ((it & 63) == 63 && globaltimer_ns() - t0 > kWaitNsCap)) break;
          __nanosleep(32);
        }
        wait_ok = all;
      }
      __syncthreads();
      if (!wait_ok) ok = false;
      const int rows_per = (n_rows + q.S - 1) / q.S;  // rows of residue s: s, s + S, ...
      const int n_work = (u1 - u0) * rows_per;
      for (int wi = warp; wi < n_work; wi += kWarps) {
        const int u = u0 + wi / rows_per, tile = u % q.T, s = u / q.T;
        const int r = s + q.S * (wi % rows_per);
        if (r >= n_rows) continue;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        const float* pr = a.part + (size_t)r * N + tile * q.ft;
        T* xr = reinterpret_cast<T*>(a.x) + (size_t)r * a.H + tile * 64 + lane * 2;
        float2 xo = make_float2(0.f, 0.f);
        if (p == 0 || p == 2) xo = ldcg_act2(xr);  // in flight with the partials
        if (q.ft == 128) {
          float4 z[8];
#pragma unroll
          for (int sp = 0; sp < 8; ++sp)
            if (sp < q.S) z[sp] = ldcg_f4(pr + (size_t)sp * kChainMaxRows * N + lane * 4);
#pragma unroll
          for (int sp = 0; sp < 8; ++sp)
            if (sp < q.S) v[0] += z[sp].x, v[1] += z[sp].y, v[2] += z[sp].z, v[3] += z[sp].w;
        } else {
          float2 z[8];
#pragma unroll
          for (int sp = 0; sp < 8; ++sp)
            if (sp < q.S) z[sp] = ldcg_f2(pr + (size_t)sp * kChainMaxRows * N + lane * 2);
#pragma unroll
          for (int sp = 0; sp < 8; ++sp)
            if (sp < q.S) v[0] += z[sp].x, v[1] += z[sp].y;
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
    }
    if (p + 1 < np) grid_barrier(bars + p * (1 + kBarGroups), a.status);
  }
  if (!ok && threadIdx.x == 0) report_timeout(a.status, kSiteLayerTail);
  // no copy may still be landing when the CTA's shared memory is released
  // (units whose tasks were skipped: no rows, or a wait that gave up)
  if (threadIdx.x == 0)
    for (int i = 0; i < nunits; ++i)
      if (!mbar_wait_bounded(&wbar[i], 0, kWaitLimit)) report_timeout(a.status, kSiteLayerTail);
}

}  // namespace

// Weight bytes of the CTA holding the most, plus the activation slices of
// the widest phase, for `n_sm` CTAs and up to `max_rows` rows.
size_t chain_smem_bytes(const ChainArgs& a, int n_sm, int max_rows) {
  if (max_rows > kChainMaxRows || n_sm < 1) return 0;
  size_t wmax = 0;
  int umax = 0;
  for (int c = 0; c < n_sm; ++c) {
    size_t w = 0;
    int n = 0;
    for (int p = 0; p < a.n_phases; ++p) {
      const Geom q = geom_of(a.ph[p]);
      int u0, u1;
      unit_range(q.U, c, n_sm, u0, u1);
      w += (size_t)(u1 - u0) * q.ubytes;
      n += u1 - u0;
    }
    wmax = w > wmax ? w : wmax;
    umax = n > umax ? n : umax;
  }
  if (umax > kMaxUnits) return 0;
  size_t amax = 0;
  for (int p = 0; p < a.n_phases; ++p) {
    const Geom q = geom_of(a.ph[p]);
    if (q.klen % 64 != 0 || q.ft % 64 != 0 || (q.ft != 64 && q.ft != 128)) return 0;
    if (q.T > kChainMaxTiles || (q.U + n_sm - 1) / n_sm > q.T) return 0;  // a chunk spans at most two slices
    const int slices = (q.U + n_sm - 1) / n_sm > 1 ? 2 : 1;
    const size_t b = (size_t)slices * kChainMaxRows * (q.klen + x_pad<true>()) * 2;
    amax = b > amax ? b : amax;
  }
  return ((wmax + 127) & ~(size_t)127) + amax;
}

cudaError_t init_chain(size_t smem) {
  for (cudaError_t e : {cudaFuncSetAttribute(k_layer_tail<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem),
                        cudaFuncSetAttribute(k_layer_tail<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)})
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

// CTAs of the layer tail that fit on one SM with `smem` bytes (must be >= 1).
int chain_blocks_per_sm(ActType at, size_t smem) {
  int n = 0;
  const cudaError_t e = at == kBF16
                            ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_layer_tail<__nv_bfloat16>, kThreads, smem)
                            : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_layer_tail<__half>, kThreads, smem);
  return e == cudaSuccess ? n : 0;
}

void launch_layer_tail(ActType at, const ChainArgs& a, int n_sm, size_t smem, cudaStream_t s) {
  if (at == kBF16)
    launch_pdl(k_layer_tail<__nv_bfloat16>, dim3(n_sm), dim3(kThreads), smem, s, a);
  else
    launch_pdl(k_layer_tail<__half>, dim3(n_sm), dim3(kThreads), smem, s, a);
}

}  // namespace fmd
