// Decode-step projections: split-K GEMV with the K split reduced inside a
// thread-block cluster, and every epilogue and norm fused.
//
// A decode step multiplies ~32 token rows by each projection of a layer
// (crates/fmd-core/src/model/linear.rs:29-65; FusedLinear :85-95). The weights
// are read once per step, so the kernels are weight-streaming GEMVs whose
// cost is latency: this file removes the extra kernels a split-K needs.
//
//  * grid (N/FT feature tiles, S k-splits, row tiles); the S CTAs of one
//    feature tile form a cluster (S <= 8). Each computes a partial
//    FT x rows tile for its 1/S of K on mma.sync (weights Q8_0 dequantised in
//    registers, or dense), keeps it in its shared memory, and after
//    cluster.sync() CTA rank r sums the S partials of rows r, r+S, ... over
//    distributed shared memory and applies the epilogue to them. No global
//    partials, no atomics, a fixed summation order.
//  * each CTA's whole weight slice (FT rows x K/S, 8-74 KB) is requested at
//    kernel start with one TMA bulk copy per row into padded shared-memory
//    rows, before griddepcontrol.wait, so the weight stream overlaps the
//    previous kernel (programmatic dependent launch) and every byte a CTA
//    needs is in flight at once; the Q8_0 scales go to registers meanwhile.
//  * RMSNorm (linear.rs:293-302) is folded into the consumer: the epilogue
//    that updates the residual stream also writes, per row, the sum of squares
//    of its FT features (ssq[row][tile]); the next projection turns the row's
//    partial sums into rsqrt(mean + eps) and normalises its activation tile as
//    it lands in shared memory (xn = rnd(x * rs * w), as the reference does).
//
// Epilogues (the reference's rounding points):
//  * kGemvQkv    FT = 128 = one head: RMSNorm of q/k per head, RoPE at the
//                row's position, q -> q buffer, k/v -> paged KV cache
//                (qwen3.rs:213-227);
//  * kGemvResid  x <- rnd(x + rnd(y)) and ssq of the new x (qwen3.rs:333-338);
//  * kGemvSwiglu gate/up rows interleaved in 32-row groups at load, so a
//                64-row tile holds 32 matching gate and up features:
//                h = rnd(rnd(silu(rnd(g))) * rnd(u)) (qwen3.rs:288-292);
//  * kGemvLogits FT = 128, S = 2: rounded logits (qwen3.rs:459-463),
//                optionally stored as f32, and the tile's (max, lowest index)
//                per row.
#include <cooperative_groups.h>
#include <algorithm>
#include <type_traits>
#include <cstdlib>
#include <cstring>
#include <float.h>
#include <math.h>

#include "fmd_gemv.cuh"
#include "fmd_kernels.cuh"

namespace cg = cooperative_groups;

namespace fmd {

namespace {

constexpr int kRows = 64;   // rows per row tile (decode steps carry one row per sequence)
constexpr int kMaxKb = 16;  // 64-wide k-blocks per CTA (K / S <= 1024)
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr int kStatusNonFinite = -5;  // FMD_EIO: a greedy pick saw no finite logit

// KG warp groups split a CTA's k-blocks (KG = 2 only where the grid leaves
// SMs free: the doubled block would otherwise cost resident CTAs).
template <typename T, bool Q8, int FW, int EPI, bool NORM, int KG>
__global__ void __launch_bounds__(FW * KG * 32) k_gemv(const T* __restrict__ x, int ldx, const int* __restrict__ row_map,
                                                 const int* __restrict__ n_rows_ptr, LinW W, GemvEpi ep, int xrows,
                                                 int max_rows, int* __restrict__ status) {
  constexpr int NW = FW * KG;  // warps: FW feature slices x KG k-block groups
  constexpr int NT = NW * 32;
  constexpr int FT = FW * 16;
  constexpr int UNIT = Q8 ? kUnitQ8 : kUnitDense;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t wbar[kMaxKb];
  __shared__ float rs_s[kRows];
  __shared__ __align__(16) T nw_s[NORM ? kMaxKb * 64 : 8];  // the RMSNorm weights of this CTA's k-slice

  const int S = gridDim.y, rank = blockIdx.y;
  const int K = W.K;
  const int klen = K / S, kbeg = rank * klen, nkb = klen >> 6;
  const uint32_t kb_bytes = FW * UNIT;  // one k-block of the tile
  uint8_t* wsm = smem;                  // the CTA's weight tile
  T* xs = reinterpret_cast<T*>(smem + ((nkb * kb_bytes + 127) & ~127u));  // [xrows][klen + pad]
  const int xstride = klen + x_pad<Q8>();
  float* part = reinterpret_cast<float*>(xs);  // after the k-loop: [xrows][FT + 4]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int kgrp = warp / FW;     // this warp's k-blocks: kgrp, kgrp + KG, ...
  const int fl = (warp % FW) * 16 + g;  // local feature row of this thread (and fl + 8)

  // ---- the whole weight tile is in flight before the dependency wait: one
  // TMA bulk copy per k-block, each on its own mbarrier so compute can start
  // on the first k-block while the rest land
  if (threadIdx.x == 0) {
    const uint8_t* src = W.pk + (size_t)(blockIdx.x * S + rank) * nkb * kb_bytes;
    for (int kb = 0; kb < nkb; ++kb) mbar_init(&wbar[kb], 1);
    fence_barrier_init();
    for (int kb = 0; kb < nkb; ++kb) {
      mbar_arrive_expect_tx(&wbar[kb], kb_bytes);
      bulk_load(wsm + kb * kb_bytes, src + (size_t)kb * kb_bytes, kb_bytes, &wbar[kb]);
    }
  }
  // RMSNorm weights of this CTA's k-slice (constant: fetched before the wait,
  // off the path that starts when the activations arrive)
  if constexpr (NORM) {
    const int4* src = reinterpret_cast<const int4*>(reinterpret_cast<const T*>(ep.norm_w) + kbeg);
    for (int i = threadIdx.x; i < (klen >> 3); i += NT) reinterpret_cast<int4*>(nw_s)[i] = src[i];
  }
  // q/k RMSNorm weights of this CTA's head (constant: fetched before the wait)
  float hnw[4] = {1.f, 1.f, 1.f, 1.f};
  if constexpr (EPI == kGemvQkv) {
    if ((int)blockIdx.x < ep.Hq + ep.Hkv) {
      const T* nw = reinterpret_cast<const T*>((int)blockIdx.x < ep.Hq ? ep.qn_w : ep.kn_w) + lane * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) hnw[i] = Act<T>::to_f(nw[i]);
    }
  }
  // The row count, the plan's positions / slots / pages and the residual
  // rows come from kernels at least two launches back (the scheduler, the
  // embedding, an earlier projection), which are complete when this kernel
  // starts: every kernel signals its dependents only after its own
  // dependency wait. So they are read before the wait, off the path that
  // starts when the previous kernel's activations land.
  const int n_rows = *n_rows_ptr;
  const int row0 = blockIdx.z * kRows;
  const int cpr = klen >> 3;  // 16-byte chunks per activation row
  const int rows = max(0, min(min(kRows, xrows), n_rows - row0));
  const int n_tiles = (rows + 7) >> 3;

  // epilogue operands, in flight during the k-loop: the first kPre rows this warp will own
  // after the cluster reduction (lr = rank + warp * S + i * NW * S)
  constexpr int FPL = FT / 32;  // features per lane in the epilogue (2 or 4)
  constexpr int kPre = 2;
  float xpre[kPre][FPL];
  int ppos[kPre], pslot[kPre], ppage[kPre];
#pragma unroll
  for (int i = 0; i < kPre; ++i) {
    const int lr = rank + warp * S + i * NW * S;
    ppos[i] = pslot[i] = ppage[i] = 0;
#pragma unroll
    for (int f = 0; f < FPL; ++f) xpre[i][f] = 0.f;
    if (lr < rows) {
      const int r = row0 + lr;
      if constexpr (EPI == kGemvResid) {
        const T* xr = reinterpret_cast<const T*>(ep.x) + (size_t)r * W.N + blockIdx.x * FT + lane * FPL;
#pragma unroll
        for (int f = 0; f < FPL; ++f) xpre[i][f] = Act<T>::to_f(xr[f]);
      } else if constexpr (EPI == kGemvQkv) {
        ppos[i] = ep.plan.row_pos[r];
        pslot[i] = ep.plan.row_slot[r];
        if ((int)blockIdx.x >= ep.Hq)
          ppage[i] = ep.kv.page_table[(size_t)pslot[i] * ep.kv.max_pages_per_slot + ppos[i] / kPageTokens];
      }
    }
  }

  // RoPE factors of those rows (constant tables), in flight during the k-loop
  float rcs[kPre][4], rsn[kPre][4];
#pragma unroll
  for (int i = 0; i < kPre; ++i)
#pragma unroll
    for (int f = 0; f < 4; ++f) rcs[i][f] = rsn[i][f] = 0.f;
  if constexpr (EPI == kGemvQkv) {
    if ((int)blockIdx.x < ep.Hq + ep.Hkv) {
      const int dd = (lane & 15) * 4;
#pragma unroll
      for (int i = 0; i < kPre; ++i)
        if (rank + warp * S + i * NW * S < rows) {
          const T* ct = reinterpret_cast<const T*>(ep.cos) + (size_t)ppos[i] * (kHeadDim / 2) + dd;
          const T* st = reinterpret_cast<const T*>(ep.sin) + (size_t)ppos[i] * (kHeadDim / 2) + dd;
#pragma unroll
          for (int f = 0; f < 4; ++f) {
            rcs[i][f] = Act<T>::to_f(ct[f]);
            rsn[i][f] = Act<T>::to_f(st[f]);
          }
        }
    }
  }
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch

  if (rows > 0) {
    // activation tile rows x klen through the row map (rows of a partial
    // n-tile zero-filled)
    for (int c = threadIdx.x; c < n_tiles * 8 * cpr; c += NT) {
      const int r = c / cpr, ch = c - r * cpr;
      const T* src = x;
      int bytes = 0;
      if (r < rows) {
        src = x + (size_t)(row_map ? row_map[row0 + r] : row0 + r) * ldx + kbeg + ch * 8;
        bytes = 16;
      }
      cp_async16(xs + (size_t)r * xstride + ch * 8, src, bytes);
    }
    cp_async_commit();
  }
  if (rows > 0) {
    // rsqrt(mean(x^2) + eps) of each row, read while the activation tile is in flight
    if constexpr (NORM) rows_rsqrt(ep.ssq, ep.ssq_tiles, row_map, row0, rows, K, ep.eps, rs_s, NT);
    cp_async_wait<0>();
    if constexpr (NORM) {
      __syncthreads();  // rs_s, nw_s
      const T* nw = nw_s;
      for (int c = threadIdx.x; c < rows * cpr; c += NT) {
        const int r = c / cpr, ch = c - r * cpr;
        int4* p = reinterpret_cast<int4*>(xs + (size_t)r * xstride + ch * 8);
        int4 v = *p;
        const int4 wv = *reinterpret_cast<const int4*>(nw + ch * 8);
        uint32_t* u = reinterpret_cast<uint32_t*>(&v);
        const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv);
        const float rsr = rs_s[r];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = Act<T>::unpack2(u[j]);
          const float2 gw = Act<T>::unpack2(uw[j]);
          u[j] = Act<T>::pack2(f.x * rsr * gw.x, f.y * rsr * gw.y);
        }
        *p = v;
      }
    }
  }
  __syncthreads();  // barrier inits (and rs_s) visible to all threads
  if (rows == 0) {
    // a whole cluster shares blockIdx.z, so it leaves together, but only
    // after its copies into shared memory have landed
    cp_async_wait<0>();
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) ok &= mbar_wait_bounded(&wbar[kb], 0, kWaitLimit);
    if (!ok) report_timeout(status, kSiteGemv);
    return;
  }

  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  bool ok = true;
  // not unrolled: the k-loop body is ~100 instructions, and a decode layer
  // cycles through four GEMV variants, so code size shows up as i-cache misses
#pragma unroll 1
  for (int kb = kgrp; kb < nkb; kb += KG) {
    {
      const bool landed = mbar_wait_bounded(&wbar[kb], 0, kWaitLimit);
      ok &= landed;
      if (landed) {
        const uint8_t* u = wsm + kb * kb_bytes + (warp % FW) * UNIT;
        WRegs w;
        gemv_wload<Q8>(u, lane, w);
        uint32_t af[4][4];
        gemv_afrag<T, Q8>(w, af);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          if (nt < n_tiles) {
            uint32_t xw[8];
            gemv_xfrag<T, Q8>(xs + (size_t)(nt * 8 + g) * xstride + kb * 64, t, xw);
            gemv_kblock<T, Q8>(acc[nt], af, xw, w);
          }
        }
      }
    }
  }
  if (!ok) report_timeout(status, kSiteGemv);
  __syncthreads();  // the activation tile is dead: `part` reuses it

  // ---- partial tile -> shared memory (k-block group 1, then group 0 adds
  // its own: a fixed order); the cluster sums the CTAs' tiles
  constexpr int PS = FT + 4;  // part row stride (floats)
  static_assert(KG == 1 || KG == 2, "one or two k-block groups");
  if (kgrp == KG - 1) {
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      if (nt < n_tiles) {
        const int lr = nt * 8 + 2 * t;
        part[lr * PS + fl] = acc[nt][0];
        part[(lr + 1) * PS + fl] = acc[nt][1];
        part[lr * PS + fl + 8] = acc[nt][2];
        part[(lr + 1) * PS + fl + 8] = acc[nt][3];
      }
    }
  }
  if (KG == 2) __syncthreads();
  if (KG == 2 && kgrp == 0) {
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      if (nt < n_tiles) {
        const int lr = nt * 8 + 2 * t;
        part[lr * PS + fl] = acc[nt][0] + part[lr * PS + fl];
        part[(lr + 1) * PS + fl] = acc[nt][1] + part[(lr + 1) * PS + fl];
        part[lr * PS + fl + 8] = acc[nt][2] + part[lr * PS + fl + 8];
        part[(lr + 1) * PS + fl + 8] = acc[nt][3] + part[(lr + 1) * PS + fl + 8];
      }
    }
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();

  // rank r owns rows r, r+S, ...; one warp per row, features across lanes
  int pi = 0;  // index of this row among the warp's rows
  for (int lr = rank + warp * S; lr < rows; lr += NW * S, ++pi) {
    float v[FPL];
#pragma unroll
    for (int i = 0; i < FPL; ++i) v[i] = 0.f;
    // the S peer loads issue together (fixed summation order s = 0 .. S-1)
    float pv[8][FPL];
#pragma unroll
    for (int s = 0; s < 8; ++s)
      if (s < S) {
        // one vector load per peer: a warp reads the row's FT floats contiguously
        const float* peer = cluster.map_shared_rank(part + lr * PS, s) + lane * FPL;
        if constexpr (FPL == 4) {
          const float4 q = *reinterpret_cast<const float4*>(peer);
          pv[s][0] = q.x;
          pv[s][1] = q.y;
          pv[s][2] = q.z;
          pv[s][3] = q.w;
        } else {
          const float2 q = *reinterpret_cast<const float2*>(peer);
          pv[s][0] = q.x;
          pv[s][1] = q.y;
        }
      }
#pragma unroll
    for (int s = 0; s < 8; ++s)
      if (s < S)
#pragma unroll
        for (int i = 0; i < FPL; ++i) v[i] += pv[s][i];
    const int r = row0 + lr;
#pragma unroll
    for (int i = 0; i < FPL; ++i) v[i] = rnd<T>(v[i]);

    if constexpr (EPI == kGemvResid) {
      T* xr = reinterpret_cast<T*>(ep.x) + (size_t)r * W.N + blockIdx.x * FT + lane * FPL;
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < FPL; ++i) {
        const float xo = pi < kPre ? (pi == 0 ? xpre[0][i] : xpre[1][i]) : Act<T>::to_f(xr[i]);
        const float nx = rnd<T>(xo + v[i]);
        xr[i] = Act<T>::from_f(nx);
        ss += nx * nx;
      }
      ss = warp_sum(ss);
      if (lane == 0) ep.ssq_out[(size_t)r * ep.ssq_tiles + blockIdx.x] = ss;
    } else if constexpr (EPI == kGemvSwiglu) {
      // FT = 64: features [0, 32) gate, [32, 64) up of intermediate index
      // tile*32 + j; lane l holds features 2l, 2l+1
      const float g0 = __shfl_sync(0xffffffffu, v[0], lane >> 1), g1 = __shfl_sync(0xffffffffu, v[1], lane >> 1);
      const float u0 = __shfl_sync(0xffffffffu, v[0], 16 + (lane >> 1));
      const float u1 = __shfl_sync(0xffffffffu, v[1], 16 + (lane >> 1));
      const float gv = (lane & 1) ? g1 : g0, uv = (lane & 1) ? u1 : u0;
      const float sg = rnd<T>(gv / (1.f + expf(-gv)));
      reinterpret_cast<T*>(ep.h)[(size_t)r * ep.I + blockIdx.x * 32 + lane] = Act<T>::from_f(sg * uv);
    } else if constexpr (EPI == kGemvQkv) {
      // FT = 128: one head; lane holds dims 4*lane .. 4*lane+3
      const int hh = blockIdx.x, Hq = ep.Hq, Hkv = ep.Hkv;
      const int pos = pi < kPre ? (pi == 0 ? ppos[0] : ppos[1]) : ep.plan.row_pos[r];
      const int slot = pi < kPre ? (pi == 0 ? pslot[0] : pslot[1]) : ep.plan.row_slot[r];
      const int kvpage = pi < kPre ? (pi == 0 ? ppage[0] : ppage[1])
                                   : (hh >= Hq ? ep.kv.page_table[(size_t)slot * ep.kv.max_pages_per_slot +
                                                                  pos / kPageTokens]
                                               : 0);
      T* kvb = reinterpret_cast<T*>(ep.kv.base);
      T* dst;
      if (hh < Hq + Hkv) {
        const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
        const float inv = rsqrtf(ss / kHeadDim + ep.eps);
        float y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) y[i] = rnd<T>(v[i] * inv * hnw[i]);
        const T* cos_t = reinterpret_cast<const T*>(ep.cos);
        const T* sin_t = reinterpret_cast<const T*>(ep.sin);
        const int dd = (lane & 15) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float pr = __shfl_xor_sync(0xffffffffu, y[i], 16);
          const float cs = pi < kPre ? (pi == 0 ? rcs[0][i] : rcs[1][i])
                                     : Act<T>::to_f(cos_t[(size_t)pos * (kHeadDim / 2) + dd + i]);
          const float sn = pi < kPre ? (pi == 0 ? rsn[0][i] : rsn[1][i])
                                     : Act<T>::to_f(sin_t[(size_t)pos * (kHeadDim / 2) + dd + i]);
          v[i] = lane < 16 ? y[i] * cs - pr * sn : pr * sn + y[i] * cs;
        }
        if (hh < Hq) {
          dst = reinterpret_cast<T*>(ep.q_out) + (size_t)r * Hq * kHeadDim + hh * kHeadDim;
        } else {
          dst = kvb + ep.kv.elem_offset(ep.layer, kvpage, 0, hh - Hq) + (size_t)(pos % kPageTokens) * kHeadDim;
        }
      } else {
        dst = kvb + ep.kv.elem_offset(ep.layer, kvpage, 1, hh - Hq - Hkv) + (size_t)(pos % kPageTokens) * kHeadDim;
      }
      uint2 o;
      o.x = Act<T>::pack2(v[0], v[1]);
      o.y = Act<T>::pack2(v[2], v[3]);
      *reinterpret_cast<uint2*>(dst + lane * 4) = o;
    } else {  // kGemvLogits: rounded logits and the tile's best per row
      const int fb = blockIdx.x * FT + lane * FPL;
      if (ep.logits) {
#pragma unroll
        for (int i = 0; i < FPL; ++i) ep.logits[(size_t)r * W.N + fb + i] = v[i];
      }
      float best = v[0];
      int bi = fb;
#pragma unroll
      for (int i = 1; i < FPL; ++i)
        if (v[i] > best) {
          best = v[i];
          bi = fb + i;
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
          best = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        ep.best_val[(size_t)r * gridDim.x + blockIdx.x] = best;
        ep.best_idx[(size_t)r * gridDim.x + blockIdx.x] = bi;
      }
    }
  }
  // peers may still be reading this CTA's partial tile: wait for every CTA of
  // the cluster to pass its reduction (a relaxed arrive: the epilogue's
  // global stores need not be performed first)
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
}

// lm_head + greedy candidates as one persistent kernel (qwen3.rs:459-463,
// engine.rs:550-559). The final RMSNorm is applied to the staged rows from
// the per-tile sums of squares (ep.ssq), or skipped when ep.ssq is null and
// the rows are already normalised. The vocabulary projection is the largest
// weight of a decode step (vocab x hidden) and the only one with more
// 128-feature tiles than there are SMs, so here one CTA per SM keeps the
// normalised activation tile resident and streams its share of tiles through
// a ring of TMA bulk copies (one stage = one 64-wide k-block of a tile, 8.5 KB
// for Q8_0):
//  * the last warp (one lane) is the producer; the others consume in G groups
//    of eight, each warp owning 16 features of a 128-feature tile. Group g
//    takes the CTA's tiles g, g + G, ...; the producer interleaves the
//    k-blocks of G tiles, so the groups stream at once. The register-level
//    Q8_0 dequantisation makes this instruction-bound, hence two groups
//    where the registers allow (batches up to 32 rows).
//  * each group owns its own ring of S/G stages: the q-th unit (k-block) of
//    group g uses stage g * S/G + q mod S/G in phase q / (S/G). A stage is
//    therefore only ever filled for, and released by, one group, so a
//    group's parity wait can only match its own copy, whatever order the
//    copies land in and however far one group runs ahead (a ring shared by
//    the groups lets a group pass a wait on the other group's phase).
//  * a warp releases a stage by arriving on its "empty" barrier. Every wait
//    is bounded; a timeout stops the ring, sets the status word and drains
//    the copies still in flight.
//  * the tile order of the packed lm_head ([tile][k-split][k-block][warp]) is
//    the full-K k-block order of each tile.
//  * each CTA keeps, per row, the best (rounded logit, lowest index) over its
//    tiles and writes one candidate per (row, CTA); k_pick_reduce finishes.
constexpr int kHeadWarps = 8;            // warps per group: 128 features per tile
constexpr int kHeadMaxStages = 16;
constexpr int kHeadSmemBudget = 220 * 1024;

// Stage and phase of a group's ring, advanced one unit at a time.
struct RingPos {
  int st, ph;
  FMD_DEV void next(int sg) {
    if (++st == sg) {
      st = 0;
      ph ^= 1;
    }
  }
};

// NTL: MMA n-tiles (8 rows each) of a row tile; G: consumer groups. Two
// groups (17 warps) leave 96 registers per thread, enough for 4 n-tiles.
// F16 (Q8_0 weights, bf16 rows): the MMAs take f16 operands. The exact int8
// -> f16 conversion is 5 instructions per 4 weights against 11 for bf16, and
// the register dequantisation is what bounds this kernel. Each staged row,
// already rounded to bf16, is scaled by 2^(14 - e) (e the exponent of its
// largest |value|) and converted to f16: exact for every value above 2^-17
// after scaling (bf16 keeps 8 significant bits, f16 11, normal from 2^-14),
// i.e. all but values 2^-31 below the row's largest, whose products sit
// under the f32 sum's own rounding. The logits are scaled back by the exact
// power of two before the rounding to bf16.
template <typename T, bool Q8, int NTL, int G, bool F16>
__global__ void __launch_bounds__((G * kHeadWarps + 1) * 32, 1)
    k_lm_head(const T* __restrict__ x, int ldx, const int* __restrict__ row_map, const int* __restrict__ n_rows_ptr,
              LinW W, GemvEpi ep, int xrows, int stages, int* __restrict__ status) {
  static_assert(!F16 || (Q8 && Act<T>::kIsBf16), "f16 operands serve Q8_0 weights with bf16 rows");
  using M = typename std::conditional<F16, __half, T>::type;  // MMA operand type
  constexpr int UNIT = Q8 ? kUnitQ8 : kUnitDense;
  constexpr uint32_t kStage = kHeadWarps * UNIT;
  constexpr int FT = kHeadWarps * 16;
  constexpr int NCW = G * kHeadWarps;  // consumer warps
  constexpr int NT = NCW * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kHeadMaxStages], empty[kHeadMaxStages];
  __shared__ float rs_s[kRows];
  __shared__ uint32_t xmax_s[F16 ? NTL * 8 : 1];  // F16: largest |value| of each staged row (f32 bits)
  __shared__ float inv_s[F16 ? NTL * 8 : 1];      // F16: 1 / the row's operand scale
  __shared__ float cand_v[NCW][NTL * 8];
  __shared__ int cand_i[NCW][NTL * 8];
  __shared__ int abort_s;

  const int K = W.K, nkb = K / 64;
  const int n_tiles = W.N / FT;
  const int my_tiles = n_tiles > (int)blockIdx.x ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  uint8_t* ring = smem;
  T* xs = reinterpret_cast<T*>(smem + (size_t)stages * kStage);  // [xrows][K + pad]
  const int xstride = K + x_pad<Q8>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int grp = warp / kHeadWarps, fw = warp % kHeadWarps;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kHeadWarps);  // one group consumes each stage
    }
    abort_s = 0;
    fence_barrier_init();
  }
  __syncthreads();

  const int SG = stages / G;  // stages per group
  if (warp == NCW) {
    // ---- producer: weights do not depend on the previous kernel, so the
    // ring starts filling before griddepcontrol.wait
    if (lane == 0) {
      RingPos pos[G];
      int q[G];
#pragma unroll
      for (int j = 0; j < G; ++j) pos[j] = RingPos{0, 0}, q[j] = 0;
      for (int p = 0; G * p < my_tiles; ++p) {
        const int in_grp = min(G, my_tiles - G * p);
        for (int kb = 0; kb < nkb; ++kb) {
#pragma unroll
          for (int j = 0; j < G; ++j) {
            if (j >= in_grp) continue;
            const int st = j * SG + pos[j].st;
            // the stage's previous use (unit q - SG of this group) must be released
            if (q[j] >= SG && !mbar_wait_bounded(&empty[st], pos[j].ph ^ 1, kWaitLimit)) {
              atomicExch(&abort_s, 1);
              goto produced;
            }
            if (*reinterpret_cast<volatile int*>(&abort_s)) goto produced;
            const int tile = blockIdx.x + (G * p + j) * gridDim.x;
            mbar_arrive_expect_tx(&full[st], kStage);
            bulk_load(ring + (size_t)st * kStage, W.pk + ((size_t)tile * nkb + kb) * kStage, kStage, &full[st]);
            pos[j].next(SG);
            ++q[j];
          }
        }
      }
    produced:;
    }
    griddep_wait();
    griddep_launch();  // only after the wait: see griddep_launch
    return;  // nothing below touches the producer warp
  }

  // ---- consumers (512 threads): normalised activation tile, then the ring
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch
  const int n_rows = *n_rows_ptr;
  const int row0 = blockIdx.y * NTL * 8;
  const int rows = max(0, min(min(NTL * 8, xrows), n_rows - row0));
  const int n_nt = (rows + 7) >> 3;
  const int cpr = K >> 3;
  for (int c = threadIdx.x; c < n_nt * 8 * cpr; c += NT) {
    const int r = c / cpr, ch = c - r * cpr;
    const T* src = x;
    int bytes = 0;
    if (r < rows) {
      src = x + (size_t)(row_map ? row_map[row0 + r] : row0 + r) * ldx + ch * 8;
      bytes = 16;
    }
    cp_async16(xs + (size_t)r * xstride + ch * 8, src, bytes);
  }
  cp_async_commit();
  const bool norm = ep.ssq != nullptr;  // else x is already normalised
  if (norm) rows_rsqrt(ep.ssq, ep.ssq_tiles, row_map, row0, rows, K, ep.eps, rs_s, NT);
  if constexpr (F16)
    for (int r = threadIdx.x; r < NTL * 8; r += NT) xmax_s[r] = 0u;
  cp_async_wait<0>();
  named_sync(1, NT);
  if (norm || F16) {
    const T* nw = reinterpret_cast<const T*>(ep.norm_w);
    for (int c = threadIdx.x; c < rows * cpr; c += NT) {
      const int r = c / cpr, ch = c - r * cpr;
      int4* p = reinterpret_cast<int4*>(xs + (size_t)r * xstride + ch * 8);
      int4 v = *p;
      uint32_t* u = reinterpret_cast<uint32_t*>(&v);
      if (norm) {
        const int4 wv = *reinterpret_cast<const int4*>(nw + ch * 8);
        const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv);
        const float rsr = rs_s[r];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = Act<T>::unpack2(u[j]);
          const float2 gw = Act<T>::unpack2(uw[j]);
          u[j] = Act<T>::pack2(f.x * rsr * gw.x, f.y * rsr * gw.y);
        }
        *p = v;
      }
      if constexpr (F16) {
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = Act<T>::unpack2(u[j]);
          m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
        if (m > 0.f) atomicMax(&xmax_s[r], __float_as_uint(m));
      }
    }
  }
  named_sync(1, NT);
  if constexpr (F16) {
    // the operand scale 2^sh of each row and its exact inverse; the padding
    // rows (all zero) keep 1
    for (int r = threadIdx.x; r < NTL * 8; r += NT) {
      const uint32_t mb = xmax_s[r];
      const int e = (int)((mb >> 23) & 0xffu) - 127;
      const int sh = mb == 0u || e > 127 ? 0 : max(-126, min(126, 14 - e));
      inv_s[r] = __uint_as_float((uint32_t)(127 - sh) << 23);
      rs_s[r] = __uint_as_float((uint32_t)(127 + sh) << 23);  // the norm's row scales are dead: reuse
    }
    named_sync(1, NT);
    for (int c = threadIdx.x; c < rows * cpr; c += NT) {
      const int r = c / cpr, ch = c - r * cpr;
      int4* p = reinterpret_cast<int4*>(xs + (size_t)r * xstride + ch * 8);
      int4 v = *p;
      uint32_t* u = reinterpret_cast<uint32_t*>(&v);
      const float sc = rs_s[r];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Act<T>::unpack2(u[j]);
        u[j] = Act<__half>::pack2(f.x * sc, f.y * sc);
      }
      *p = v;
    }
    named_sync(1, NT);
  }
  const M* xm = reinterpret_cast<const M*>(xs);

  // running best of this thread's rows (nt * 8 + 2t + {0, 1}) over its features
  float bv[NTL][2];
  int bi[NTL][2];
#pragma unroll
  for (int nt = 0; nt < NTL; ++nt) {
    bv[nt][0] = bv[nt][1] = -INFINITY;
    bi[nt][0] = bi[nt][1] = 0x7fffffff;
  }
  bool ok = true;
  RingPos rp{0, 0};  // this group's ring position
  if (rows == 0) {
    // the producer started before the row count was known: release every
    // stage of this group's tiles so that no copy is left in flight when the
    // CTA retires
    for (int i = grp; i < my_tiles && ok; i += G)
      for (int kb = 0; kb < nkb; ++kb) {
        const int st = grp * SG + rp.st;
        if (*reinterpret_cast<volatile int*>(&abort_s) || !mbar_wait_bounded(&full[st], rp.ph, kWaitLimit)) {
          atomicExch(&abort_s, 1);
          ok = false;
          break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        rp.next(SG);
      }
  }
  for (int i = grp; i < my_tiles && ok && rows > 0; i += G) {
    const int tile = blockIdx.x + i * gridDim.x;
    float acc[NTL][4];
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll 1
    for (int kb = 0; kb < nkb; ++kb) {
      const int st = grp * SG + rp.st;
      if (*reinterpret_cast<volatile int*>(&abort_s) || !mbar_wait_bounded(&full[st], rp.ph, kWaitLimit)) {
        atomicExch(&abort_s, 1);
        ok = false;
        break;
      }
      rp.next(SG);
      const uint8_t* un = ring + (size_t)st * kStage + fw * UNIT;
      WRegs w;
      gemv_wload<Q8>(un, lane, w);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);  // this warp's fragments are in registers
      uint32_t af[4][4];
      gemv_afrag<M, Q8>(w, af);
#pragma unroll
      for (int nt = 0; nt < NTL; ++nt) {
        if (nt < n_nt) {
          uint32_t xw[8];
          gemv_xfrag<M, Q8>(xm + (size_t)(nt * 8 + g) * xstride + kb * 64, t, xw);
          gemv_kblock<M, Q8>(acc[nt], af, xw, w);
        }
      }
    }
    if (!ok) break;
    // rounded logits (the reference rounds lm_head output to the activation
    // type) and the running best; features fl and fl + 8 of this tile
    const int f0 = tile * FT + fw * 16 + g;
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt) {
      if (nt < n_nt) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int lr = nt * 8 + 2 * t + h;
          const float is = F16 ? inv_s[lr] : 1.f;
          const float va = rnd<T>(acc[nt][h] * is), vb = rnd<T>(acc[nt][2 + h] * is);
          if (ep.logits && lr < rows) {
            float* lg = ep.logits + (size_t)(row0 + lr) * W.N;
            lg[f0] = va;
            lg[f0 + 8] = vb;
          }
          if (va > bv[nt][h] || (va == bv[nt][h] && f0 < bi[nt][h])) {
            bv[nt][h] = va;
            bi[nt][h] = f0;
          }
          if (vb > bv[nt][h] || (vb == bv[nt][h] && f0 + 8 < bi[nt][h])) {
            bv[nt][h] = vb;
            bi[nt][h] = f0 + 8;
          }
        }
      }
    }
  }
  if (!ok && threadIdx.x == 0) report_timeout(status, kSiteLmHead);

  // ---- per-row best over this CTA's tiles: lanes of equal t, then warps
#pragma unroll
  for (int nt = 0; nt < NTL; ++nt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float v = bv[nt][h];
      int ix = bi[nt][h];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
        if (ov > v || (ov == v && oi < ix)) {
          v = ov;
          ix = oi;
        }
      }
      if (g == 0) {
        cand_v[warp][nt * 8 + 2 * t + h] = v;
        cand_i[warp][nt * 8 + 2 * t + h] = ix;
      }
    }
  }
  named_sync(1, NT);
  for (int r = threadIdx.x; r < rows; r += NT) {
    float v = cand_v[0][r];
    int ix = cand_i[0][r];
    for (int w = 1; w < NCW; ++w)
      if (cand_v[w][r] > v || (cand_v[w][r] == v && cand_i[w][r] < ix)) {
        v = cand_v[w][r];
        ix = cand_i[w][r];
      }
    ep.best_val[(size_t)(row0 + r) * gridDim.x + blockIdx.x] = v;
    ep.best_idx[(size_t)(row0 + r) * gridDim.x + blockIdx.x] = ix;
  }

  // drain: a copy still in flight must land before the CTA's shared memory
  // is released (only after an abort can one be outstanding here)
  if (threadIdx.x == 0 && *reinterpret_cast<volatile int*>(&abort_s)) {
    for (int j = 0; j < G; ++j) {
      const int n_j = (my_tiles > j ? (my_tiles - j + G - 1) / G : 0) * nkb;  // units of group j
      for (int sl = 0; sl < SG && sl < n_j; ++sl) {
        // the last use of the group's stage sl is its unit qlast
        const int qlast = sl + ((n_j - 1 - sl) / SG) * SG;
        mbar_wait_bounded(&full[j * SG + sl], (qlast / SG) & 1, kWaitLimit);
      }
    }
  }
}

// Greedy pick (engine.rs:550-559): max over the per-tile candidates of a row,
// lowest vocabulary index among equal maxima.
__global__ void __launch_bounds__(256) k_pick_reduce(const int* __restrict__ n_sample_ptr,
                                                     const float* __restrict__ best_val,
                                                     const int* __restrict__ best_idx, int n_parts,
                                                     int* __restrict__ next_ids, int vocab,
                                                     int* __restrict__ status) {
  __shared__ float sv[8];
  __shared__ int si[8];
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch
  const int n = *n_sample_ptr;
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n_parts; i += blockDim.x) {
      const float v = best_val[(size_t)r * n_parts + i];
      const int ix = best_idx[(size_t)r * n_parts + i];
      if (v > best || (v == best && ix < bi)) {
        best = v;
        bi = ix;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
      sv[warp] = best;
      si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < 8; ++w)
        if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
          best = sv[w];
          bi = si[w];
        }
      // no finite logit in the row (all candidates NaN): report it instead of
      // handing an index outside the vocabulary to the next step
      if (bi < 0 || bi >= vocab) {
        bi = 0;
        atomicExch(status, kStatusNonFinite);
      }
      next_ids[r] = bi;
    }
    __syncthreads();
  }
}

size_t gemv_smem_bytes(int FT, bool q8, int klen, int xrows) {
  const size_t w = ((size_t)(klen / 64) * (FT / 16) * (q8 ? kUnitQ8 : kUnitDense) + 127) & ~(size_t)127;
  const size_t xb = (size_t)xrows * (klen + (q8 ? x_pad<true>() : x_pad<false>())) * 2;
  const size_t pb = (size_t)xrows * (FT + 4) * 4;
  return w + (xb > pb ? xb : pb);
}

template <typename T, bool Q8, int FW, int EPI, bool NORM, int KG>
void launch_gemv_t(const LinW& W, int S, const void* x, int ldx, const int* row_map, const int* n_rows_ptr,
                   int max_rows, const GemvEpi& ep, int* status, cudaStream_t s) {
  const int xrows = ((max_rows < kRows ? max_rows : kRows) + 7) & ~7;
  const size_t smem = gemv_smem_bytes(FW * 16, Q8, W.K / S, xrows);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = S;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(W.N / (FW * 16), S, (max_rows + kRows - 1) / kRows);
  cfg.blockDim = dim3(FW * KG * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, k_gemv<T, Q8, FW, EPI, NORM, KG>, (const T*)x, ldx, row_map, n_rows_ptr, W, ep, xrows,
                     max_rows, status);
}


template <typename T, bool Q8, int NTL, int G, bool F16>
int launch_lm_head_t(const LinW& W, const void* x, int ldx, const int* row_map, const int* n_rows_ptr,
                     int max_rows, const GemvEpi& ep, int* status, cudaStream_t s) {
  static int n_sm = 0;
  if (n_sm == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (n_sm <= 0) n_sm = 148;
  }
  constexpr int kTileRows = NTL * 8;
  const int xrows = ((max_rows < kTileRows ? max_rows : kTileRows) + 7) & ~7;
  const size_t xbytes = (size_t)xrows * (W.K + x_pad<Q8>()) * sizeof(T);
  const size_t stage = (size_t)kHeadWarps * (Q8 ? kUnitQ8 : kUnitDense);
  if (xbytes + 2 * stage > (size_t)kHeadSmemBudget) return 0;
  int stages = (int)((kHeadSmemBudget - xbytes) / stage);
  if (stages > kHeadMaxStages) stages = kHeadMaxStages;
  // each of the G groups owns stages / G of the stages (its own ring)
  stages -= stages % G;
  const int n_tiles = W.N / (kHeadWarps * 16);
  const int grid = n_tiles < n_sm ? n_tiles : n_sm;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, (max_rows + kTileRows - 1) / kTileRows, 1);
  cfg.blockDim = dim3((G * kHeadWarps + 1) * 32);
  cfg.dynamicSmemBytes = (size_t)stages * stage + xbytes;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k_lm_head<T, Q8, NTL, G, F16>, (const T*)x, ldx, row_map, n_rows_ptr, W, ep, xrows, stages,
                     status);
  return grid;
}

template <typename T, bool Q8>
cudaError_t init_gemv_t() {
  cudaError_t e = cudaSuccess;
  const int lim = 220 * 1024;  // opt-in limit less room for the static barriers, row scales and norm weights
  for (cudaError_t r : {
           cudaFuncSetAttribute(k_gemv<T, Q8, 8, kGemvQkv, true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim),
           cudaFuncSetAttribute(k_gemv<T, Q8, 8, kGemvQkv, false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim),
           cudaFuncSetAttribute(k_gemv<T, Q8, 4, kGemvResid, false, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim),
           cudaFuncSetAttribute(k_gemv<T, Q8, 4, kGemvSwiglu, true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim),
           cudaFuncSetAttribute(k_gemv<T, Q8, 8, kGemvLogits, true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, lim),
           cudaFuncSetAttribute(k_lm_head<T, Q8, 4, 2, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kHeadSmemBudget),
           cudaFuncSetAttribute(k_lm_head<T, Q8, 8, 1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kHeadSmemBudget)})
    if (r != cudaSuccess) e = r;
  if constexpr (Q8 && Act<T>::kIsBf16)
    for (cudaError_t r : {cudaFuncSetAttribute(k_lm_head<T, Q8, 4, 2, true>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kHeadSmemBudget),
                          cudaFuncSetAttribute(k_lm_head<T, Q8, 8, 1, true>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kHeadSmemBudget)})
      if (r != cudaSuccess) e = r;
  return e;
}

}  // namespace

cudaError_t init_gemv() {
  for (cudaError_t e : {init_gemv_t<__nv_bfloat16, true>(), init_gemv_t<__nv_bfloat16, false>(),
                        init_gemv_t<__half, true>(), init_gemv_t<__half, false>()})
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}


int gemv_tile_features(int epi) { return (epi == kGemvQkv || epi == kGemvLogits) ? 128 : 64; }

// K split of one projection: the widest cluster (<= 8, portable; a smaller
// cap from FMD_GEMV_SPLIT in the environment, read once, for measurements)
// whose slices are whole 64-wide k-blocks, but for lm_head only 2, since its
// activation tile is re-read by each of the vocab/128 feature tiles. 0 if no
// split keeps a slice within kMaxKb k-blocks.
int gemv_split(int epi, int K) {
  static const int cap = [] {
    const char* v = std::getenv("FMD_GEMV_SPLIT");
    const int c = v ? std::atoi(v) : 8;
    return c == 1 || c == 2 || c == 4 ? c : 8;
  }();
  for (int s = epi == kGemvLogits ? std::min(2, cap) : cap; s >= 1; s >>= 1)
    if (K % (64 * s) == 0 && K / s <= 64 * kMaxKb) return s;
  return 0;
}

size_t gemv_packed_bytes(int epi, int N, int K, bool q8) {
  return (size_t)(N / 16) * (K / 64) * (q8 ? kUnitQ8 : kUnitDense);
}

// Tile (feature tile f, k-split s) is the contiguous range
// [(f * S + s) * nkb * FW * UNIT, +nkb * FW * UNIT), k-block major.
void gemv_pack(int epi, int N, int K, bool q8, const int8_t* qs, const uint16_t* d, const uint16_t* w,
               uint8_t* out) {
  const int FT = gemv_tile_features(epi), FW = FT / 16, S = gemv_split(epi, K);
  const int klen = K / S, nkb = klen / 64, KB = K / kQ8Block;
  const int unit = q8 ? kUnitQ8 : kUnitDense;
  for (int f = 0; f < N / FT; ++f)
    for (int s = 0; s < S; ++s)
      for (int kb = 0; kb < nkb; ++kb)
        for (int wp = 0; wp < FW; ++wp) {
          uint8_t* u = out + ((((size_t)f * S + s) * nkb + kb) * FW + wp) * unit;
          const int r0 = f * FT + wp * 16, k0 = s * klen + kb * 64;
          for (int lane = 0; lane < 32; ++lane) {
            const int g = lane >> 2, t = lane & 3;
            const size_t a = (size_t)(r0 + g) * K + k0 + 16 * t, b = a + (size_t)8 * K;
            if (q8) {
              // k [8t, 8t + 8) of block 0, then k [32 + 8t, 32 + 8t + 8) of block 1
              const size_t qa = (size_t)(r0 + g) * K + k0 + 8 * t, qb = qa + (size_t)8 * K;
              std::memcpy(u + lane * 16, qs + qa, 8);
              std::memcpy(u + lane * 16 + 8, qs + qa + 32, 8);
              std::memcpy(u + 512 + lane * 16, qs + qb, 8);
              std::memcpy(u + 512 + lane * 16 + 8, qs + qb + 32, 8);
            } else {
              std::memcpy(u + lane * 16, w + a, 16);
              std::memcpy(u + 512 + lane * 16, w + a + 8, 16);
              std::memcpy(u + 1024 + lane * 16, w + b, 16);
              std::memcpy(u + 1536 + lane * 16, w + b + 8, 16);
            }
          }
          if (q8) {
            uint16_t* sc = reinterpret_cast<uint16_t*>(u + 1024);
            for (int j = 0; j < 32; ++j) sc[j] = d[(size_t)(r0 + (j >> 1)) * KB + k0 / kQ8Block + (j & 1)];
          }
        }
}

bool launch_gemv(ActType at, int epi, bool norm, const LinW& W, const void* x, int ldx, const int* row_map,
                 const int* n_rows_ptr, int max_rows, const GemvEpi& ep, int* status, cudaStream_t s) {
  const int S = gemv_split(epi, W.K);
  if (S == 0 || W.pk == nullptr || W.N % gemv_tile_features(epi) != 0) return false;
#define FMD_GEMV(T, Q8)                                                                                           \
  switch (epi) {                                                                                                \
    case kGemvQkv:                                                                                              \
      if (norm) launch_gemv_t<T, Q8, 8, kGemvQkv, true, 1>(W, S, x, ldx, row_map, n_rows_ptr, max_rows, ep, status, s);     \
      else launch_gemv_t<T, Q8, 8, kGemvQkv, false, 1>(W, S, x, ldx, row_map, n_rows_ptr, max_rows, ep, status, s);         \
      break;                                                                                                    \
    case kGemvResid: launch_gemv_t<T, Q8, 4, kGemvResid, false, 2>(W, S, x, ldx, row_map, n_rows_ptr, max_rows, ep, status, s); break; \
    case kGemvSwiglu: launch_gemv_t<T, Q8, 4, kGemvSwiglu, true, 1>(W, S, x, ldx, row_map, n_rows_ptr, max_rows, ep, status, s); break; \
    default: launch_gemv_t<T, Q8, 8, kGemvLogits, true, 1>(W, S, x, ldx, row_map, n_rows_ptr, max_rows, ep, status, s); break; \
  }
  if (at == kBF16) {
    if (W.q8) { FMD_GEMV(__nv_bfloat16, true) } else { FMD_GEMV(__nv_bfloat16, false) }
  } else {
    if (W.q8) { FMD_GEMV(__half, true) } else { FMD_GEMV(__half, false) }
  }
#undef FMD_GEMV
  return true;
}

int launch_lm_head(ActType at, const LinW& W, const void* x, int ldx, const int* row_map, const int* n_rows_ptr,
                   int max_rows, const GemvEpi& ep, int* status, cudaStream_t s, bool tc, bool f16ops,
                   bool* used_tc) {
  if (used_tc) *used_tc = false;
  if (W.pk == nullptr || W.N % (kHeadWarps * 16) != 0 || W.K % 64 != 0) return 0;
  int parts = tc ? launch_lm_head_tc(at, W, x, ldx, row_map, n_rows_ptr, max_rows, ep, status, s) : 0;
  if (parts > 0) {
    if (used_tc) *used_tc = true;
    return parts;
  }
  // row tiles of 32 rows (4 MMA n-tiles) up to a batch of 32, else 64
  // (Q8_0 with bf16 rows: f16 operands unless f16ops is off)
#define FMD_HEAD(T, Q8, F16)                                                                                      \
  (max_rows <= 32 ? launch_lm_head_t<T, Q8, 4, 2, F16>(W, x, ldx, row_map, n_rows_ptr, max_rows, ep, status, s) \
                  : launch_lm_head_t<T, Q8, 8, 1, F16>(W, x, ldx, row_map, n_rows_ptr, max_rows, ep, status, s))
  if (at == kBF16)
    parts = !W.q8   ? FMD_HEAD(__nv_bfloat16, false, false)
            : f16ops ? FMD_HEAD(__nv_bfloat16, true, true)
                     : FMD_HEAD(__nv_bfloat16, true, false);
  else
    parts = W.q8 ? FMD_HEAD(__half, true, false) : FMD_HEAD(__half, false, false);
#undef FMD_HEAD
  if (parts > 0) return parts;
  // activation tile too large for the resident kernel: the cluster GEMV,
  // which normalises on the fly and so needs the sums of squares
  if (ep.ssq == nullptr) return 0;
  return launch_gemv(at, kGemvLogits, true, W, x, ldx, row_map, n_rows_ptr, max_rows, ep, status, s)
             ? W.N / gemv_tile_features(kGemvLogits)
             : 0;
}

void launch_pick_reduce(const int* n_sample_ptr, int B, const float* best_val, const int* best_idx, int n_parts,
                        int* next_ids, int vocab, int* status, cudaStream_t s) {
  launch_pdl(k_pick_reduce, dim3(B), dim3(256), 0, s, n_sample_ptr, best_val, best_idx, n_parts, next_ids, vocab,
             status);
}

}  // namespace fmd
