// sm_100a kernels of the batched Qwen3 decoder step.
//
// Every kernel reads its row counts from the device plan (`PlanCounts`), so
// grids are fixed per handle and a whole step can be captured once in a CUDA
// graph and replayed while the device scheduler changes the batch.
//
// Arithmetic contract (mirrors the reference's rounding points,
// crates/fmd-core/src/model/qwen3.rs and linear.rs): every op result that the
// reference stores in the activation dtype is rounded to it here too; matmuls
// and reductions accumulate in f32.
#include <float.h>
#include <math.h>

#include "fmd_kernels.cuh"

namespace fmd {

namespace {

template <int NT>
FMD_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s += red[i];
  __syncthreads();
  return s;
}

// ---------------------------------------------------------------------------
// Embedding gather (qwen3.rs:405-412) fused with layer 0's input RMSNorm
// (linear.rs:293-302). Rows come from the token table or, for prompt rows,
// from the prompt-embedding arena (the spliced audio/text embeddings). As the
// first kernel of a decode step it also clears the step's synchronisation
// counters (`zero`, `zero_n` ints) of the persistent layer-tail kernels.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(128) k_embed_norm(Plan p, const T* __restrict__ table, const T* __restrict__ arena,
                                                    T* __restrict__ x, const T* __restrict__ w, T* __restrict__ xn,
                                                    int H, float eps, float* __restrict__ ssq, int ssq_tiles,
                                                    int* __restrict__ zero, int zero_n) {
  __shared__ float red[4];
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch
  if (zero != nullptr)
    for (int i = blockIdx.x * 128 + threadIdx.x; i < zero_n; i += gridDim.x * 128) zero[i] = 0;
  const int n_rows = p.counts->n_rows;
  for (int r = blockIdx.x; r < n_rows; r += gridDim.x) {
  const int tok = p.row_tok[r];
  const T* src = tok >= 0 ? table + (size_t)tok * H : arena + (size_t)p.row_emb[r] * H;
  T* xr = x + (size_t)r * H;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += 128 * 8) {
    const int4 v = *reinterpret_cast<const int4*>(src + i);
    *reinterpret_cast<int4*>(xr + i) = v;
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = Act<T>::unpack2(u[j]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  const float tot = block_sum<128>(ss, red);
  const float inv = rsqrtf(tot / H + eps);
  if (ssq != nullptr)
    for (int i = threadIdx.x; i < ssq_tiles; i += 128) ssq[(size_t)r * ssq_tiles + i] = i == 0 ? tot : 0.f;
  for (int i = threadIdx.x * 8; i < H; i += 128 * 8) {
    const int4 v = *reinterpret_cast<const int4*>(src + i);
    const int4 wv = *reinterpret_cast<const int4*>(w + i);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = Act<T>::unpack2(u[j]);
      const float2 g = Act<T>::unpack2(uw[j]);
      o[j] = Act<T>::pack2(f.x * inv * g.x, f.y * inv * g.y);
    }
    *reinterpret_cast<int4*>(xn + (size_t)r * H + i) = *reinterpret_cast<int4*>(o);
  }
  }
}

// ---------------------------------------------------------------------------
// Residual add + RMSNorm: x <- rnd(x + rnd(sum_s part[s])); xn <- rmsnorm(x).
// The O-projection and down-projection epilogues (qwen3.rs:333-338) fused with
// the next norm (post-attention, next layer's input, or the final norm).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(128) k_residual_norm(const int* __restrict__ n_rows_ptr, T* __restrict__ x,
                                                       const float* __restrict__ part, PartSplit split,
                                                       size_t split_stride, const T* __restrict__ w,
                                                       T* __restrict__ xn, int H, float eps) {
  __shared__ float red[4];
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch
  const int n_rows = *n_rows_ptr;
  const int S = split.at(n_rows);
  for (int r = blockIdx.x; r < n_rows; r += gridDim.x) {
  T* xr = x + (size_t)r * H;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += 128 * 8) {
    int4 v = *reinterpret_cast<const int4*>(xr + i);
    uint32_t* u = reinterpret_cast<uint32_t*>(&v);
    if (part != nullptr) {
      float acc[8];
      const float* p0 = part + (size_t)r * H + i;
      float4 a = *reinterpret_cast<const float4*>(p0), b = *reinterpret_cast<const float4*>(p0 + 4);
      acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w; acc[4] = b.x; acc[5] = b.y; acc[6] = b.z; acc[7] = b.w;
#pragma unroll 4
      for (int s = 1; s < S; ++s) {  // unrolled: the partial loads are issued together
        const float* ps = p0 + (size_t)s * split_stride;
        a = *reinterpret_cast<const float4*>(ps);
        b = *reinterpret_cast<const float4*>(ps + 4);
        acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
        acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Act<T>::unpack2(u[j]);
        u[j] = Act<T>::pack2(f.x + rnd<T>(acc[2 * j]), f.y + rnd<T>(acc[2 * j + 1]));
      }
      *reinterpret_cast<int4*>(xr + i) = v;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = Act<T>::unpack2(u[j]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  const float inv = rsqrtf(block_sum<128>(ss, red) / H + eps);
  for (int i = threadIdx.x * 8; i < H; i += 128 * 8) {
    const int4 v = *reinterpret_cast<const int4*>(xr + i);
    const int4 wv = *reinterpret_cast<const int4*>(w + i);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = Act<T>::unpack2(u[j]);
      const float2 g = Act<T>::unpack2(uw[j]);
      o[j] = Act<T>::pack2(f.x * inv * g.x, f.y * inv * g.y);
    }
    *reinterpret_cast<int4*>(xn + (size_t)r * H + i) = *reinterpret_cast<int4*>(o);
  }
  }
}

// ---------------------------------------------------------------------------
// Skinny GEMM y = x W^T on the tensor cores (mma.sync m16n8k16, f32 acc),
// weights fed straight from HBM into A-fragments (Q8_0 dequantised in
// registers), activations staged in shared memory.
//
// Swap-AB: A = 16 output features x 16 k, B = 16 k x 8 token rows. The k order
// inside one 64-wide k-block is permuted identically for A and B so that each
// thread reads 16 CONSECUTIVE weights of a row (one 16-byte Q8_0 load, within
// a single 32-value block, so one scale) and 16 consecutive activations:
// fragment k-column {2t,2t+1 | 2t+8,2t+9} of MMA j <-> k = 16t + 4j + {0,1 | 2,3}.
//
// CTA = 4 warps = 64 output features; grid.y splits K when the pass has
// <= 64 rows (decode), writing f32 partials that the consumer kernel sums;
// grid.z strides over 64-row tiles.
// ---------------------------------------------------------------------------
struct WRaw {
  int4 a, b, c, d;
  float da, db;
};

template <typename T, bool Q8>
__global__ void __launch_bounds__(128) k_linear(const T* __restrict__ x, int ldx, const int* __restrict__ row_map,
                                                const int* __restrict__ n_rows_ptr, LinW W, float* __restrict__ out,
                                                size_t split_stride, int decode_only) {
  __shared__ __align__(16) T xs[2][64][72];
  const int K = W.K, N = W.N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int f0 = blockIdx.x * 64 + warp * 16 + g;
  const int KB = K / kQ8Block;
  auto load_w_at = [&](int kbeg_, int kb, WRaw& w) {
    const int k = kbeg_ + kb * 64 + 16 * t;
    if constexpr (Q8) {
      w.a = ld_stream16(W.qs + (size_t)f0 * K + k);
      w.b = ld_stream16(W.qs + (size_t)(f0 + 8) * K + k);
      w.da = h2f_bits(W.d[(size_t)f0 * KB + (k >> 5)]);
      w.db = h2f_bits(W.d[(size_t)(f0 + 8) * KB + (k >> 5)]);
    } else {
      const T* wp = reinterpret_cast<const T*>(W.w);
      w.a = ld_stream16(wp + (size_t)f0 * K + k);
      w.b = ld_stream16(wp + (size_t)f0 * K + k + 8);
      w.c = ld_stream16(wp + (size_t)(f0 + 8) * K + k);
      w.d = ld_stream16(wp + (size_t)(f0 + 8) * K + k + 8);
    }
  };
  // Decode-only passes use the full K split, known before the plan is read:
  // the CTA's first two weight k-blocks are fetched while the previous kernel
  // is still finishing.
  WRaw wc, wn;
  bool pre = false;
  if (decode_only && (int)blockIdx.y < W.split) {
    const int kbeg0 = blockIdx.y * (K / W.split);
    load_w_at(kbeg0, 0, wc);
    if ((K / W.split) >> 6 > 1) load_w_at(kbeg0, 1, wn);
    pre = true;
  }
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch
  const int n_rows = *n_rows_ptr;
  const int S = effective_split(W.split, n_rows);
  if ((int)blockIdx.y >= S) return;
  const int klen = K / S;
  const int kbeg = blockIdx.y * klen;
  const int nkb = klen >> 6;
  pre = pre && S == W.split;  // the prefetch matches this pass's split

  for (int row0 = blockIdx.z * 64; row0 < n_rows; row0 += gridDim.z * 64) {
    const int rows = min(64, n_rows - row0);
    const int n_tiles = (rows + 7) >> 3;

    // per-thread source rows of the activation tile (4 x 16-byte chunks)
    const T* xsrc[4];
    int xbytes[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (threadIdx.x >> 3) + 16 * i;
      const int ch = threadIdx.x & 7;
      if (r < rows) {
        const int gr = row_map ? row_map[row0 + r] : row0 + r;
        xsrc[i] = x + (size_t)gr * ldx + kbeg + ch * 8;
        xbytes[i] = 16;
      } else {
        xsrc[i] = x;
        xbytes[i] = 0;
      }
    }
    auto load_x = [&](int stage, int kb) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = (threadIdx.x >> 3) + 16 * i;
        const int ch = threadIdx.x & 7;
        cp_async16(&xs[stage][r][ch * 8], xbytes[i] ? xsrc[i] + kb * 64 : xsrc[i], xbytes[i]);
      }
      cp_async_commit();
    };
    auto load_w = [&](int kb, WRaw& w) { load_w_at(kbeg, kb, w); };

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    load_x(0, 0);
    if (!pre) load_w(0, wc);
    for (int kb = 0; kb < nkb; ++kb) {
      if (kb + 1 < nkb) {
        load_x((kb + 1) & 1, kb + 1);
        if (!(pre && kb == 0)) load_w(kb + 1, wn);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();

      // A fragments for the 4 MMAs of this k-block
      uint32_t af[4][4];
      if constexpr (Q8) {
        const uint32_t* ua = reinterpret_cast<const uint32_t*>(&wc.a);
        const uint32_t* ub = reinterpret_cast<const uint32_t*>(&wc.b);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float e[4], f[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            // exact int8 -> f32 via the 2^23 magic (byte placed in the mantissa)
            e[i] = (__int_as_float(__byte_perm(ua[j] ^ 0x80808080u, 0x4B000000u, 0x7440u | i)) - 8388736.f) * wc.da;
            f[i] = (__int_as_float(__byte_perm(ub[j] ^ 0x80808080u, 0x4B000000u, 0x7440u | i)) - 8388736.f) * wc.db;
          }
          af[j][0] = Act<T>::pack2(e[0], e[1]);
          af[j][1] = Act<T>::pack2(f[0], f[1]);
          af[j][2] = Act<T>::pack2(e[2], e[3]);
          af[j][3] = Act<T>::pack2(f[2], f[3]);
        }
      } else {
        const uint32_t* ua = reinterpret_cast<const uint32_t*>(&wc.a);
        const uint32_t* ub = reinterpret_cast<const uint32_t*>(&wc.b);
        const uint32_t* uc = reinterpret_cast<const uint32_t*>(&wc.c);
        const uint32_t* ud = reinterpret_cast<const uint32_t*>(&wc.d);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t* r0 = j < 2 ? ua : ub;
          const uint32_t* r1 = j < 2 ? uc : ud;
          af[j][0] = r0[(2 * j) & 3];
          af[j][2] = r0[(2 * j + 1) & 3];
          af[j][1] = r1[(2 * j) & 3];
          af[j][3] = r1[(2 * j + 1) & 3];
        }
      }
      const int st = kb & 1;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        if (nt < n_tiles) {
          const int4 x0 = *reinterpret_cast<const int4*>(&xs[st][nt * 8 + g][16 * t]);
          const int4 x1 = *reinterpret_cast<const int4*>(&xs[st][nt * 8 + g][16 * t + 8]);
          const uint32_t xw[8] = {(uint32_t)x0.x, (uint32_t)x0.y, (uint32_t)x0.z, (uint32_t)x0.w,
                                  (uint32_t)x1.x, (uint32_t)x1.y, (uint32_t)x1.z, (uint32_t)x1.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) mma16816<T>(acc[nt], af[j], xw[2 * j], xw[2 * j + 1]);
        }
      }
      __syncthreads();
      wc = wn;
    }

    pre = false;  // a further row tile streams its weights again
    float* o = out + (size_t)blockIdx.y * split_stride;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      if (nt < n_tiles) {
        const int lr = nt * 8 + 2 * t;
        if (lr < rows) {
          o[(size_t)(row0 + lr) * N + f0] = acc[nt][0];
          o[(size_t)(row0 + lr) * N + f0 + 8] = acc[nt][2];
        }
        if (lr + 1 < rows) {
          o[(size_t)(row0 + lr + 1) * N + f0] = acc[nt][1];
          o[(size_t)(row0 + lr + 1) * N + f0 + 8] = acc[nt][3];
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// QKV epilogue (qwen3.rs:213-227): sum K-split partials, round, per-head
// RMSNorm of q and k (q_norm / k_norm), RoPE with the activation-dtype tables
// at the row's own position, then q -> q buffer and k, v -> the paged cache.
// One warp per head, 4 dims per lane; the RoPE partner dim (d +- 64) lives 16
// lanes away.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) k_qkv_epilogue(Plan p, const float* __restrict__ part, PartSplit split,
                                                      size_t split_stride, int Hq, int Hkv,
                                                      const T* __restrict__ qn_w, const T* __restrict__ kn_w,
                                                      const T* __restrict__ cos_t, const T* __restrict__ sin_t,
                                                      T* __restrict__ q_out, KvView kv, int layer, float eps) {
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch
  const int n_rows = p.counts->n_rows;
  const int S = split.at(n_rows);
  const int N = (Hq + 2 * Hkv) * kHeadDim;
  for (int r = blockIdx.x; r < n_rows; r += gridDim.x) {
  const int pos = p.row_pos[r], slot = p.row_slot[r];
  const int page = kv.page_table[(size_t)slot * kv.max_pages_per_slot + (pos / kPageTokens)];
  const int off = pos % kPageTokens;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  T* kvb = reinterpret_cast<T*>(kv.base);
  for (int hh = warp; hh < Hq + 2 * Hkv; hh += 8) {
    const int c = hh * kHeadDim + lane * 4;
    float v[4];
    {
      const float* p0 = part + (size_t)r * N + c;
      float4 a = *reinterpret_cast<const float4*>(p0);
#pragma unroll 8
      for (int s = 1; s < S; ++s) {  // unrolled: the partial loads are issued together
        const float4 b = *reinterpret_cast<const float4*>(p0 + (size_t)s * split_stride);
        a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
      }
      v[0] = rnd<T>(a.x); v[1] = rnd<T>(a.y); v[2] = rnd<T>(a.z); v[3] = rnd<T>(a.w);
    }
    T* dst;
    if (hh < Hq + Hkv) {
      const T* nw = hh < Hq ? qn_w : kn_w;
      const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
      const float inv = rsqrtf(ss / kHeadDim + eps);
      float y[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = rnd<T>(v[i] * inv * Act<T>::to_f(nw[lane * 4 + i]));
      const int dd = (lane & 15) * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float pr = __shfl_xor_sync(0xffffffffu, y[i], 16);
        const float cs = Act<T>::to_f(cos_t[(size_t)pos * (kHeadDim / 2) + dd + i]);
        const float sn = Act<T>::to_f(sin_t[(size_t)pos * (kHeadDim / 2) + dd + i]);
        v[i] = lane < 16 ? y[i] * cs - pr * sn : pr * sn + y[i] * cs;
      }
      dst = hh < Hq ? q_out + (size_t)r * Hq * kHeadDim + hh * kHeadDim
                    : kvb + kv.elem_offset(layer, page, 0, hh - Hq) + (size_t)off * kHeadDim;
    } else {
      dst = kvb + kv.elem_offset(layer, page, 1, hh - Hq - Hkv) + (size_t)off * kHeadDim;
    }
    uint2 o;
    o.x = Act<T>::pack2(v[0], v[1]);
    o.y = Act<T>::pack2(v[2], v[3]);
    *reinterpret_cast<uint2*>(dst + lane * 4) = o;
  }
  }
}

// ---------------------------------------------------------------------------
// SwiGLU (qwen3.rs:288-292): h = rnd(rnd(silu(rnd(gate))) * rnd(up)); gate/up
// columns are interleaved in 32-groups (gate_col / up_col).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) k_silu_mul(const int* __restrict__ n_rows_ptr, const float* __restrict__ part,
                                                  PartSplit split, size_t split_stride, int I, T* __restrict__ h) {
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch
  const int n_rows = *n_rows_ptr;
  const int S = split.at(n_rows);
  for (int r = blockIdx.x; r < n_rows; r += gridDim.x) {
  const float* p0 = part + (size_t)r * 2 * I;
  for (int c = threadIdx.x * 4; c < I; c += blockDim.x * 4) {
    const int gc = gate_col(c), uc = up_col(c);  // 4 consecutive features never cross a 32-group
    float4 gs = *reinterpret_cast<const float4*>(p0 + gc);
    float4 us = *reinterpret_cast<const float4*>(p0 + uc);
#pragma unroll 4
    for (int s = 1; s < S; ++s) {  // unrolled: the partial loads are issued together
      const float4 a = *reinterpret_cast<const float4*>(p0 + (size_t)s * split_stride + gc);
      const float4 b = *reinterpret_cast<const float4*>(p0 + (size_t)s * split_stride + uc);
      gs.x += a.x; gs.y += a.y; gs.z += a.z; gs.w += a.w;
      us.x += b.x; us.y += b.y; us.z += b.z; us.w += b.w;
    }
    const float gv[4] = {gs.x, gs.y, gs.z, gs.w}, uv[4] = {us.x, us.y, us.z, us.w};
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float gr = rnd<T>(gv[i]);
      const float sg = rnd<T>(gr / (1.f + expf(-gr)));
      o[i] = sg * rnd<T>(uv[i]);
    }
    uint2 w;
    w.x = Act<T>::pack2(o[0], o[1]);
    w.y = Act<T>::pack2(o[2], o[3]);
    *reinterpret_cast<uint2*>(h + (size_t)r * I + c) = w;
  }
  }
}

// ---------------------------------------------------------------------------
// Logits + greedy pick (qwen3.rs:459-463, engine.rs:550-559): logits are the
// lm_head result rounded to the activation dtype, then widened to f32; the
// argmax takes the lowest index among equal maxima.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(1024) k_logits_argmax(const int* __restrict__ n_sample_ptr,
                                                        const float* __restrict__ part, int V,
                                                        float* __restrict__ logits, int* __restrict__ next_ids) {
  __shared__ float sv[32];
  __shared__ int si[32];
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch
  const int r = blockIdx.x;
  if (r >= *n_sample_ptr) return;
  const float* pr = part + (size_t)r * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = threadIdx.x * 4; v < V; v += 1024 * 4) {
    float4 a = *reinterpret_cast<const float4*>(pr + v);
    a.x = rnd<T>(a.x); a.y = rnd<T>(a.y); a.z = rnd<T>(a.z); a.w = rnd<T>(a.w);
    if (logits) *reinterpret_cast<float4*>(logits + (size_t)r * V + v) = a;
    if (a.x > best) { best = a.x; bi = v; }
    if (a.y > best) { best = a.y; bi = v + 1; }
    if (a.z > best) { best = a.z; bi = v + 2; }
    if (a.w > best) { best = a.w; bi = v + 3; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    best = sv[lane];
    bi = si[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) next_ids[r] = bi;
  }
}

// Dequantise / widen one stored projection to f32 (inspection only).
template <typename T>
__global__ void k_dequant(LinW W, float* __restrict__ out) {
  const size_t total = (size_t)W.N * W.K;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    if (W.q8) {
      const size_t n = i / W.K, k = i % W.K;
      out[i] = (float)W.qs[i] * h2f_bits(W.d[n * (W.K / kQ8Block) + k / kQ8Block]);
    } else {
      out[i] = Act<T>::to_f(reinterpret_cast<const T*>(W.w)[i]);
    }
  }
}

}  // namespace

// ---- launchers ----------------------------------------------------------------------

#define FMD_DISPATCH(at, ...)                  \
  do {                                         \
    if ((at) == kBF16) {                       \
      using T = __nv_bfloat16;                 \
      __VA_ARGS__;                             \
    } else {                                   \
      using T = __half;                        \
      __VA_ARGS__;                             \
    }                                          \
  } while (0)

void launch_embed_norm(ActType at, const Plan& p, int R, const void* table, const void* arena, void* x, const void* w,
                       void* xn, int H, float eps, float* ssq, int ssq_tiles, cudaStream_t s, int* zero, int zero_n) {
  FMD_DISPATCH(at, launch_pdl(k_embed_norm<T>, R, 128, 0, s, p, (const T*)table, (const T*)arena, (T*)x, (const T*)w,
                                                      (T*)xn, H, eps, ssq, ssq_tiles, zero, zero_n));
}

void launch_linear(ActType at, const LinW& W, const void* x, int ldx, const int* row_map, const int* n_rows_ptr,
                   int max_rows, float* out, size_t split_stride, bool decode_only, cudaStream_t s) {
  const int row_tiles = (max_rows + 63) / 64;
  dim3 grid(W.N / 64, W.split, row_tiles < 8 ? row_tiles : 8);
  FMD_DISPATCH(at, {
    if (W.q8)
      launch_pdl(k_linear<T, true>, grid, 128, 0, s, (const T*)x, ldx, row_map, n_rows_ptr, W, out, split_stride, (int)decode_only);
    else
      launch_pdl(k_linear<T, false>, grid, 128, 0, s, (const T*)x, ldx, row_map, n_rows_ptr, W, out, split_stride, (int)decode_only);
  });
}

void launch_qkv_epilogue(ActType at, const Plan& p, int R, const float* part, PartSplit split, size_t split_stride,
                         int Hq, int Hkv, const void* qn_w, const void* kn_w, const void* cos, const void* sin,
                         void* q_out, const KvView& kv, int layer, float eps, cudaStream_t s) {
  FMD_DISPATCH(at, launch_pdl(k_qkv_epilogue<T>, R, 256, 0, s, p, part, split, split_stride, Hq, Hkv, (const T*)qn_w,
                                                        (const T*)kn_w, (const T*)cos, (const T*)sin, (T*)q_out, kv,
                                                        layer, eps));
}

void launch_residual_norm(ActType at, const int* n_rows_ptr, int R, void* x, const float* part, PartSplit split,
                          size_t split_stride, const void* w, void* xn, int H, float eps, cudaStream_t s) {
  FMD_DISPATCH(at, launch_pdl(k_residual_norm<T>, R, 128, 0, s, n_rows_ptr, (T*)x, part, split, split_stride, (const T*)w,
                                                         (T*)xn, H, eps));
}

void launch_silu_mul(ActType at, const int* n_rows_ptr, int R, const float* part, PartSplit split, size_t split_stride,
                     int I, void* h, cudaStream_t s) {
  FMD_DISPATCH(at, launch_pdl(k_silu_mul<T>, R, 256, 0, s, n_rows_ptr, part, split, split_stride, I, (T*)h));
}

void launch_logits_argmax(ActType at, const int* n_sample_ptr, int B, const float* part, int V, float* logits,
                          int* next_ids, cudaStream_t s) {
  FMD_DISPATCH(at, launch_pdl(k_logits_argmax<T>, B, 1024, 0, s, n_sample_ptr, part, V, logits, next_ids));
}

// One bounded mbarrier wait on a barrier that nothing arrives on, with the
// caller's iteration limit: the wait every ring kernel uses, made to run out.
// The timeout path is the one the kernels take (status word set, no copy in
// flight, the CTA returns), so the host can check that a wait which gives up
// surfaces as FMD_ETIMEDOUT and leaves the context usable.
__global__ void k_wait_probe(uint32_t limit, int* __restrict__ status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    if (!mbar_wait_bounded(&bar, 0, limit)) report_timeout(status, kSiteWaitProbe);
  }
}

void launch_wait_probe(uint32_t limit, int* status, cudaStream_t s) { k_wait_probe<<<1, 32, 0, s>>>(limit, status); }

// Issue cost of tcgen05.mma (M 128 x N x K 16, kind::f16, zero operands in
// shared memory) in the two forms a kernel can take: form 0, one thread of a
// diverged warp runs the loop (`if (threadIdx.x == 0)`); form 1, the whole
// warp runs the loop and its elected lane issues, the form every tensor-core
// kernel of this library uses. cycles[0] = SM cycles per MMA from the first
// issue to the completion of the last (clock64, one CTA), or -1 if the final
// wait gave up.
__global__ void __launch_bounds__(128, 1) k_mma_issue_probe(int form, int n, int iters, long long* cycles,
                                                            int* status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_base_s;
  const uint32_t raw_u = smem_u32(smem_raw);
  const uint32_t base = (raw_u + 1023u) & ~1023u;  // A: 128 x 128 B, B: up to 256 x 128 B, swizzle atoms aligned
  uint8_t* base_p = smem_raw + (base - raw_u);
  for (int i = threadIdx.x; i < (48 * 1024) / 16; i += blockDim.x)
    reinterpret_cast<int4*>(base_p)[i] = make_int4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    fence_barrier_init();
  }
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  if (threadIdx.x < 32) {
    tmem_alloc(&tmem_base_s, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s, a = base, b = base + 16 * 1024;
  const uint32_t idesc = umma_idesc_f16(false, 128, n);
  if (threadIdx.x < 32) {
    long long t0 = 0, t1 = 0;
    bool ok = true;
    if (form == 0) {
      if (threadIdx.x == 0) {
        t0 = clock64();
        for (int i = 0; i < iters; ++i) {
          const uint32_t ko = (uint32_t)(i & 3) * 32u;
          umma_f16(tmem + (uint32_t)(((i >> 2) & 1) * n), umma_desc_sw128(a + ko), umma_desc_sw128(b + ko), idesc,
                   (i & 3) != 0);
        }
        umma_commit(&done);
        ok = mbar_wait_bounded(&done, 0, 1u << 24);
        t1 = clock64();
      }
      __syncwarp();
    } else {
      t0 = clock64();
      for (int i = 0; i < iters; ++i) {
        const uint32_t ko = (uint32_t)(i & 3) * 32u;
        if (elect_one())
          umma_f16(tmem + (uint32_t)(((i >> 2) & 1) * n), umma_desc_sw128(a + ko), umma_desc_sw128(b + ko), idesc,
                   (i & 3) != 0);
        __syncwarp();
      }
      if (elect_one()) umma_commit(&done);
      __syncwarp();
      ok = mbar_wait_warp(&done, 0, 1u << 24);
      t1 = clock64();
    }
    if (threadIdx.x == 0) {
      if (!ok) report_timeout(status, kSiteWaitProbe);
      cycles[0] = ok ? (t1 - t0) : -1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem, 512);
}

cudaError_t launch_mma_issue_probe(int form, int n, int iters, long long* cycles, int* status, cudaStream_t s) {
  constexpr int kSmem = 48 * 1024 + 1024;
  cudaError_t e = cudaFuncSetAttribute(k_mma_issue_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  k_mma_issue_probe<<<1, 128, kSmem, s>>>(form, n, iters, cycles, status);
  return cudaGetLastError();
}

cudaError_t init_kernels() { return cudaSuccess; }

void launch_dequant(ActType at, const LinW& W, float* out, cudaStream_t s) {
  FMD_DISPATCH(at, k_dequant<T><<<1024, 256, 0, s>>>(W, out));
}

// The two halves of a split decode step: rows [0, split) and [split, n).
__global__ void k_half_counts(const PlanCounts* __restrict__ full, PlanCounts* __restrict__ halves, int split) {
  griddep_wait();
  griddep_launch();  // only after the wait: see griddep_launch
  if (threadIdx.x == 0) {
    const int n = full->n_decode;
    PlanCounts lo{}, hi{};
    lo.n_rows = lo.n_decode = lo.n_sample = n < split ? n : split;
    hi.n_rows = hi.n_decode = hi.n_sample = n > split ? n - split : 0;
    halves[0] = lo;
    halves[1] = hi;
  }
}

void launch_half_counts(const PlanCounts* full, PlanCounts* halves, int split, cudaStream_t s) {
  launch_pdl(k_half_counts, dim3(1), dim3(32), 0, s, full, halves, split);
}

}  // namespace fmd
