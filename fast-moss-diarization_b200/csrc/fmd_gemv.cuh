// Fragment-level building blocks of the decode-step projections, shared by
// the per-projection GEMV kernels and the persistent layer-tail kernel
// (fmd_gemv.cu, fmd_chain.cu): the decode-packed weight unit format, the
// exact Q8_0 operand conversion and the per-block scaled MMA.
#pragma once

#include "fmd_common.cuh"

namespace fmd {

// Decode-packed weights. Each CTA's slice (FT features x K/S) is one
// contiguous tile in HBM, ordered [k-block][warp][fragment] so that a k-block
// is one TMA bulk copy and a warp's fragment reads are 512 consecutive bytes
// (conflict-free, no padding). One (k-block, warp) unit covers 16 features x
// 64 k (two Q8_0 blocks of 32):
//  * Q8_0: [0, 512) lane-major 16 bytes of feature g, [512, 1024) feature
//    g + 8, [1024, 1088) the f16 scales of the unit's 16 features x 2 blocks
//    (feature-major), so the scales travel with the quants. Lane (g, t)
//    holds k [8t, 8t + 8) of block 0 followed by k [32 + 8t, 32 + 8t + 8) of
//    block 1, so that two k16 MMAs cover exactly one block;
//  * 16-bit: four 512-byte planes: feature g k 16t + 0-7 | 8-15, g + 8 the
//    same.
constexpr int kUnitQ8 = 1088;
constexpr int kUnitDense = 2048;

struct WRegs {
  int4 a, b, c, d;
  uint32_t sg, sh;  // Q8_0: f16 scales of (feature g | g + 8) x (block 0, block 1)
};

// Activation row stride (elements) of a staged tile: the Q8_0 fragments read
// 16 bytes at k 8t and 32 + 8t, the dense ones at 16t and 16t + 8; a row
// stride of 64 (Q8_0) or 16 (dense) bytes modulo 128 keeps the 8 lanes of a
// quarter-warp on distinct banks.
template <bool Q8>
constexpr int x_pad() {
  return Q8 ? 32 : 8;
}

// rs[r] = rsqrt(mean(x^2) + eps) of rows r < rows from the per-tile sums of
// squares ssq[row][tiles]: one thread per row, each chunk of 16 partials
// loaded together (one round trip per chunk), summed in order.
FMD_DEV void rows_rsqrt(const float* __restrict__ ssq, int tiles, const int* __restrict__ row_map, int row0, int rows,
                        int K, float eps, float* __restrict__ rs, int nthreads) {
  for (int r = threadIdx.x; r < rows; r += nthreads) {
    const float* sp = ssq + (size_t)(row_map ? row_map[row0 + r] : row0 + r) * tiles;
    float ss = 0.f;
    for (int i0 = 0; i0 < tiles; i0 += 16) {
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = i0 + i < tiles ? sp[i0 + i] : 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) ss += v[i];
    }
    rs[r] = rsqrtf(ss / K + eps);
  }
}

// Four int8 weights (one 32-bit word) -> two packed 16-bit operands holding
// exactly the same integers (|q| <= 127 is exact in f16 and bf16):
// lo = (q0, q1), hi = (q2, q3).
template <typename T>
FMD_DEV void i8x4_to_act(uint32_t w, uint32_t& lo, uint32_t& hi);
template <>
FMD_DEV void i8x4_to_act<__half>(uint32_t w, uint32_t& lo, uint32_t& hi) {
  // biased bytes u = q + 128 as the low mantissa bits of 1024 (f16 0x6400):
  // the f16 value 1024 + u, minus 1152 = q, all steps exact
  const uint32_t v = w ^ 0x80808080u;
  uint32_t a = __byte_perm(v, 0x64646464u, 0x4140u), b = __byte_perm(v, 0x64646464u, 0x4342u);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  const __half2 qa = __hsub2(*reinterpret_cast<__half2*>(&a), bias), qb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
  lo = *reinterpret_cast<const uint32_t*>(&qa);
  hi = *reinterpret_cast<const uint32_t*>(&qb);
}
template <>
FMD_DEV void i8x4_to_act<__nv_bfloat16>(uint32_t w, uint32_t& lo, uint32_t& hi) {
  // biased bytes as the low mantissa bits of 2^23 (f32 0x4B000000): the f32
  // value 2^23 + u, minus 2^23 + 128 = q exactly; bf16 packing of an integer
  // of at most 7 bits is exact
  const uint32_t v = w ^ 0x80808080u;
  float f[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) f[i] = __int_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | i)) - 8388736.f;
  lo = Act<__nv_bfloat16>::pack2(f[0], f[1]);
  hi = Act<__nv_bfloat16>::pack2(f[2], f[3]);
}

// d = a * b + 0 (the accumulator starts at zero: one block's partial sum)
template <typename T>
FMD_DEV void mma16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
FMD_DEV void mma16816_z<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}
template <>
FMD_DEV void mma16816_z<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// A fragments of the 4 MMAs of one 64-wide k-block.
//  * Q8_0: MMA j covers block j >> 1, k 32 (j >> 1) + 8t + 4 (j & 1) + {0..3}
//    for lane t (k16 fragment order: logical k 2t, 2t+1 -> the first two,
//    2t+8, 2t+9 -> the last two), i.e. word j of the lane's 16 bytes;
//  * 16-bit: MMA j covers k 16t + 4j + {0..3} (the same logical-to-physical
//    k permutation as fmd_kernels.cu's k_linear).
// The activation fragments use the same k permutation (gemv_xfrag).
template <typename T, bool Q8>
FMD_DEV void gemv_afrag(const WRegs& w, uint32_t (&af)[4][4]) {
  if constexpr (Q8) {
    const uint32_t* ua = reinterpret_cast<const uint32_t*>(&w.a);
    const uint32_t* ub = reinterpret_cast<const uint32_t*>(&w.b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      i8x4_to_act<T>(ua[j], af[j][0], af[j][2]);
      i8x4_to_act<T>(ub[j], af[j][1], af[j][3]);
    }
  } else {
    const uint32_t* ua = reinterpret_cast<const uint32_t*>(&w.a);
    const uint32_t* ub = reinterpret_cast<const uint32_t*>(&w.b);
    const uint32_t* uc = reinterpret_cast<const uint32_t*>(&w.c);
    const uint32_t* ud = reinterpret_cast<const uint32_t*>(&w.d);
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
}

// One warp's fragment registers of a staged (k-block, warp) unit.
template <bool Q8>
FMD_DEV void gemv_wload(const uint8_t* u, int lane, WRegs& w) {
  w.a = *reinterpret_cast<const int4*>(u + lane * 16);
  w.b = *reinterpret_cast<const int4*>(u + 512 + lane * 16);
  if constexpr (Q8) {
    const int g = lane >> 2;
    const uint32_t* sc = reinterpret_cast<const uint32_t*>(u + 1024);
    w.sg = sc[g];
    w.sh = sc[g + 8];
  } else {
    w.c = *reinterpret_cast<const int4*>(u + 1024 + lane * 16);
    w.d = *reinterpret_cast<const int4*>(u + 1536 + lane * 16);
  }
}

// The activation fragment words of one 8-row n-tile for a 64-wide k-block:
// `xr` points at the lane's row (g) and k-block start.
template <typename T, bool Q8>
FMD_DEV void gemv_xfrag(const T* xr, int t, uint32_t (&xw)[8]) {
  const int4 x0 = *reinterpret_cast<const int4*>(xr + (Q8 ? 8 * t : 16 * t));
  const int4 x1 = *reinterpret_cast<const int4*>(xr + (Q8 ? 32 + 8 * t : 16 * t + 8));
  xw[0] = (uint32_t)x0.x, xw[1] = (uint32_t)x0.y, xw[2] = (uint32_t)x0.z, xw[3] = (uint32_t)x0.w;
  xw[4] = (uint32_t)x1.x, xw[5] = (uint32_t)x1.y, xw[6] = (uint32_t)x1.z, xw[7] = (uint32_t)x1.w;
}

// acc (16 features x 8 rows, the mma C layout) += W_kblock x X_kblock.
// Q8_0: each 32-wide block's product of the exact int8 weights is summed on
// its own and then scaled by the block's f16 scale in f32, i.e.
// sum_b d_b * sum_{k in b} q_k x_k: the reference's dequantise-then-matmul
// (q * d in f32) up to the f32 summation order.
template <typename T, bool Q8>
FMD_DEV void gemv_kblock(float (&acc)[4], const uint32_t (&af)[4][4], const uint32_t (&xw)[8], const WRegs& w) {
  if constexpr (Q8) {
    float t0[4], t1[4];
    mma16816_z<T>(t0, af[0], xw[0], xw[1]);
    mma16816<T>(t0, af[1], xw[2], xw[3]);
    mma16816_z<T>(t1, af[2], xw[4], xw[5]);
    mma16816<T>(t1, af[3], xw[6], xw[7]);
    const float2 dg = __half22float2(*reinterpret_cast<const __half2*>(&w.sg));
    const float2 dh = __half22float2(*reinterpret_cast<const __half2*>(&w.sh));
    acc[0] = fmaf(dg.y, t1[0], fmaf(dg.x, t0[0], acc[0]));
    acc[1] = fmaf(dg.y, t1[1], fmaf(dg.x, t0[1], acc[1]));
    acc[2] = fmaf(dh.y, t1[2], fmaf(dh.x, t0[2], acc[2]));
    acc[3] = fmaf(dh.y, t1[3], fmaf(dh.x, t0[3], acc[3]));
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) mma16816<T>(acc, af[j], xw[2 * j], xw[2 * j + 1]);
  }
}

}  // namespace fmd
