// Data-movement and normalisation kernels of the audio tower: the operand
// layouts of the two convolutions, LayerNorm, and weight conversion.
//
// The reference's front convolutions are candle `conv1d` calls over the
// (batch, n_mels, frames) log-mel tensor (whisper_encoder.rs:142-155): conv1
// kernel 3 / stride 1 / padding 1, conv2 kernel 3 / stride 2 / padding 1. Here
// both become GEMMs on the tensor cores over "unfolded" operands, row = output
// frame, column = (tap k, input channel c): conv1 reads mel[c][t + k - 1],
// conv2 reads the conv1 output row 2 t + k - 1 (zero outside the chunk). The
// weights are reordered once to the same (k, c) column order.
// LayerNorm (`LayerNorm::forward`, linear.rs:321-328, eps 1e-5 in the encoder)
// reads the f32 residual stream: mean, then the mean of squared deviations,
// both in f32, one warp per row.
#include <algorithm>

#include "../../include/fmd_decoder.h"
#include "fmd_audio.cuh"

namespace fmd {

namespace {

template <int DT>
FMD_DEV float ld_f(const void* p, size_t i) {
  if constexpr (DT == FMD_DT_F32) {
    return static_cast<const float*>(p)[i];
  } else if constexpr (DT == FMD_DT_F16) {
    return __half2float(static_cast<const __half*>(p)[i]);
  } else {
    return __uint_as_float((uint32_t)static_cast<const uint16_t*>(p)[i] << 16);
  }
}

constexpr int kMelRows = 32;   // output frames per block
constexpr int kMaxMels = 128;

template <typename T, int DT>
__global__ void __launch_bounds__(256) k_im2col_mel(const void* __restrict__ mel, int n_mels, int F, int kp,
                                                    T* __restrict__ a1) {
  __shared__ float tile[kMaxMels][kMelRows + 3];
  const int b = blockIdx.y, t0 = blockIdx.x * kMelRows;
  const size_t mel0 = (size_t)b * n_mels * F;
  for (int i = threadIdx.x; i < n_mels * (kMelRows + 2); i += blockDim.x) {
    const int c = i / (kMelRows + 2), tt = i % (kMelRows + 2);
    const int t = t0 - 1 + tt;
    tile[c][tt] = (t >= 0 && t < F) ? ld_f<DT>(mel, mel0 + (size_t)c * F + t) : 0.f;
  }
  __syncthreads();
  const int rows = min(kMelRows, F - t0);
  for (int i = threadIdx.x; i < rows * kp; i += blockDim.x) {
    const int r = i / kp, col = i % kp;
    const int k = col / n_mels, c = col % n_mels;
    const float v = col < 3 * n_mels ? tile[c][r + k] : 0.f;
    a1[((size_t)b * F + t0 + r) * kp + col] = Act<T>::from_f(v);
  }
}

__global__ void __launch_bounds__(256) k_im2col_conv2(const uint4* __restrict__ x1, int F, int D8, size_t total,
                                                      uint4* __restrict__ a2) {
  const int Tp = F / 2, row8 = 3 * D8;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / row8;
    const int rem = (int)(i % row8);
    const int k = rem / D8, c8 = rem % D8;
    const int b = (int)(row / Tp), t = (int)(row % Tp);
    const int tin = 2 * t + k - 1;
    a2[i] = (tin >= 0 && tin < F) ? __ldg(x1 + ((size_t)b * F + tin) * D8 + c8) : make_uint4(0, 0, 0, 0);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) k_layernorm(const float* __restrict__ x, const int2* __restrict__ rowmap,
                                                   int rows, int D, const float* __restrict__ w,
                                                   const float* __restrict__ bias, float eps, T* __restrict__ out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int2 m = rowmap ? rowmap[warp] : make_int2(warp, warp);
  const int nv = D / 128;  // float4s per lane
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)m.x * D);
  float4 v[16];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i < nv) {
      v[i] = xr[i * 32 + lane];
      sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
  }
  const float mean = warp_sum(sum) / (float)D;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i < nv) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      sq += (a * a + b * b) + (c * c + d * d);
    }
  }
  const float rstd = rsqrtf(warp_sum(sq) / (float)D + eps);
  T* orow = out + (size_t)m.y * D;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i < nv) {
      const int col = (i * 32 + lane) * 4;
      const float4 g = __ldg(reinterpret_cast<const float4*>(w + col));
      const float4 bb = __ldg(reinterpret_cast<const float4*>(bias + col));
      uint2 u;
      u.x = Act<T>::pack2((v[i].x - mean) * rstd * g.x + bb.x, (v[i].y - mean) * rstd * g.y + bb.y);
      u.y = Act<T>::pack2((v[i].z - mean) * rstd * g.z + bb.z, (v[i].w - mean) * rstd * g.w + bb.w);
      *reinterpret_cast<uint2*>(orow + col) = u;
    }
  }
}

template <typename T, int DT>
__global__ void k_convert_act(const void* __restrict__ src, size_t n, T* __restrict__ dst) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = Act<T>::from_f(ld_f<DT>(src, i));
}

template <int DT>
__global__ void k_convert_f32(const void* __restrict__ src, size_t n, float* __restrict__ dst) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = ld_f<DT>(src, i);
}

template <typename T, int DT>
__global__ void k_conv_weight(const void* __restrict__ src, int O, int C, int kp, T* __restrict__ dst) {
  const size_t n = (size_t)O * kp;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int o = (int)(i / kp), col = (int)(i % kp);
    const int k = col / C, c = col % C;
    dst[i] = Act<T>::from_f(col < 3 * C ? ld_f<DT>(src, ((size_t)o * C + c) * 3 + k) : 0.f);
  }
}

int grid_for(size_t n) { return (int)std::min<size_t>((n + 255) / 256, 148 * 32); }

template <typename T>
void im2col_mel_t(const void* mel, int mel_dt, int n_chunks, int n_mels, int F, int kp, void* a1, cudaStream_t s) {
  const dim3 grid((F + kMelRows - 1) / kMelRows, n_chunks);
  T* out = static_cast<T*>(a1);
  if (mel_dt == FMD_DT_F32) k_im2col_mel<T, FMD_DT_F32><<<grid, 256, 0, s>>>(mel, n_mels, F, kp, out);
  else if (mel_dt == FMD_DT_F16) k_im2col_mel<T, FMD_DT_F16><<<grid, 256, 0, s>>>(mel, n_mels, F, kp, out);
  else k_im2col_mel<T, FMD_DT_BF16><<<grid, 256, 0, s>>>(mel, n_mels, F, kp, out);
}

template <typename T>
void convert_act_t(const void* src, int dt, size_t n, void* dst, cudaStream_t s) {
  T* o = static_cast<T*>(dst);
  if (dt == FMD_DT_F32) k_convert_act<T, FMD_DT_F32><<<grid_for(n), 256, 0, s>>>(src, n, o);
  else if (dt == FMD_DT_F16) k_convert_act<T, FMD_DT_F16><<<grid_for(n), 256, 0, s>>>(src, n, o);
  else k_convert_act<T, FMD_DT_BF16><<<grid_for(n), 256, 0, s>>>(src, n, o);
}

template <typename T>
void conv_weight_t(const void* src, int dt, int O, int C, int kp, void* dst, cudaStream_t s) {
  const size_t n = (size_t)O * kp;
  T* o = static_cast<T*>(dst);
  if (dt == FMD_DT_F32) k_conv_weight<T, FMD_DT_F32><<<grid_for(n), 256, 0, s>>>(src, O, C, kp, o);
  else if (dt == FMD_DT_F16) k_conv_weight<T, FMD_DT_F16><<<grid_for(n), 256, 0, s>>>(src, O, C, kp, o);
  else k_conv_weight<T, FMD_DT_BF16><<<grid_for(n), 256, 0, s>>>(src, O, C, kp, o);
}

}  // namespace

void launch_im2col_mel(ActType at, const void* mel, int mel_dt, int n_chunks, int n_mels, int n_frames, int kp,
                       void* a1, cudaStream_t s) {
  if (at == kBF16) im2col_mel_t<__nv_bfloat16>(mel, mel_dt, n_chunks, n_mels, n_frames, kp, a1, s);
  else im2col_mel_t<__half>(mel, mel_dt, n_chunks, n_mels, n_frames, kp, a1, s);
}

void launch_im2col_conv2(ActType, const void* x1, int n_chunks, int n_frames, int D, void* a2, cudaStream_t s) {
  const size_t total = (size_t)n_chunks * (n_frames / 2) * 3 * (D / 8);
  k_im2col_conv2<<<grid_for(total), 256, 0, s>>>(static_cast<const uint4*>(x1), n_frames, D / 8, total,
                                                static_cast<uint4*>(a2));
}

void launch_layernorm(ActType at, const float* x, const int2* rowmap, int rows, int D, const float* w,
                      const float* b, float eps, void* out, cudaStream_t s) {
  const int blocks = (rows + 7) / 8;  // 8 warps (rows) per block
  if (at == kBF16)
    k_layernorm<__nv_bfloat16><<<blocks, 256, 0, s>>>(x, rowmap, rows, D, w, b, eps, (__nv_bfloat16*)out);
  else
    k_layernorm<__half><<<blocks, 256, 0, s>>>(x, rowmap, rows, D, w, b, eps, (__half*)out);
}

void launch_convert_act(ActType at, const void* src, int src_dt, size_t n, void* dst, cudaStream_t s) {
  if (n == 0) return;
  if (at == kBF16) convert_act_t<__nv_bfloat16>(src, src_dt, n, dst, s);
  else convert_act_t<__half>(src, src_dt, n, dst, s);
}

void launch_convert_f32(const void* src, int src_dt, size_t n, float* dst, cudaStream_t s) {
  if (n == 0) return;
  if (src_dt == FMD_DT_F32) k_convert_f32<FMD_DT_F32><<<grid_for(n), 256, 0, s>>>(src, n, dst);
  else if (src_dt == FMD_DT_F16) k_convert_f32<FMD_DT_F16><<<grid_for(n), 256, 0, s>>>(src, n, dst);
  else k_convert_f32<FMD_DT_BF16><<<grid_for(n), 256, 0, s>>>(src, n, dst);
}

void launch_conv_weight(ActType at, const void* src, int src_dt, int O, int C, int kp, void* dst, cudaStream_t s) {
  if (at == kBF16) conv_weight_t<__nv_bfloat16>(src, src_dt, O, C, kp, dst, s);
  else conv_weight_t<__half>(src, src_dt, O, C, kp, dst, s);
}

}  // namespace fmd
