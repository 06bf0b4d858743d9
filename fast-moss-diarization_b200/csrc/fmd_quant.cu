// GGML Q8_0 quantisation on the GPU: the `QTensor::quantize(&w,
// GgmlDType::Q8_0)` step the reference applies to every large projection at
// load time, from the f32 value of each weight
// (crates/fmd-core/src/model/linear.rs:194-202, :239-251; tied head
// qwen3.rs:566-578).
//
// GGML's published Q8_0: blocks of 32 consecutive values of a row-major
// matrix; d = amax / 127 in f32, stored as an IEEE f16 (round to nearest
// even); id = 1 / d (0 when d == 0); q = roundf(x * id), halves away from
// zero. Every step is a single IEEE operation, so the device result equals the
// host quantiser's bit for bit. One warp per block: lane j converts value j
// to f32 (exact for f16 and bf16 sources), the warp reduces |x| to amax.
#include <algorithm>

#include "../../include/fmd_decoder.h"
#include "fmd_common.cuh"

namespace fmd {

namespace {

template <int DT>
FMD_DEV float load_f32(const void* src, long long i) {
  if constexpr (DT == FMD_DT_F32) {
    return static_cast<const float*>(src)[i];
  } else if constexpr (DT == FMD_DT_F16) {
    return __half2float(static_cast<const __half*>(src)[i]);
  } else {
    return __uint_as_float((uint32_t)static_cast<const uint16_t*>(src)[i] << 16);
  }
}

template <int DT>
__global__ void __launch_bounds__(256) k_q8_0_quantize(const void* __restrict__ src, long long n_blocks,
                                                       int8_t* __restrict__ qs, uint16_t* __restrict__ d) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long b = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n_blocks; b += warps) {
    const float x = load_f32<DT>(src, b * 32 + lane);
    float amax = fabsf(x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float dd = amax / 127.f;
    const float id = dd != 0.f ? 1.f / dd : 0.f;
    qs[b * 32 + lane] = (int8_t)roundf(x * id);
    if (lane == 0) d[b] = __half_as_ushort(__float2half_rn(dd));
  }
}

bool device_or_managed(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

}  // namespace

}  // namespace fmd

extern "C" int fmd_q8_0_quantize_device(const void* src, int32_t src_dtype, int64_t rows, int64_t cols, int8_t* qs,
                                        uint16_t* d, void* stream) {
  using namespace fmd;
  if (!src || !qs || !d || rows < 0 || cols < 0 || cols % 32 != 0) return FMD_EINVAL;
  if (src_dtype != FMD_DT_F32 && src_dtype != FMD_DT_F16 && src_dtype != FMD_DT_BF16) return FMD_EINVAL;
  if (rows == 0 || cols == 0) return FMD_OK;
  if (!device_or_managed(src) || !device_or_managed(qs) || !device_or_managed(d)) return FMD_EINVAL;
  const long long n_blocks = (long long)rows * (cols / 32);
  const int grid = (int)std::min<long long>((n_blocks + 7) / 8, 148LL * 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (src_dtype == FMD_DT_F32) k_q8_0_quantize<FMD_DT_F32><<<grid, 256, 0, s>>>(src, n_blocks, qs, d);
  else if (src_dtype == FMD_DT_F16) k_q8_0_quantize<FMD_DT_F16><<<grid, 256, 0, s>>>(src, n_blocks, qs, d);
  else k_q8_0_quantize<FMD_DT_BF16><<<grid, 256, 0, s>>>(src, n_blocks, qs, d);
  return cudaGetLastError() == cudaSuccess ? FMD_OK : FMD_EIO;
}
