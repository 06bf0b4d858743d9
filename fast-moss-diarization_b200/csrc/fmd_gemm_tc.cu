// Projections of a mixed (prefill-carrying) step on the 5th-generation tensor
// cores: out[split][rows][N] (f32) = X[rows][K] . W[N][K]^T.
//
// The reference runs these as one GEMM per projection over the chunk's rows
// (crates/fmd-core/src/model/linear.rs:29-65 through qwen3.rs:213-338). Here:
//  * both operands are 16-bit K-major tiles fetched by TMA with the 128-byte
//    swizzle: X through a tensor map over the activation buffer, W through one
//    over the projection's 16-bit weights (the Q8_0 weights' expansion, made
//    at load time: the values the dequantisation produces, so results are
//    unchanged);
//  * a CTA owns a 128-row x BN-feature tile (BN = 128 or 256) and a K range
//    (split-K over gridDim.z when the feature count alone leaves SMs idle).
//    Warp 0 (one lane) runs a STAGES-deep full/empty mbarrier ring of TMA
//    loads, warp 1 allocates BN tensor-memory columns and one lane issues
//    tcgen05.mma (M = 128, N = BN, K = 16; four per 64-wide k-block) and
//    releases each stage with tcgen05.commit, warps 2-5 read the f32
//    accumulator back with tcgen05.ld (warp w owns lanes 32 * (w % 4) ...)
//    and store the rows;
//  * every wait is bounded; a timeout sets the status word, and the CTA
//    drains its copies in flight and frees its tensor memory before leaving.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "fmd_kernels.cuh"

namespace fmd {

namespace {

constexpr int kTcBM = 128;  // rows per tile (MMA M)
constexpr int kTcBK = 64;   // 64 16-bit values = one 128-byte swizzle row
constexpr uint32_t kTcWaitLimit = 1u << 24;
constexpr int kTcStatusTimeout = -110;

template <typename T, int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
              const int* __restrict__ n_rows_ptr, int K, int N, float* __restrict__ out, size_t split_stride,
              int* __restrict__ status) {
  constexpr uint32_t A_BYTES = kTcBM * kTcBK * 2;
  constexpr uint32_t B_BYTES = BN * kTcBK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], done;
  __shared__ uint32_t tmem_base_s;
  griddep_launch();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t tiles = (raw + 1023u) & ~1023u;  // swizzle atoms need 1024-byte alignment
  uint8_t* tiles_p = smem_raw + (tiles - raw);

  griddep_wait();  // X and the row count come from earlier kernels
  const int n_rows = *n_rows_ptr;
  const int row0 = blockIdx.x * kTcBM;
  if (row0 >= n_rows) return;  // whole CTA, before any barrier or tensor memory exists
  const int n0 = blockIdx.y * BN;
  const int klen = K / gridDim.z, kbeg = blockIdx.z * klen, nk = klen / kTcBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&amap);
      prefetch_tmap(&bmap);
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int st = kb % STAGES;
        if (kb >= STAGES && !mbar_wait_bounded(&empty[st], ((kb / STAGES) + 1) & 1, kTcWaitLimit)) {
          ok = false;
          break;
        }
        uint8_t* a = tiles_p + st * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[st], STAGE_BYTES);
        tma_load_2d(a, &amap, kbeg + kb * kTcBK, row0, &full[st]);
        tma_load_2d(a + A_BYTES, &bmap, kbeg + kb * kTcBK, n0, &full[st]);
        issued = kb + 1;
      }
      if (!ok) {
        // the MMA side stopped consuming: let the copies in flight land
        for (int kb = issued - STAGES > 0 ? issued - STAGES : 0; kb < issued; ++kb)
          mbar_wait_bounded(&full[kb % STAGES], (kb / STAGES) & 1, kTcWaitLimit);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(Act<T>::kIsBf16, kTcBM, BN);
      for (int kb = 0; kb < nk; ++kb) {
        const int st = kb % STAGES;
        if (!mbar_wait_bounded(&full[st], (kb / STAGES) & 1, kTcWaitLimit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = tiles + st * STAGE_BYTES, b = a + A_BYTES;
#pragma unroll
        for (int j = 0; j < kTcBK / 16; ++j)
          umma_f16(tmem, umma_desc_sw128(a + j * 32), umma_desc_sw128(b + j * 32), idesc, (kb | j) != 0);
        umma_commit(&empty[st]);  // the stage is free once these MMAs have read it
      }
      umma_commit(&done);  // also after an abort: the epilogue must not wait forever
    }
  } else {
    // epilogue: warp w reads tensor-memory lanes 32 * (w % 4) .. + 31 = rows
    const int q = warp & 3;
    if (!mbar_wait_bounded(&done, 0, kTcWaitLimit)) ok = false;
    tc_fence_after();
    const int row = row0 + q * 32 + lane;
    float* orow = out + (size_t)blockIdx.z * split_stride + (size_t)row * N + n0;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
      tmem_ld_wait();
      if (ok && row < n_rows) {
        float4* o4 = reinterpret_cast<float4*>(orow + c * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          o4[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]), __uint_as_float(v[4 * i + 2]),
                              __uint_as_float(v[4 * i + 3]));
      }
    }
  }
  if (!ok) atomicExch(status, kTcStatusTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

template <int BN>
constexpr int tc_stages() {
  return BN == 256 ? 4 : 6;  // 192 KB of tiles either way
}

template <int BN>
size_t tc_smem_bytes() {
  return (size_t)tc_stages<BN>() * (kTcBM * kTcBK * 2 + BN * kTcBK * 2) + 1024;
}

template <typename T, int BN>
void launch_gemm_tc_t(const CUtensorMap& amap, const TcLinear& W, const int* n_rows_ptr, int max_rows, float* out,
                      size_t split_stride, int* status, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((max_rows + kTcBM - 1) / kTcBM, W.N / BN, W.split);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = tc_smem_bytes<BN>();
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k_gemm_tc<T, BN, tc_stages<BN>()>, amap, W.wmap, n_rows_ptr, W.K, W.N, out, split_stride,
                     status);
}

template <typename T>
cudaError_t init_gemm_tc_t() {
  cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<T, 128, tc_stages<128>()>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_bytes<128>());
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_gemm_tc<T, 256, tc_stages<256>()>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)tc_smem_bytes<256>());
}

}  // namespace

cudaError_t init_gemm_tc() {
  cudaError_t e = init_gemm_tc_t<__nv_bfloat16>();
  return e != cudaSuccess ? e : init_gemm_tc_t<__half>();
}

bool tc_plan(int N, int K, int* bn, int* split) {
  if (N % 128 || K % kTcBK) return false;
  *bn = (N % 256 == 0 && N >= 4096) ? 256 : 128;
  // narrow projections (hidden-sized outputs) leave SMs idle at 128 x 128
  // tiles: split their K in two when the halves stay >= 512 deep
  *split = (N <= 2048 && K % (2 * kTcBK) == 0 && K / 2 >= 512) ? 2 : 1;
  return true;
}

bool tc_make_map(void* encode_fn, CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
                 uint32_t box_outer) {
  if (encode_fn == nullptr || (reinterpret_cast<uintptr_t>(base) & 15) || (inner * 2) % 16 || box_outer > 256)
    return false;
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(encode_fn);
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBK, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool launch_gemm_tc(ActType at, const CUtensorMap& amap, const TcLinear& W, const int* n_rows_ptr, int max_rows,
                    float* out, size_t split_stride, int* status, cudaStream_t s) {
  if (!W.ok || (W.bn != 128 && W.bn != 256) || W.K % (kTcBK * W.split)) return false;
  if (at == kBF16) {
    if (W.bn == 256) launch_gemm_tc_t<__nv_bfloat16, 256>(amap, W, n_rows_ptr, max_rows, out, split_stride, status, s);
    else launch_gemm_tc_t<__nv_bfloat16, 128>(amap, W, n_rows_ptr, max_rows, out, split_stride, status, s);
  } else {
    if (W.bn == 256) launch_gemm_tc_t<__half, 256>(amap, W, n_rows_ptr, max_rows, out, split_stride, status, s);
    else launch_gemm_tc_t<__half, 128>(amap, W, n_rows_ptr, max_rows, out, split_stride, status, s);
  }
  return true;
}

}  // namespace fmd
