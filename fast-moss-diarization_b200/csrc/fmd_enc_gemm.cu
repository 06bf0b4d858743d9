// Projections of the audio tower on the 5th-generation tensor cores, with the
// elementwise work that follows each one fused into the epilogue:
// out[M][N] = epilogue(A[M][K] . W[N][K]^T + bias).
//
// The reference runs each as a dense candle matmul followed by separate
// broadcast_add / gelu_erf / silu / residual-add ops in the activation dtype
// (crates/fmd-core/src/model/whisper_encoder.rs:45-64, :88-100, :142-163;
// adaptor.rs:54-58; linear.rs:29-65). Here one kernel per projection:
//  * A (activations) and W (weights) are 16-bit K-major tiles fetched by TMA
//    with the 128-byte swizzle into a STAGES-deep full/empty mbarrier ring
//    (warp 0, one lane);
//  * warp 1 allocates BN tensor-memory columns and one lane issues
//    tcgen05.mma (M = 128, N = BN, K = 16; four per 64-wide k-block),
//    releasing each stage with tcgen05.commit;
//  * warps 2-5 read the f32 accumulator back with tcgen05.ld (warp w owns
//    lanes 32 * (w % 4) ... = tile rows), add the bias and apply the fused
//    epilogue (q/k scaling, erf-GELU, SiLU, the positional rows, or the
//    residual add into the f32 residual stream) before a single store.
// The residual stream is kept in f32 (the reference rounds it to the
// activation dtype after every add); LayerNorm reads it in f32.
// Every wait is bounded; a timeout sets the status word, the CTA drains its
// copies in flight and frees its tensor memory before leaving.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "fmd_audio.cuh"

namespace fmd {

namespace {

constexpr int kEgBM = 128;
constexpr int kEgBK = 64;
constexpr uint32_t kEgWaitLimit = 1u << 24;
constexpr int kEgStatusTimeout = -110;

FMD_DEV float gelu_erf(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

template <typename T, int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(192, 1)
    k_enc_gemm(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, int M, int K, int N,
               EncEpiArgs ep, int* __restrict__ status) {
  constexpr uint32_t A_BYTES = kEgBM * kEgBK * 2;
  constexpr uint32_t B_BYTES = BN * kEgBK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], done;
  __shared__ uint32_t tmem_base_s;
  griddep_launch();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t tiles = (raw + 1023u) & ~1023u;  // swizzle atoms need 1024-byte alignment
  uint8_t* tiles_p = smem_raw + (tiles - raw);
  const int row0 = blockIdx.x * kEgBM;
  const int n0 = blockIdx.y * BN;
  const int nk = K / kEgBK;

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
  griddep_wait();  // A (and the residual stream) come from earlier kernels

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&amap);
      prefetch_tmap(&bmap);
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int st = kb % STAGES;
        if (kb >= STAGES && !mbar_wait_bounded(&empty[st], ((kb / STAGES) + 1) & 1, kEgWaitLimit)) {
          ok = false;
          break;
        }
        uint8_t* a = tiles_p + st * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[st], STAGE_BYTES);
        tma_load_2d(a, &amap, kb * kEgBK, row0, &full[st]);
        tma_load_2d(a + A_BYTES, &bmap, kb * kEgBK, n0, &full[st]);
        issued = kb + 1;
      }
      if (!ok) {
        for (int kb = issued - STAGES > 0 ? issued - STAGES : 0; kb < issued; ++kb)
          mbar_wait_bounded(&full[kb % STAGES], (kb / STAGES) & 1, kEgWaitLimit);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(Act<T>::kIsBf16, kEgBM, BN);
      for (int kb = 0; kb < nk; ++kb) {
        const int st = kb % STAGES;
        if (!mbar_wait_bounded(&full[st], (kb / STAGES) & 1, kEgWaitLimit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = tiles + st * STAGE_BYTES, b = a + A_BYTES;
#pragma unroll
        for (int j = 0; j < kEgBK / 16; ++j)
          umma_f16(tmem, umma_desc_sw128(a + j * 32), umma_desc_sw128(b + j * 32), idesc, (kb | j) != 0);
        umma_commit(&empty[st]);
      }
      umma_commit(&done);  // also after an abort: the epilogue must not wait forever
    }
  } else {
    const int q = warp & 3;
    if (!mbar_wait_bounded(&done, 0, kEgWaitLimit)) ok = false;
    tc_fence_after();
    const int row = row0 + q * 32 + lane;
    const bool live = ok && row < M;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), r);
      tmem_ld_wait();
      if (!live) continue;
      const int col0 = n0 + c * 32;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      if (ep.bias != nullptr) {
        const float4* b4 = reinterpret_cast<const float4*>(ep.bias + col0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 bb = __ldg(b4 + i);
          v[4 * i] += bb.x;
          v[4 * i + 1] += bb.y;
          v[4 * i + 2] += bb.z;
          v[4 * i + 3] += bb.w;
        }
      }
      if constexpr (EPI == kEpiQkv) {
        if (col0 < ep.scale_cols) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= ep.scale;
        }
      } else if constexpr (EPI == kEpiGelu || EPI == kEpiGeluPos) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
      } else if constexpr (EPI == kEpiSilu) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = v[i] / (1.f + expf(-v[i]));
      }
      if constexpr (EPI == kEpiQkv || EPI == kEpiGelu || EPI == kEpiSilu) {
        uint4* o4 = reinterpret_cast<uint4*>(static_cast<T*>(ep.out) + (size_t)row * N + col0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 u;
          u.x = Act<T>::pack2(v[8 * i + 0], v[8 * i + 1]);
          u.y = Act<T>::pack2(v[8 * i + 2], v[8 * i + 3]);
          u.z = Act<T>::pack2(v[8 * i + 4], v[8 * i + 5]);
          u.w = Act<T>::pack2(v[8 * i + 6], v[8 * i + 7]);
          o4[i] = u;
        }
      } else {
        float4* o4 = reinterpret_cast<float4*>(static_cast<float*>(ep.out) + (size_t)row * N + col0);
        if constexpr (EPI == kEpiResid) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 x = o4[i];
            o4[i] = make_float4(x.x + v[4 * i], x.y + v[4 * i + 1], x.z + v[4 * i + 2], x.w + v[4 * i + 3]);
          }
        } else if constexpr (EPI == kEpiGeluPos) {
          const float4* p4 = reinterpret_cast<const float4*>(ep.pos + (size_t)(row % ep.period) * N + col0);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 p = __ldg(p4 + i);
            o4[i] = make_float4(v[4 * i] + p.x, v[4 * i + 1] + p.y, v[4 * i + 2] + p.z, v[4 * i + 3] + p.w);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
      }
    }
  }
  if (!ok) atomicExch(status, kEgStatusTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

template <int BN>
constexpr int eg_stages() {
  return BN == 256 ? 4 : 6;  // 192 KB of tiles either way
}

template <int BN>
size_t eg_smem_bytes() {
  return (size_t)eg_stages<BN>() * (kEgBM * kEgBK * 2 + BN * kEgBK * 2) + 1024;
}

template <typename T, int BN, int EPI>
void launch_t(const CUtensorMap& amap, const CUtensorMap& bmap, int M, int N, int K, const EncEpiArgs& ep,
              int* status, cudaStream_t s) {
  launch_pdl(k_enc_gemm<T, BN, eg_stages<BN>(), EPI>, dim3((M + kEgBM - 1) / kEgBM, N / BN), dim3(192),
             eg_smem_bytes<BN>(), s, amap, bmap, M, K, N, ep, status);
}

template <typename T, int BN>
void launch_bn(int epi, const CUtensorMap& amap, const CUtensorMap& bmap, int M, int N, int K, const EncEpiArgs& ep,
               int* status, cudaStream_t s) {
  switch (epi) {
    case kEpiQkv: launch_t<T, BN, kEpiQkv>(amap, bmap, M, N, K, ep, status, s); break;
    case kEpiGelu: launch_t<T, BN, kEpiGelu>(amap, bmap, M, N, K, ep, status, s); break;
    case kEpiResid: launch_t<T, BN, kEpiResid>(amap, bmap, M, N, K, ep, status, s); break;
    case kEpiGeluPos: launch_t<T, BN, kEpiGeluPos>(amap, bmap, M, N, K, ep, status, s); break;
    case kEpiSilu: launch_t<T, BN, kEpiSilu>(amap, bmap, M, N, K, ep, status, s); break;
    default: launch_t<T, BN, kEpiF32>(amap, bmap, M, N, K, ep, status, s); break;
  }
}

template <typename T, int BN, int EPI>
cudaError_t set_smem() {
  return cudaFuncSetAttribute(k_enc_gemm<T, BN, eg_stages<BN>(), EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)eg_smem_bytes<BN>());
}

template <typename T, int BN>
cudaError_t init_bn() {
  cudaError_t e;
  if ((e = set_smem<T, BN, kEpiQkv>()) != cudaSuccess) return e;
  if ((e = set_smem<T, BN, kEpiGelu>()) != cudaSuccess) return e;
  if ((e = set_smem<T, BN, kEpiResid>()) != cudaSuccess) return e;
  if ((e = set_smem<T, BN, kEpiGeluPos>()) != cudaSuccess) return e;
  if ((e = set_smem<T, BN, kEpiSilu>()) != cudaSuccess) return e;
  return set_smem<T, BN, kEpiF32>();
}

}  // namespace

cudaError_t init_enc_attn();

cudaError_t init_enc_kernels() {
  cudaError_t e;
  if ((e = init_bn<__nv_bfloat16, 128>()) != cudaSuccess) return e;
  if ((e = init_bn<__nv_bfloat16, 256>()) != cudaSuccess) return e;
  if ((e = init_bn<__half, 128>()) != cudaSuccess) return e;
  if ((e = init_bn<__half, 256>()) != cudaSuccess) return e;
  return init_enc_attn();
}

int enc_gemm_bn(int N) {
  if (N % 256 == 0) return 256;
  if (N % 128 == 0) return 128;
  return 0;
}

bool enc_make_map2(void* encode_fn, CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                   uint32_t box_rows) {
  if (encode_fn == nullptr || (reinterpret_cast<uintptr_t>(base) & 15) || (cols * 2) % 16 || box_rows > 256)
    return false;
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(encode_fn);
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kEgBK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool enc_make_map3(void* encode_fn, CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                   uint64_t chunks) {
  if (encode_fn == nullptr || (reinterpret_cast<uintptr_t>(base) & 15) || (cols * 2) % 16) return false;
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(encode_fn);
  const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)chunks};
  const cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)cols * 2 * rows};
  const cuuint32_t box[3] = {(cuuint32_t)kEgBK, 64, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void launch_enc_gemm(ActType at, int epi, const CUtensorMap& amap, const CUtensorMap& bmap, int bn, int M, int N,
                     int K, const EncEpiArgs& ep, int* status, cudaStream_t s) {
  if (at == kBF16) {
    if (bn == 256) launch_bn<__nv_bfloat16, 256>(epi, amap, bmap, M, N, K, ep, status, s);
    else launch_bn<__nv_bfloat16, 128>(epi, amap, bmap, M, N, K, ep, status, s);
  } else {
    if (bn == 256) launch_bn<__half, 256>(epi, amap, bmap, M, N, K, ep, status, s);
    else launch_bn<__half, 128>(epi, amap, bmap, M, N, K, ep, status, s);
  }
}

}  // namespace fmd
