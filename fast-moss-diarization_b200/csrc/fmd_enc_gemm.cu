// Projections of the audio tower on the 5th-generation tensor cores, with the
// elementwise work that follows each one fused into the epilogue:
// out[M][N] = epilogue(A[M][K] . W[N][K]^T + bias).
//
// The reference runs each as a dense candle matmul followed by separate
// broadcast_add / gelu_erf / silu / residual-add ops in the activation dtype
// (crates/fmd-core/src/model/whisper_encoder.rs:45-64, :88-100, :142-163;
// adaptor.rs:54-58; linear.rs:29-65). Here one persistent kernel per
// projection, one CTA per SM walking 128 x BN output tiles (tile t: feature
// block t / m_tiles, row block t % m_tiles, so the CTAs in flight share a
// weight tile in L2):
//  * warp 0 (one lane) streams A (activations) and W (weights) k-blocks as
//    16-bit K-major tiles by TMA with the 128-byte swizzle through a
//    STAGES-deep full/empty mbarrier ring that runs on across tiles;
//  * warp 1 allocates two BN-column f32 accumulators in tensor memory and,
//    the whole warp running the loop, its elected lane issues tcgen05.mma
//    (M = 128, N = BN, K = 16; four per k-block) into
//    accumulator i % 2, releasing each stage with tcgen05.commit and handing
//    the finished accumulator over with a commit to acc_full;
//  * warps 2-9 are the epilogue: warp w reads tensor-memory lanes
//    32 * (w % 4) ... (tile rows) for half (w - 2) / 4 of the columns, adds the
//    bias and applies the fused epilogue (q/k scaling, erf-GELU, SiLU, the
//    positional rows, or the residual add into the f32 residual stream) before
//    one store, then frees the accumulator (acc_empty). The epilogue of tile i
//    runs while the MMAs of tile i + 1 fill the other accumulator.
// The residual stream is kept in f32 (the reference rounds it to the
// activation dtype after every add); LayerNorm reads it in f32.
// Every wait is bounded; a timeout sets the status word, every role stops, the
// CTA waits (bounded) for its copies and MMAs in flight and frees its tensor
// memory before leaving.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>

#include "fmd_audio.cuh"

namespace fmd {

namespace {

constexpr int kEgBM = 128;
constexpr int kEgBK = 64;
constexpr int kEgThreads = 320;  // producer warp, MMA warp, 8 epilogue warps
constexpr uint32_t kEgWaitLimit = 1u << 24;
constexpr int kEgStatusTimeout = -110;
int g_sm_count = 148;

FMD_DEV float gelu_erf(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

// Bias + fused epilogue of 32 consecutive columns [col0, col0 + 32) of `row`.
template <typename T, int EPI>
FMD_DEV void epilogue32(const uint32_t (&r)[32], int row, int col0, int N, const EncEpiArgs& ep) {
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
      const float sc = col0 < ep.q_cols ? ep.scale_q : ep.scale;  // q_cols, scale_cols: multiples of 32
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= sc;
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

template <typename T, int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kEgThreads, 1)
    k_enc_gemm(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, int M, int K, int N,
               EncEpiArgs ep, int* __restrict__ status) {
  constexpr uint32_t A_BYTES = kEgBM * kEgBK * 2;
  constexpr uint32_t B_BYTES = BN * kEgBK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t tiles = (raw + 1023u) & ~1023u;  // swizzle atoms need 1024-byte alignment
  uint8_t* tiles_p = smem_raw + (tiles - raw);
  const int m_tiles = (M + kEgBM - 1) / kEgBM;
  const int n_tiles = m_tiles * (N / BN);
  const int nk = K / kEgBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one arrival per epilogue warp
    }
    mbar_init(&mma_done, 1);
    abort_s = 0;
    fence_barrier_init();
  }
  // Tensor memory only after the dependency wait: the previous kernel has
  // then finished, so none of its CTAs can hold the columns this CTA needs
  // while it waits for this one.
  griddep_wait();  // A (and the residual stream) come from earlier kernels
  griddep_launch();  // only after the wait: see griddep_launch
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  volatile int* abort_v = &abort_s;

  // Parity waits never alias: the ring and the two accumulators are each
  // waited on in use order by one role, which has already seen the previous
  // use of the same slot complete.
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&amap);
      prefetch_tmap(&bmap);
      int g = 0;  // k-block position in the ring across tiles
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
        const int row0 = (t % m_tiles) * kEgBM, n0 = (t / m_tiles) * BN;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int st = g % STAGES;
          if (g >= STAGES &&
              (*abort_v || !mbar_wait_bounded(&empty[st], ((g / STAGES) + 1) & 1, kEgWaitLimit))) {
            ok = false;
            break;
          }
          uint8_t* a = tiles_p + st * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[st], STAGE_BYTES);
          tma_load_2d(a, &amap, kb * kEgBK, row0, &full[st]);
          tma_load_2d(a + A_BYTES, &bmap, kb * kEgBK, n0, &full[st]);
        }
      }
      if (!ok) *abort_v = 1;
      // copies still in flight land before the CTA retires (bounded)
      for (int j = g - STAGES > 0 ? g - STAGES : 0; j < g; ++j)
        mbar_wait_bounded(&full[j % STAGES], (j / STAGES) & 1, kEgWaitLimit);
    }
  } else if (warp == 1) {
    {
      // the whole warp runs the loop; the elected lane issues (elect_one)
      constexpr uint32_t idesc = umma_idesc_f16(Act<T>::kIsBf16, kEgBM, BN);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (i >= 2 && (*abort_v || !mbar_wait_warp(&acc_empty[buf], ((i >> 1) - 1) & 1, kEgWaitLimit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int st = g % STAGES;
          if (*abort_v || !mbar_wait_warp(&full[st], (g / STAGES) & 1, kEgWaitLimit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = tiles + st * STAGE_BYTES, b = a + A_BYTES;
          if (elect_one()) {
#pragma unroll
            for (int j = 0; j < kEgBK / 16; ++j)
              umma_f16(acc, umma_desc_sw128(a + j * 32), umma_desc_sw128(b + j * 32), idesc, (kb | j) != 0);
            umma_commit(&empty[st]);  // the stage is free once these MMAs have read it
          }
          __syncwarp();
        }
        if (ok && elect_one()) umma_commit(&acc_full[buf]);
        __syncwarp();
      }
      if (!ok) *abort_v = 1;
      if (elect_one()) umma_commit(&mma_done);  // every MMA issued so far has completed when this fires
      __syncwarp();
      mbar_wait_warp(&mma_done, 0, kEgWaitLimit);
    }
  } else {
    const int q = warp & 3, half = (warp - 2) >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    int i = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
      const int buf = i & 1;
      // the tensor-memory loads below are warp-wide: the warp goes on only
      // if the wait passed for all of its lanes
      const bool got = !*abort_v && mbar_wait_bounded(&acc_full[buf], (i >> 1) & 1, kEgWaitLimit);
      if (!__all_sync(0xffffffffu, got)) {
        *abort_v = 1;
        break;
      }
      tc_fence_after();
      const int row = (t % m_tiles) * kEgBM + q * 32 + lane;
      const int n0 = (t / m_tiles) * BN + half * (BN / 2);
#pragma unroll 1
      for (int c = 0; c < BN / 64; ++c) {
        uint32_t r[32];
        tmem_ld32(lane_base + (uint32_t)(buf * BN + half * (BN / 2) + c * 32), r);
        tmem_ld_wait();
        if (row < M) epilogue32<T, EPI>(r, row, n0 + c * 32, N, ep);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && abort_s) atomicExch(status, kEgStatusTimeout);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
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
  const int n_tiles = (M + kEgBM - 1) / kEgBM * (N / BN);
  launch_pdl(k_enc_gemm<T, BN, eg_stages<BN>(), EPI>, dim3(std::min(n_tiles, g_sm_count)), dim3(kEgThreads),
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
  int dev = 0, sms = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  g_sm_count = sms > 0 ? sms : 148;
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
