// Projections of a mixed (prefill-carrying) step on the 5th-generation tensor
// cores: out[split][rows][N] (f32) = X[rows][K] . W[N][K]^T.
//
// The reference runs these as one GEMM per projection over the chunk's rows
// (crates/fmd-core/src/model/linear.rs:29-65 through qwen3.rs:213-338). Here:
//  * X is a 16-bit K-major tile fetched by TMA with the 128-byte swizzle
//    through a tensor map over the activation buffer. Dense W likewise, from
//    the projection's 16-bit weights. Q8_0 W is fetched as its int8 tile
//    (TMA over the int8 [N][K] matrix, 64-byte rows, no swizzle) and
//    dequantised in shared memory: the four epilogue warps, idle until the
//    accumulator is ready, turn each k-block's BN x 64 int8 values and their
//    f16 block scales into q * d rounded to the activation type, written in
//    the 128-byte-swizzled K-major layout the MMA reads, one stage ahead of
//    the MMA issuer. The int8 weights are the only copy in HBM the GEMM
//    reads (no 16-bit expansion);
//  * a CTA owns a 128-row x BN-feature tile (BN = 128 or 256) and a K range
//    (split-K over gridDim.z when the feature count alone leaves SMs idle).
//    Warp 0 (one lane) runs a STAGES-deep full/empty mbarrier ring of TMA
//    loads, warp 1 allocates BN tensor-memory columns and its elected lane
//    (the whole warp running the loop) issues tcgen05.mma (M = 128, N = BN, K = 16; four per 64-wide k-block) and
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

// One converter lane's 16 int8 weights (16 bytes) times their block scale,
// rounded to the activation type: 8 packed words, k order preserved.
template <typename T>
FMD_DEV void dequant16(const int4 q, float d, uint32_t (&o)[8]) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(&q);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t v = w[j] ^ 0x80808080u;  // biased bytes q + 128
    float f[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = (__int_as_float(__byte_perm(v, 0x4B000000u, 0x7440u | i)) - 8388736.f) * d;
    o[2 * j] = Act<T>::pack2(f[0], f[1]);
    o[2 * j + 1] = Act<T>::pack2(f[2], f[3]);
  }
}

template <typename T, int BN, int STAGES, bool Q8>
__global__ void __launch_bounds__(192, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
              const int* __restrict__ n_rows_ptr, int K, int N, float* __restrict__ out, size_t split_stride,
              int* __restrict__ status, const uint16_t* __restrict__ wd) {
  constexpr uint32_t A_BYTES = kTcBM * kTcBK * 2;
  constexpr uint32_t B_BYTES = BN * kTcBK * 2;
  constexpr uint32_t Q_BYTES = Q8 ? BN * kTcBK : 0;  // the int8 tile of a Q8_0 stage
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES + Q_BYTES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], conv[STAGES], done;
  __shared__ uint32_t tmem_base_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t tiles = (raw + 1023u) & ~1023u;  // swizzle atoms need 1024-byte alignment
  uint8_t* tiles_p = smem_raw + (tiles - raw);

  griddep_wait();  // X and the row count come from earlier kernels
  griddep_launch();  // only after the wait: see griddep_launch
  const int n_rows = *n_rows_ptr;
  const int row0 = blockIdx.x * kTcBM;
  if (row0 >= n_rows) return;  // whole CTA, before any barrier or tensor memory exists
  const int n0 = blockIdx.y * BN;
  const int klen = K / gridDim.z, kbeg = blockIdx.z * klen, nk = klen / kTcBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 4);  // Q8_0: one arrival per converter warp
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
        mbar_arrive_expect_tx(&full[st], A_BYTES + (Q8 ? Q_BYTES : B_BYTES));
        tma_load_2d(a, &amap, kbeg + kb * kTcBK, row0, &full[st]);
        tma_load_2d(a + A_BYTES + (Q8 ? B_BYTES : 0), &bmap, kbeg + kb * kTcBK, n0, &full[st]);
        issued = kb + 1;
      }
      if (!ok) {
        // the MMA side stopped consuming: let the copies in flight land
        for (int kb = issued - STAGES > 0 ? issued - STAGES : 0; kb < issued; ++kb)
          mbar_wait_bounded(&full[kb % STAGES], (kb / STAGES) & 1, kTcWaitLimit);
      }
    }
  } else if (warp == 1) {
    {
      // the whole warp runs the loop; the elected lane issues (elect_one)
      constexpr uint32_t idesc = umma_idesc_f16(Act<T>::kIsBf16, kTcBM, BN);
      for (int kb = 0; kb < nk; ++kb) {
        const int st = kb % STAGES;
        if (!mbar_wait_warp(&full[st], (kb / STAGES) & 1, kTcWaitLimit) ||
            (Q8 && !mbar_wait_warp(&conv[st], (kb / STAGES) & 1, kTcWaitLimit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = tiles + st * STAGE_BYTES, b = a + A_BYTES;
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < kTcBK / 16; ++j)
            umma_f16(tmem, umma_desc_sw128(a + j * 32), umma_desc_sw128(b + j * 32), idesc, (kb | j) != 0);
          umma_commit(&empty[st]);  // the stage is free once these MMAs have read it
        }
        __syncwarp();
      }
      if (elect_one()) umma_commit(&done);  // also after an abort: the epilogue must not wait forever
      __syncwarp();
    }
  } else {
    if constexpr (Q8) {
      // converters: warp cw turns rows cw*8 + 32*i + (lane >> 2) of each
      // stage's int8 tile into the swizzled 16-bit B tile; lane & 3 picks 16
      // consecutive k (one Q8_0 block half), so a lane needs one scale. The
      // stage's previous B tile is free: its new copy landed only after the
      // MMAs that read the old one completed (the producer waited on empty).
      const int cw = warp - 2, c = lane & 3;
      const int KB = K / 32;
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int st = kb % STAGES;
        // scales of this k-block first: their latency overlaps the copy's
        float dsc[BN / 32];
#pragma unroll
        for (int i = 0; i < BN / 32; ++i) {
          const int r = cw * 8 + 32 * i + (lane >> 2);
          dsc[i] = h2f_bits(__ldg(wd + (size_t)(n0 + r) * KB + (kbeg + kb * kTcBK) / 32 + (c >> 1)));
        }
        if (!mbar_wait_bounded(&full[st], (kb / STAGES) & 1, kTcWaitLimit)) {
          ok = false;
          break;
        }
        const uint8_t* qt = tiles_p + st * STAGE_BYTES + A_BYTES + B_BYTES;
        uint8_t* bt = tiles_p + st * STAGE_BYTES + A_BYTES;
#pragma unroll 4
        for (int i = 0; i < BN / 32; ++i) {
          const int r = cw * 8 + 32 * i + (lane >> 2);
          const int4 q = *reinterpret_cast<const int4*>(qt + r * kTcBK + c * 16);
          uint32_t o[8];
          dequant16<T>(q, dsc[i], o);
          // 16-byte chunk j of row r sits at chunk j ^ (r % 8) (128-byte swizzle)
          uint8_t* row = bt + r * 128;
          *reinterpret_cast<int4*>(row + (((2 * c) ^ (r & 7)) << 4)) = make_int4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<int4*>(row + (((2 * c + 1) ^ (r & 7)) << 4)) = make_int4(o[4], o[5], o[6], o[7]);
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // visible to tcgen05.mma
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[st]);
      }
    }
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
  if (!ok) report_timeout(status, kSiteGemmTc);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

template <int BN, bool Q8>
constexpr int tc_stages() {
  // 192 KB of tiles for 16-bit W; Q8_0 stages also hold the int8 tile
  return Q8 ? (BN == 256 ? 3 : 5) : (BN == 256 ? 4 : 6);
}

template <int BN, bool Q8>
size_t tc_smem_bytes() {
  return (size_t)tc_stages<BN, Q8>() * (kTcBM * kTcBK * 2 + BN * kTcBK * 2 + (Q8 ? BN * kTcBK : 0)) + 1024;
}

template <typename T, int BN, bool Q8>
void launch_gemm_tc_t(const CUtensorMap& amap, const TcLinear& W, const int* n_rows_ptr, int max_rows, float* out,
                      size_t split_stride, int* status, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((max_rows + kTcBM - 1) / kTcBM, W.N / BN, W.split);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = tc_smem_bytes<BN, Q8>();
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k_gemm_tc<T, BN, tc_stages<BN, Q8>(), Q8>, amap, W.wmap, n_rows_ptr, W.K, W.N, out,
                     split_stride, status, W.d);
}

template <typename T>
cudaError_t init_gemm_tc_t() {
  for (cudaError_t e : {
           cudaFuncSetAttribute(k_gemm_tc<T, 128, tc_stages<128, false>(), false>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_bytes<128, false>()),
           cudaFuncSetAttribute(k_gemm_tc<T, 256, tc_stages<256, false>(), false>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_bytes<256, false>()),
           cudaFuncSetAttribute(k_gemm_tc<T, 128, tc_stages<128, true>(), true>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_bytes<128, true>()),
           cudaFuncSetAttribute(k_gemm_tc<T, 256, tc_stages<256, true>(), true>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_bytes<256, true>())})
    if (e != cudaSuccess) return e;
  return cudaSuccess;
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

// 2D map over a row-major int8 [outer][inner] matrix, box {64, box_outer},
// no swizzle (the Q8_0 weights of the tensor-core GEMM).
bool tc_make_map_i8(void* encode_fn, CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
                    uint32_t box_outer) {
  if (encode_fn == nullptr || (reinterpret_cast<uintptr_t>(base) & 15) || inner % 16 || box_outer > 256)
    return false;
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(encode_fn);
  const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  const cuuint64_t strides[1] = {(cuuint64_t)inner};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBK, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
  if (!W.ok || (W.bn != 128 && W.bn != 256) || W.K % (kTcBK * W.split) || (W.q8 && W.d == nullptr)) return false;
#define FMD_TC(T, Q8)                                                                                      \
  if (W.bn == 256) launch_gemm_tc_t<T, 256, Q8>(amap, W, n_rows_ptr, max_rows, out, split_stride, status, s); \
  else launch_gemm_tc_t<T, 128, Q8>(amap, W, n_rows_ptr, max_rows, out, split_stride, status, s);
  if (at == kBF16) {
    if (W.q8) { FMD_TC(__nv_bfloat16, true) } else { FMD_TC(__nv_bfloat16, false) }
  } else {
    if (W.q8) { FMD_TC(__half, true) } else { FMD_TC(__half, false) }
  }
#undef FMD_TC
  return true;
}

}  // namespace fmd
