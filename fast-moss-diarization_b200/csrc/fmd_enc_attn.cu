// Dense bidirectional self-attention of the Whisper encoder on the
// 5th-generation tensor cores (flash attention, head_dim 64).
//
// Computes `Attention::forward` of crates/fmd-core/src/model/whisper_encoder.rs:45-64
// for every 30 s chunk and head: softmax(q k^T) v over all `frames` positions
// of the chunk, no mask (every chunk is exactly 30 s, whisper_encoder.rs:1-5).
// q and k arrive pre-scaled by head_dim^-1/4 (the QKV GEMM's epilogue), as in
// the reference (whisper_encoder.rs:52-55); q also carries the factor log2(e),
// so S = q k^T is the score in the exp2 domain.
//
// One CTA per (128-query tile, head, chunk); two CTAs fit on an SM:
//  * warp 0 (one lane): TMA loads through a 3D tensor map
//    [chunk][frame][q | k | v columns] with box {64, 64, 1}, so a tile that runs
//    past the chunk's last frame is zero-filled rather than reading the next
//    chunk: the query tile (two boxes) and, per 64-key tile, K and V (8 KB
//    each, 128-byte swizzle) into a 3-stage full/empty ring;
//  * warp 1 (the whole warp, one elected lane issuing): tcgen05.mma with f32 accumulators in tensor memory:
//    S_j = Q K_j^T (M 128, N 64 keys, K 64 dims; S double-buffered), then
//    O += P_j V_j (M 128, N 64 dims, K 64 keys; V read MN-major from its tile);
//  * warps 2-5 (one thread per query row = tensor-memory lane): online softmax
//    in the exp2 domain with a lazily moved reference maximum (O is rescaled in
//    tensor memory only when a row maximum exceeds it by more than 2^8); keys
//    past the chunk end are masked; P_j goes as 16-bit values into a
//    double-buffered 128-byte-swizzled shared tile (the A operand of PV). At the
//    end each thread divides its row of O by the row sum and stores ctx.
// Every wait is bounded; a timeout sets the status word, stops issuing work,
// waits (bounded) for copies and MMAs in flight and frees tensor memory.
#include <cuda.h>
#include <float.h>
#include <math.h>

#include "fmd_audio.cuh"

namespace fmd {

namespace {

constexpr int kEaStages = 3;
constexpr int kEaBox = 8192;               // one 64 x 64 box of 16-bit values
constexpr int kEaQBytes = 2 * kEaBox;      // 128 query rows x 64 dims
constexpr int kEaKvBytes = 2 * kEaBox;     // K + V of one 64-key tile
constexpr int kEaPBytes = 16384;           // one P buffer: 128 rows x 64 keys
constexpr uint32_t kEaWaitLimit = 1u << 24;
constexpr int kEaStatusTimeout = -110;
constexpr int kEaTmemCols = 256;           // S0 [0, 64), S1 [64, 128), O [128, 192)
constexpr float kEaRescale = 8.f;          // log2 headroom before the reference maximum moves

FMD_DEV void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n" ::
          "r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// MN-major operand with the 128-byte swizzle: 64 contiguous MN elements per
// 128-byte row, one row per K index, 8-row atoms 1024 bytes apart along K.
FMD_DEV uint64_t desc_sw128_mn(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(kEaBox >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// 2^x with the MUFU approximation (PTX ex2.approx.ftz.f32: relative error
// below 2^-22, 2^-inf = 0), ample for probabilities stored as 16-bit values.
FMD_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

FMD_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

template <typename T>
__global__ void __launch_bounds__(192, 2)
    k_enc_attn(const __grid_constant__ CUtensorMap map, int frames, int D, T* __restrict__ ctx,
               int* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full, kv_full[kEaStages], kv_empty[kEaStages], s_full[2], s_empty[2],
      p_full[2], p_empty[2], o_full, o_final, mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_p = smem_raw + (base - raw);
  const uint32_t q_s = base, p_s = base + kEaQBytes, kv_s = p_s + 2 * kEaPBytes;
  uint8_t* p_sp = base_p + kEaQBytes;

  const int qt = blockIdx.x, h = blockIdx.y, chunk = blockIdx.z;
  const int q0 = qt * 128;
  const int n_tiles = (frames + 63) / 64;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kEaStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 128);
      mbar_init(&p_full[s], 128);
      mbar_init(&p_empty[s], 1);
    }
    mbar_init(&o_full, 1);
    mbar_init(&o_final, 1);
    mbar_init(&mma_done, 1);
    abort_s = 0;
    fence_barrier_init();
  }
  // Tensor memory only after the dependency wait: the previous kernel has
  // then finished, so none of its CTAs can hold the columns this CTA needs
  // while it waits for this one.
  griddep_wait();  // qkv comes from the previous kernel
  griddep_launch();  // only after the wait: see griddep_launch
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, kEaTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  volatile int* abort_v = &abort_s;

  // Parity waits never alias: each waits for a phase whose successor needs
  // work that the waiting role itself releases later, and whose predecessor
  // has completed (MMAs of one thread complete in issue order, and s_full(j)
  // fires only after PV_{j-2}); the final O has a barrier of its own.
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&map);
      const int xq = h * 64, xk = D + h * 64, xv = 2 * D + h * 64;
      mbar_arrive_expect_tx(&q_full, kEaQBytes);
      tma_load_3d(base_p, &map, xq, q0, chunk, &q_full);
      tma_load_3d(base_p + kEaBox, &map, xq, q0 + 64, chunk, &q_full);
      int issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % kEaStages;
        if (j >= kEaStages &&
            (*abort_v || !mbar_wait_bounded(&kv_empty[st], ((j / kEaStages) - 1) & 1, kEaWaitLimit))) {
          *abort_v = 1;
          break;
        }
        uint8_t* dst = base_p + kEaQBytes + 2 * kEaPBytes + st * kEaKvBytes;
        mbar_arrive_expect_tx(&kv_full[st], kEaKvBytes);
        tma_load_3d(dst, &map, xk, j * 64, chunk, &kv_full[st]);
        tma_load_3d(dst + kEaBox, &map, xv, j * 64, chunk, &kv_full[st]);
        issued = j + 1;
      }
      mbar_wait_bounded(&q_full, 0, kEaWaitLimit);
      for (int j = issued > kEaStages ? issued - kEaStages : 0; j < issued; ++j)
        mbar_wait_bounded(&kv_full[j % kEaStages], (j / kEaStages) & 1, kEaWaitLimit);
    }
  } else if (warp == 1) {
    {
      // the whole warp runs the loop; the elected lane issues (elect_one)
      constexpr bool kBf = Act<T>::kIsBf16;
      constexpr uint32_t idesc_s = umma_idesc_f16(kBf, 128, 64);
      constexpr uint32_t idesc_o = umma_idesc_f16(kBf, 128, 64) | (1u << 16);  // B (V) MN-major
      const uint32_t o_tmem = tmem + 128;
      auto pv = [&](int i) -> bool {
        const int pb = i & 1;
        if (*abort_v || !mbar_wait_warp(&p_full[pb], (i >> 1) & 1, kEaWaitLimit)) return false;
        tc_fence_after();
        const uint32_t v = kv_s + (i % kEaStages) * kEaKvBytes + kEaBox;
        const uint32_t pa = p_s + pb * kEaPBytes;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(o_tmem, umma_desc_sw128(pa + kk * 32), desc_sw128_mn(v + kk * 2048), idesc_o, (i | kk) != 0);
          umma_commit(&o_full);
          umma_commit(&p_empty[pb]);
          umma_commit(&kv_empty[i % kEaStages]);
        }
        __syncwarp();
        return true;
      };
      bool ok = !*abort_v && mbar_wait_warp(&q_full, 0, kEaWaitLimit);
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j % kEaStages, sb = j & 1;
        if (*abort_v || !mbar_wait_warp(&kv_full[st], (j / kEaStages) & 1, kEaWaitLimit) ||
            (j >= 2 && !mbar_wait_warp(&s_empty[sb], ((j >> 1) - 1) & 1, kEaWaitLimit))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k = kv_s + st * kEaKvBytes;
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + sb * 64, umma_desc_sw128(q_s + kk * 32), umma_desc_sw128(k + kk * 32), idesc_s, kk != 0);
          umma_commit(&s_full[sb]);
        }
        __syncwarp();
        if (j >= 1 && !pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) ok = pv(n_tiles - 1);
      if (ok && elect_one()) umma_commit(&o_final);
      __syncwarp();
      if (!ok) *abort_v = 1;
      if (elect_one()) umma_commit(&mma_done);
      __syncwarp();
      mbar_wait_warp(&mma_done, 0, kEaWaitLimit);
    }
  } else {
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(q4 * 32) << 16);
    const uint32_t o_addr = lane_addr + 128;
    float m_ref = -INFINITY, l = 0.f;
    // tcgen05.ld / st are warp-wide (.sync.aligned): every branch around them
    // is taken by the whole warp. A wait counts as passed only when it passed
    // for all 32 lanes, so no lane goes on to a tensor-memory access alone.
    auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
      const bool mine = !*abort_v && mbar_wait_bounded(bar, parity, kEaWaitLimit);
      return __all_sync(0xffffffffu, mine);
    };
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int sb = j & 1;
      if (!wwait(&s_full[sb], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[64];
      {
        uint32_t v0[32], v1[32];
        tmem_ld32(lane_addr + sb * 64, v0);
        tmem_ld32(lane_addr + sb * 64 + 32, v1);
        tmem_ld_wait();
#pragma unroll
        for (int i2 = 0; i2 < 32; ++i2) {
          s[i2] = __uint_as_float(v0[i2]);
          s[32 + i2] = __uint_as_float(v1[i2]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      const int valid = frames - j * 64;  // keys of this tile inside the chunk (>= 1)
      if (valid < 64) {  // only the chunk's last tile (uniform across the CTA)
#pragma unroll
        for (int c = 0; c < 64; ++c) s[c] = c < valid ? s[c] : -INFINITY;
      }
      float m4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int c = 4; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], s[c]);
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      // a row moves its reference maximum past 2^8 of headroom; the rescale
      // of O in tensor memory is warp-wide, so the warp does it when any of
      // its rows moves and the others scale by 1 (their O is unchanged)
      bool moves = false;
      if (j == 0)
        m_ref = mx;  // finite: key 0 is inside the chunk
      else
        moves = mx > m_ref + kEaRescale;
      if (__any_sync(0xffffffffu, moves)) {
        if (!wwait(&o_full, (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float f = moves ? ex2(m_ref - mx) : 1.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld32(o_addr + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i2 = 0; i2 < 32; ++i2) v[i2] = __float_as_uint(__uint_as_float(v[i2]) * f);
          tmem_st32(o_addr + c * 32, v);
        }
        tmem_st_wait();
        if (moves) {
          l *= f;
          m_ref = mx;
        }
      }
      float p4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        s[c] = ex2(s[c] - m_ref);
        p4[c & 3] += s[c];
      }
      l += (p4[0] + p4[1]) + (p4[2] + p4[3]);
      if (j >= 2 && !wwait(&p_empty[sb], ((j - 2) >> 1) & 1)) {
        ok = false;
        break;
      }
      uint8_t* prow = p_sp + sb * kEaPBytes + row * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 u;
        u.x = Act<T>::pack2(s[8 * c + 0], s[8 * c + 1]);
        u.y = Act<T>::pack2(s[8 * c + 2], s[8 * c + 3]);
        u.z = Act<T>::pack2(s[8 * c + 4], s[8 * c + 5]);
        u.w = Act<T>::pack2(s[8 * c + 6], s[8 * c + 7]);
        *reinterpret_cast<uint4*>(prow + ((c ^ (row & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    if (ok && !wwait(&o_final, 0)) ok = false;
    if (!ok) *abort_v = 1;
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l;
      const int qi = q0 + row;
      T* dst = ctx + ((size_t)chunk * frames + qi) * D + h * 64;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[32];
        tmem_ld32(o_addr + c * 32, v);
        tmem_ld_wait();
        if (qi < frames) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint4 u;
            u.x = Act<T>::pack2(__uint_as_float(v[8 * q8 + 0]) * inv, __uint_as_float(v[8 * q8 + 1]) * inv);
            u.y = Act<T>::pack2(__uint_as_float(v[8 * q8 + 2]) * inv, __uint_as_float(v[8 * q8 + 3]) * inv);
            u.z = Act<T>::pack2(__uint_as_float(v[8 * q8 + 4]) * inv, __uint_as_float(v[8 * q8 + 5]) * inv);
            u.w = Act<T>::pack2(__uint_as_float(v[8 * q8 + 6]) * inv, __uint_as_float(v[8 * q8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + 8 * q8) = u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && abort_s) atomicExch(status, kEaStatusTimeout);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kEaTmemCols);
  }
}

size_t enc_attn_smem_bytes() { return 1024 + kEaQBytes + 2 * kEaPBytes + kEaStages * kEaKvBytes; }

}  // namespace

cudaError_t init_enc_attn() {
  const int bytes = (int)enc_attn_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(k_enc_attn<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_enc_attn<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

void launch_enc_attn(ActType at, const CUtensorMap& qkv_map, int n_chunks, int frames, int D, int heads, void* ctx,
                     int* status, cudaStream_t s) {
  const dim3 grid((frames + 127) / 128, heads, n_chunks);
  const size_t smem = enc_attn_smem_bytes();
  if (at == kBF16)
    launch_pdl(k_enc_attn<__nv_bfloat16>, grid, dim3(192), smem, s, qkv_map, frames, D, (__nv_bfloat16*)ctx, status);
  else
    launch_pdl(k_enc_attn<__half>, grid, dim3(192), smem, s, qkv_map, frames, D, (__half*)ctx, status);
}

}  // namespace fmd
