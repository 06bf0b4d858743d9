// Prompt-embedding assembly on the GPU: `MossModel::splice_audio`
// (crates/fmd-core/src/model/mod.rs:134-180).
//
// The reference walks the prompt ids as alternating runs of text and audio
// placeholders, embeds each text run (`Qwen3::embed`, qwen3.rs:405-412),
// narrows each audio run out of the encoder output (converted to the
// activation dtype, mod.rs:141), and concatenates the parts. Here every prompt
// position is one row gather: the host turns the ids into one source code per
// position (>= 0: that vocabulary row of the embedding table; < 0: audio row
// -code - 1), and one kernel copies each row with 16-byte vectors from the
// table or from the audio embeddings straight into the caller's device buffer
// (for instance the engine's prompt arena). It is HBM-bound: H x 2 bytes read
// and written per position (+ 2x the read for f32 audio rows).
#include <algorithm>

#include "fmd_kernels.cuh"

namespace fmd {

namespace {

// grid-stride over rows; a CTA copies one row per iteration, each thread
// 8 elements (16 bytes of output) per vector
template <typename T>
__global__ void __launch_bounds__(128) k_splice(const int* __restrict__ src, long long n, const T* __restrict__ table,
                                                const void* __restrict__ audio, int audio_f32, int H,
                                                T* __restrict__ out) {
  const int nvec = H >> 3;
  for (long long r = blockIdx.x; r < n; r += gridDim.x) {
    const int code = __ldg(src + r);
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)r * H);
    if (code >= 0) {
      const uint4* s = reinterpret_cast<const uint4*>(table + (size_t)code * H);
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) dst[v] = __ldg(s + v);
    } else if (!audio_f32) {
      const uint4* s = reinterpret_cast<const uint4*>(static_cast<const T*>(audio) + (size_t)(-code - 1) * H);
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) dst[v] = __ldg(s + v);
    } else {
      const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(audio) + (size_t)(-code - 1) * H);
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        const float4 a = __ldg(s + 2 * v), b = __ldg(s + 2 * v + 1);
        dst[v] = make_uint4(Act<T>::pack2(a.x, a.y), Act<T>::pack2(a.z, a.w), Act<T>::pack2(b.x, b.y),
                            Act<T>::pack2(b.z, b.w));
      }
    }
  }
}

}  // namespace

void launch_splice(ActType at, const int* src, long long n, const void* table, const void* audio, bool audio_f32,
                   int H, void* out, cudaStream_t s) {
  if (n <= 0) return;
  const int grid = (int)std::min<long long>(n, 148LL * 16);
  if (at == kBF16)
    k_splice<__nv_bfloat16><<<grid, 128, 0, s>>>(src, n, (const __nv_bfloat16*)table, audio, audio_f32 ? 1 : 0, H,
                                                 (__nv_bfloat16*)out);
  else
    k_splice<__half><<<grid, 128, 0, s>>>(src, n, (const __half*)table, audio, audio_f32 ? 1 : 0, H, (__half*)out);
}

}  // namespace fmd
