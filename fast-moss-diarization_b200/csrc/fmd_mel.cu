// Whisper log-mel frontend on the GPU (`MelFrontend::log_mel`,
// crates/fmd-core/src/audio/mel.rs:84-133) behind include/fmd_audio.h.
//
// The reference runs a 400-point real FFT per frame on the host (realfft, f32,
// rayon over chunks). Here the short-time transform is a direct DFT against a
// precomputed basis, evaluated in f64 on the GPU:
//  * k_mel_frames: one CTA per (32 consecutive frames, chunk). The samples the
//    32 frames cover (31 x hop + n_fft of them, reflect-indexed at the window
//    edges as np.pad(mode="reflect") does, mel.rs:141-156) are staged in
//    shared memory as f64; thread k owns frequency bin k and accumulates
//    sum_n x[n] w[n] cos / sin(2 pi k n / N) for all 32 frames (the periodic
//    Hann window w is folded into the basis, which each thread reads once per
//    n for 32 frames); the power spectrum goes to shared memory, then each
//    (mel band, frame) output sums its filter's non-zero span, takes
//    log10(max(., 1e-10)) and is written in the [n_mels][frames] layout; the
//    chunk's peak is folded in with an atomic max;
//  * k_mel_finish: (max(v, peak - 8) + 4) / 4 over the chunk (mel.rs:119-131).
// The basis and the filterbank are built on the host exactly as mel.rs builds
// them (window in f64 cast to f32, filterbank in f32 arithmetic).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "../../include/fmd_audio.h"
#include "fmd_common.cuh"

namespace {

constexpr int kMelFt = 32;       // frames per CTA
constexpr int kMelThreads = 256; // >= frequency bins

// Order-preserving map of an f32 to an unsigned key (larger value, larger key).
__device__ __forceinline__ unsigned f2key(float f) {
  const unsigned b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(unsigned k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ long long reflect(long long i, long long len) {
  if (len <= 1) return 0;
  const long long period = 2 * (len - 1);
  long long r = i % period;
  if (r < 0) r += period;
  return r >= len ? period - r : r;
}

__global__ void __launch_bounds__(kMelThreads) k_mel_frames(const float* __restrict__ samples, int n_samples,
                                                            int n_frames, int hop, int n_fft, int n_freq,
                                                            const double* __restrict__ basis,
                                                            const float* __restrict__ fb,
                                                            const int2* __restrict__ span, int n_mels,
                                                            float* __restrict__ out, unsigned* __restrict__ peak) {
  extern __shared__ double smem_d[];
  const int win = (kMelFt - 1) * hop + n_fft;
  double* xs = smem_d;               // [win]
  double* pw = smem_d + win;         // [kMelFt][n_freq]
  __shared__ unsigned blk_peak;
  const int chunk = blockIdx.y, t0 = blockIdx.x * kMelFt;
  const float* x = samples + (size_t)chunk * n_samples;
  const long long origin = (long long)t0 * hop - n_fft / 2;
  if (threadIdx.x == 0) blk_peak = 0u;
  for (int i = threadIdx.x; i < win; i += blockDim.x) xs[i] = (double)__ldg(x + reflect(origin + i, n_samples));
  __syncthreads();

  const int k = threadIdx.x;
  if (k < n_freq) {
    double re[kMelFt], im[kMelFt];
#pragma unroll
    for (int f = 0; f < kMelFt; ++f) re[f] = im[f] = 0.0;
    const double* bre = basis + k;                   // [n][0 .. n_freq): w[n] cos
    const double* bim = basis + (size_t)n_fft * n_freq + k;  // [n][0 .. n_freq): w[n] sin
#pragma unroll 2
    for (int n = 0; n < n_fft; ++n) {
      const double c = __ldg(bre + (size_t)n * n_freq), s = __ldg(bim + (size_t)n * n_freq);
#pragma unroll
      for (int f = 0; f < kMelFt; ++f) {
        const double v = xs[f * hop + n];
        re[f] = fma(v, c, re[f]);
        im[f] = fma(v, s, im[f]);
      }
    }
#pragma unroll
    for (int f = 0; f < kMelFt; ++f) pw[f * n_freq + k] = re[f] * re[f] + im[f] * im[f];
  }
  __syncthreads();

  float local = -INFINITY;
  for (int i = threadIdx.x; i < n_mels * kMelFt; i += blockDim.x) {
    const int m = i / kMelFt, f = i % kMelFt;
    if (t0 + f >= n_frames) continue;
    const int2 sp = span[m];
    double acc = 0.0;
    for (int j = sp.x; j < sp.x + sp.y; ++j) acc = fma((double)__ldg(fb + (size_t)m * n_freq + j), pw[f * n_freq + j], acc);
    const float v = log10f(fmaxf((float)acc, 1e-10f));
    out[((size_t)chunk * n_mels + m) * n_frames + t0 + f] = v;
    local = fmaxf(local, v);
  }
  local = fmd::warp_max(local);
  if ((threadIdx.x & 31) == 0 && local > -INFINITY) atomicMax(&blk_peak, f2key(local));
  __syncthreads();
  if (threadIdx.x == 0 && blk_peak != 0u) atomicMax(peak + chunk, blk_peak);
}

__global__ void k_mel_finish(float* __restrict__ out, const unsigned* __restrict__ peak, size_t per_chunk,
                             size_t total) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const float floor_v = key2f(peak[i / per_chunk]) - 8.f;
    out[i] = (fmaxf(out[i], floor_v) + 4.f) / 4.f;
  }
}

// ---- host: window, basis and filterbank exactly as mel.rs builds them ----

// Periodic Hann (mel.rs:158-165): computed in f64, stored as f32.
std::vector<float> hann_periodic(int n) {
  std::vector<float> w(n);
  for (int i = 0; i < n; ++i) {
    const double x = 2.0 * M_PI * (double)i / (double)n;
    w[i] = (float)(0.5 - 0.5 * std::cos(x));
  }
  return w;
}

// Slaney mel scale (mel.rs:167-181), f32 arithmetic.
float hz_to_mel(float freq) {
  const float f_sp = 200.0f / 3.0f, min_log_hz = 1000.0f, min_log_mel = min_log_hz / f_sp;
  const float logstep = std::log(6.4f) / 27.0f;
  return freq >= min_log_hz ? min_log_mel + std::log(freq / min_log_hz) / logstep : freq / f_sp;
}

float mel_to_hz(float mel) {
  const float f_sp = 200.0f / 3.0f, min_log_hz = 1000.0f, min_log_mel = min_log_hz / f_sp;
  const float logstep = std::log(6.4f) / 27.0f;
  return mel >= min_log_mel ? min_log_hz * std::exp(logstep * (mel - min_log_mel)) : f_sp * mel;
}

// Dense (n_mels x n_freq) Slaney-normalised triangles (mel.rs:183-240); each
// filter keeps its first contiguous run of positive weights.
std::vector<float> filter_bank(int n_freq, int n_mels, float f_min, float f_max, float sample_rate,
                               std::vector<std::pair<int, int>>* spans) {
  std::vector<float> freqs(n_freq);
  for (int i = 0; i < n_freq; ++i) freqs[i] = (float)i * (sample_rate / 2.0f) / (float)(n_freq - 1);
  const float mel_min = hz_to_mel(f_min), mel_max = hz_to_mel(f_max);
  std::vector<float> pts(n_mels + 2);
  for (int i = 0; i < n_mels + 2; ++i)
    pts[i] = mel_to_hz(mel_min + (mel_max - mel_min) * (float)i / (float)(n_mels + 1));
  std::vector<float> fb((size_t)n_mels * n_freq, 0.f);
  if (spans) spans->assign(n_mels, {0, 0});
  for (int m = 0; m < n_mels; ++m) {
    const float left = pts[m], center = pts[m + 1], right = pts[m + 2];
    const float enorm = 2.0f / (right - left);
    int start = -1, len = 0;
    for (int k = 0; k < n_freq; ++k) {
      const float lower = (freqs[k] - left) / (center - left);
      const float upper = (right - freqs[k]) / (right - center);
      const float w = std::max(std::min(lower, upper), 0.0f) * enorm;
      if (w > 0.0f) {
        if (start < 0) start = k;
        fb[(size_t)m * n_freq + k] = w;
        ++len;
      } else if (start >= 0) {
        break;
      }
    }
    if (spans) (*spans)[m] = {start < 0 ? 0 : start, len};
  }
  return fb;
}

bool cfg_ok(const fmd_feature_config& c) {
  return c.feature_size >= 1 && c.sampling_rate >= 1 && c.hop_length >= 1 && c.n_fft >= 2 && c.n_samples >= 1 &&
         c.nb_max_frames == c.n_samples / c.hop_length && c.nb_max_frames >= 1;
}

size_t frames_smem(const fmd_feature_config& c) {
  const int n_freq = c.n_fft / 2 + 1;
  return ((size_t)(kMelFt - 1) * c.hop_length + c.n_fft + (size_t)kMelFt * n_freq) * sizeof(double);
}

}  // namespace

struct fmd_mel {
  fmd_feature_config cfg{};
  int device = 0;
  int n_freq = 0;
  cudaStream_t stream = nullptr;
  std::string err;
  double* basis = nullptr;   // [2][n_fft][n_freq]
  float* fb = nullptr;       // [n_mels][n_freq]
  int2* span = nullptr;      // [n_mels]
  unsigned* peak = nullptr;  // [max chunks]
  int peak_cap = 0;
  float* stage = nullptr;    // host samples staged per call
  size_t stage_bytes = 0;
};

namespace {

int mfail(fmd_mel* h, int code, const std::string& msg) {
  if (h) h->err = msg;
  return code;
}

#define MCK(call)                                                                                        \
  do {                                                                                                   \
    cudaError_t e_ = (call);                                                                             \
    if (e_ != cudaSuccess)                                                                               \
      return mfail(h, e_ == cudaErrorMemoryAllocation ? FMD_ENOMEM : FMD_EIO,                             \
                   std::string(#call) + ": " + cudaGetErrorString(e_));                                   \
  } while (0)

bool mel_on_device(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

}  // namespace

extern "C" {

int fmd_mel_filters(const fmd_feature_config* cfg, float* out) {
  if (cfg == nullptr || out == nullptr || !cfg_ok(*cfg)) return FMD_EINVAL;
  const int n_freq = cfg->n_fft / 2 + 1;
  const std::vector<float> fb = filter_bank(n_freq, cfg->feature_size, 0.0f, (float)cfg->sampling_rate / 2.0f,
                                            (float)cfg->sampling_rate, nullptr);
  std::copy(fb.begin(), fb.end(), out);
  return FMD_OK;
}

int fmd_mel_create(const fmd_feature_config* cfg, int32_t device, fmd_mel** out) {
  if (cfg == nullptr || out == nullptr) return FMD_EINVAL;
  *out = nullptr;
  if (!cfg_ok(*cfg)) return FMD_EINVAL;
  const int n_freq = cfg->n_fft / 2 + 1;
  if (n_freq > kMelThreads || frames_smem(*cfg) > 200 * 1024) return FMD_ENOTSUP;
  fmd_mel* h = new fmd_mel();
  *out = h;
  h->cfg = *cfg;
  h->device = device;
  h->n_freq = n_freq;
  MCK(cudaSetDevice(device));
  MCK(cudaFuncSetAttribute(k_mel_frames, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)frames_smem(*cfg)));
  MCK(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));

  const int N = cfg->n_fft;
  const std::vector<float> w = hann_periodic(N);
  std::vector<double> basis((size_t)2 * N * n_freq);
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < n_freq; ++k) {
      const double ang = 2.0 * M_PI * (double)(((long long)k * n) % N) / (double)N;
      basis[(size_t)n * n_freq + k] = (double)w[n] * std::cos(ang);
      basis[(size_t)N * n_freq + (size_t)n * n_freq + k] = (double)w[n] * std::sin(ang);
    }
  std::vector<std::pair<int, int>> spans;
  const std::vector<float> fb = filter_bank(n_freq, cfg->feature_size, 0.0f, (float)cfg->sampling_rate / 2.0f,
                                            (float)cfg->sampling_rate, &spans);
  std::vector<int2> sp(spans.size());
  for (size_t i = 0; i < spans.size(); ++i) sp[i] = make_int2(spans[i].first, spans[i].second);
  MCK(cudaMalloc(&h->basis, basis.size() * sizeof(double)));
  MCK(cudaMalloc(&h->fb, fb.size() * sizeof(float)));
  MCK(cudaMalloc(&h->span, sp.size() * sizeof(int2)));
  MCK(cudaMemcpy(h->basis, basis.data(), basis.size() * sizeof(double), cudaMemcpyHostToDevice));
  MCK(cudaMemcpy(h->fb, fb.data(), fb.size() * sizeof(float), cudaMemcpyHostToDevice));
  MCK(cudaMemcpy(h->span, sp.data(), sp.size() * sizeof(int2), cudaMemcpyHostToDevice));
  return FMD_OK;
}

int fmd_mel_destroy(fmd_mel* h) {
  if (h == nullptr) return FMD_OK;
  cudaSetDevice(h->device);
  if (h->stream) cudaStreamSynchronize(h->stream);
  for (void* p : {(void*)h->basis, (void*)h->fb, (void*)h->span, (void*)h->peak, (void*)h->stage})
    if (p) cudaFree(p);
  if (h->stream) cudaStreamDestroy(h->stream);
  delete h;
  return FMD_OK;
}

const char* fmd_mel_last_error(const fmd_mel* h) { return h ? h->err.c_str() : ""; }

int fmd_mel_log_mel(fmd_mel* h, const float* samples, int32_t n_chunks, float* out) {
  if (h == nullptr) return FMD_EINVAL;
  h->err.clear();
  if (n_chunks < 0) return mfail(h, FMD_EINVAL, "n_chunks < 0");
  if (n_chunks == 0) return FMD_OK;
  if (samples == nullptr || out == nullptr) return mfail(h, FMD_EINVAL, "samples / out is NULL");
  if (!mel_on_device(out)) return mfail(h, FMD_EINVAL, "out must be device memory");
  const fmd_feature_config& c = h->cfg;
  MCK(cudaSetDevice(h->device));
  const size_t in_bytes = (size_t)n_chunks * c.n_samples * sizeof(float);
  const float* src = samples;
  if (!mel_on_device(samples)) {
    if (h->stage_bytes < in_bytes) {
      if (h->stage) cudaFree(h->stage);
      h->stage = nullptr;
      h->stage_bytes = 0;
      MCK(cudaMalloc(&h->stage, in_bytes));
      h->stage_bytes = in_bytes;
    }
    MCK(cudaMemcpyAsync(h->stage, samples, in_bytes, cudaMemcpyHostToDevice, h->stream));
    src = h->stage;
  }
  if (h->peak_cap < n_chunks) {
    if (h->peak) cudaFree(h->peak);
    h->peak = nullptr;
    h->peak_cap = 0;
    MCK(cudaMalloc(&h->peak, (size_t)n_chunks * sizeof(unsigned)));
    h->peak_cap = n_chunks;
  }
  MCK(cudaMemsetAsync(h->peak, 0, (size_t)n_chunks * sizeof(unsigned), h->stream));
  const dim3 grid((c.nb_max_frames + kMelFt - 1) / kMelFt, n_chunks);
  k_mel_frames<<<grid, kMelThreads, frames_smem(c), h->stream>>>(src, c.n_samples, c.nb_max_frames, c.hop_length,
                                                                  c.n_fft, h->n_freq, h->basis, h->fb, h->span,
                                                                  c.feature_size, out, h->peak);
  const size_t per_chunk = (size_t)c.feature_size * c.nb_max_frames, total = per_chunk * n_chunks;
  k_mel_finish<<<(int)std::min<size_t>((total + 255) / 256, 148 * 16), 256, 0, h->stream>>>(out, h->peak, per_chunk,
                                                                                          total);
  MCK(cudaGetLastError());
  MCK(cudaStreamSynchronize(h->stream));
  return FMD_OK;
}

}  // extern "C"
