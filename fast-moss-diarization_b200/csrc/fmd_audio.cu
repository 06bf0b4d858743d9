// Host runtime of the audio tower behind include/fmd_audio.h: weight upload,
// work buffers, the kernel sequence of one encoder pass and the
// `encode_audio` batching / trimming / per-file reassembly.
//
// One encoder pass over n chunks (`WhisperEncoder::forward`,
// crates/fmd-core/src/model/whisper_encoder.rs:142-163), F = 2 x frames:
//   im2col(mel) -> conv1 GEMM (+bias, GELU)          [n F][D]
//   im2col(conv1 out, stride 2) -> conv2 GEMM (+bias, GELU, + positions) -> x (f32)
//   per layer (whisper_encoder.rs:88-100):
//     LN -> QKV GEMM (+bias, q/k x head_dim^-1/4) -> attention -> out_proj GEMM (x += )
//     LN -> fc1 GEMM (+bias, GELU) -> fc2 GEMM (x += )
//   final LN -> frames (activation dtype)
// The adaptor (`VqAdaptor::merge_and_project`, adaptor.rs:41-64) reads the
// frames of a batch as [n frames / merge][merge D] (the time merge is a
// reshape of row-major frames): layers.0 GEMM (+bias, SiLU) -> layers.2 GEMM
// (+bias, f32) -> LN that writes each kept row straight to its place in the
// caller's output, which realises the per-chunk trim and the per-file
// concatenation of `MossModel::encode_audio` (model/mod.rs:82-126): every row
// after the encoder is computed independently, so projecting all rows of a
// chunk and keeping the first `tokens` equals trimming first.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/fmd_audio.h"
#include "fmd_audio.cuh"

using namespace fmd;

namespace {

struct EncLayer {
  void* qkv_w = nullptr;  // [3D][D]: q | k | v rows
  void* o_w = nullptr;
  void* fc1_w = nullptr;
  void* fc2_w = nullptr;
  float* qkv_b = nullptr;  // [3D]: q bias | 0 | v bias
  float* o_b = nullptr;
  float* fc1_b = nullptr;
  float* fc2_b = nullptr;
  float *ln1_w = nullptr, *ln1_b = nullptr, *ln2_w = nullptr, *ln2_b = nullptr;
  alignas(64) CUtensorMap qkv_m, o_m, fc1_m, fc2_m;
};

constexpr float kLnEps = 1e-5f;  // whisper_encoder.rs:14

}  // namespace

struct fmd_audio {
  fmd_audio_config cfg{};
  ActType at = kBF16;
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string err;
  std::vector<void*> allocs;
  int64_t weight_bytes = 0, work_bytes = 0;
  void* encode_fn = nullptr;
  int D = 0, F = 0, Tp = 0, H = 0, FF = 0, kp1 = 0, hid = 0, merge = 0, n_mels = 0;
  // weights
  void *conv1_w = nullptr, *conv2_w = nullptr, *ad1_w = nullptr, *ad2_w = nullptr;
  float *conv1_b = nullptr, *conv2_b = nullptr, *pos = nullptr, *lnf_w = nullptr, *lnf_b = nullptr;
  float *ad1_b = nullptr, *ad2_b = nullptr, *adn_w = nullptr, *adn_b = nullptr;
  std::vector<EncLayer> layers;
  alignas(64) CUtensorMap conv1_m, conv2_m, ad1_m, ad2_m;
  // work buffers for max_batch chunks (bufA/B/C are shared by the front convolutions and the layers)
  int max_batch = 0;
  // host mel is staged batch by batch through two pinned + two device slots on
  // a copy stream, so batch k + 1 is copied while batch k computes
  void* mel_dev[2] = {nullptr, nullptr};
  void* pinned[2] = {nullptr, nullptr};
  size_t mel_stage_bytes = 0;
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t ev_copied[2] = {nullptr, nullptr}, ev_consumed[2] = {nullptr, nullptr};
  int2* rowmap_all = nullptr;  // the adaptor row maps of every batch of a call
  size_t rowmap_cap = 0;
  void *bufA = nullptr, *bufB = nullptr, *bufC = nullptr, *hbuf = nullptr, *enc = nullptr, *ah = nullptr;
  float *x = nullptr, *af = nullptr;
  int* d_status = nullptr;
  void* stage = nullptr;  // weight upload staging
  size_t stage_bytes = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  double last_ms = 0.0;
  int64_t last_kernels = 0;
};

namespace {

int fail(fmd_audio* h, int code, const std::string& msg) {
  if (h) h->err = msg;
  return code;
}

#define ACK(call)                                                                                        \
  do {                                                                                                   \
    cudaError_t e_ = (call);                                                                             \
    if (e_ != cudaSuccess)                                                                               \
      return fail(h, e_ == cudaErrorMemoryAllocation ? FMD_ENOMEM : FMD_EIO,                              \
                  std::string(#call) + ": " + cudaGetErrorString(e_));                                    \
  } while (0)

template <typename P>
int alloc(fmd_audio* h, size_t bytes, P** out, int64_t* counter) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(h, FMD_ENOMEM, "cudaMalloc of " + std::to_string(bytes) + " bytes failed: " + cudaGetErrorString(e));
  }
  h->allocs.push_back(p);
  *counter += (int64_t)bytes;
  *out = static_cast<P*>(p);
  return FMD_OK;
}

size_t dt_size(int32_t dt) { return dt == FMD_DT_F32 ? 4 : 2; }

bool dense_dt(int32_t dt) { return dt == FMD_DT_F32 || dt == FMD_DT_F16 || dt == FMD_DT_BF16; }

// Host tensor of n values -> staging -> converted into `dst` (act dtype, or f32).
int put(fmd_audio* h, const fmd_tensor& t, size_t n, void* dst, bool f32, const char* what) {
  if (t.data == nullptr) return fail(h, FMD_EINVAL, std::string("missing tensor ") + what);
  if (!dense_dt(t.dtype)) return fail(h, FMD_EINVAL, std::string(what) + ": dtype must be f32, f16 or bf16");
  const size_t bytes = n * dt_size(t.dtype);
  if (bytes > h->stage_bytes) return fail(h, FMD_EINVAL, std::string(what) + ": larger than any tensor of the shape");
  ACK(cudaMemcpyAsync(h->stage, t.data, bytes, cudaMemcpyHostToDevice, h->stream));
  if (f32) launch_convert_f32(h->stage, t.dtype, n, static_cast<float*>(dst), h->stream);
  else launch_convert_act(h->at, h->stage, t.dtype, n, dst, h->stream);
  ACK(cudaGetLastError());
  return FMD_OK;
}

int weight_act(fmd_audio* h, const fmd_tensor& t, size_t n, void** out, const char* what) {
  int rc = alloc(h, n * 2, out, &h->weight_bytes);
  return rc ? rc : put(h, t, n, *out, false, what);
}

int weight_f32(fmd_audio* h, const fmd_tensor& t, size_t n, float** out, const char* what) {
  int rc = alloc(h, n * 4, out, &h->weight_bytes);
  return rc ? rc : put(h, t, n, *out, true, what);
}

int encoder_fn(fmd_audio* h) {
  if (h->encode_fn != nullptr) return FMD_OK;
  void* f = nullptr;
  cudaDriverEntryPointQueryResult qr;
  ACK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr));
  if (f == nullptr || qr != cudaDriverEntryPointSuccess)
    return fail(h, FMD_EIO, "cuTensorMapEncodeTiled is unavailable in this driver");
  h->encode_fn = f;
  return FMD_OK;
}

// Weight map of an [N][K] projection, box rows = the GEMM's tile width.
int wmap(fmd_audio* h, CUtensorMap* m, const void* w, int N, int K) {
  if (!enc_make_map2(h->encode_fn, m, w, (uint64_t)K, (uint64_t)N, (uint32_t)enc_gemm_bn(N)))
    return fail(h, FMD_EIO, "tensor map of an encoder weight could not be encoded");
  return FMD_OK;
}

int amap(fmd_audio* h, CUtensorMap* m, const void* a, int K, int M) {
  if (!enc_make_map2(h->encode_fn, m, a, (uint64_t)K, (uint64_t)M, 128))
    return fail(h, FMD_EIO, "tensor map of an encoder activation could not be encoded");
  return FMD_OK;
}

bool on_device(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

void gemm(fmd_audio* h, int epi, const CUtensorMap& a, const CUtensorMap& w, int M, int N, int K,
          const EncEpiArgs& ep, int64_t* kernels) {
  launch_enc_gemm(h->at, epi, a, w, enc_gemm_bn(N), M, N, K, ep, h->d_status, h->stream);
  ++*kernels;
}

EncEpiArgs epi_args(void* out, const float* bias) {
  EncEpiArgs e;
  e.out = out;
  e.bias = bias;
  return e;
}

// One encoder pass over n (<= max_batch) chunks already on the device;
// frames -> `out` ([n Tp][D], act dtype).
int run_encoder(fmd_audio* h, const void* mel, int mel_dt, int n, void* out, int64_t* kernels) {
  const int D = h->D, F = h->F, Tp = h->Tp, FF = h->FF;
  const int M1 = n * F, M2 = n * Tp;
  alignas(64) CUtensorMap a1_m, a2_m, h_m, ctx_m, ff_m, qkv3_m;
  int rc;
  if ((rc = amap(h, &a1_m, h->bufA, h->kp1, M1)) || (rc = amap(h, &a2_m, h->bufC, 3 * D, M2)) ||
      (rc = amap(h, &h_m, h->hbuf, D, M2)) || (rc = amap(h, &ctx_m, h->bufA, D, M2)) ||
      (rc = amap(h, &ff_m, h->bufC, FF, M2)))
    return rc;
  if (!enc_make_map3(h->encode_fn, &qkv3_m, h->bufB, (uint64_t)3 * D, (uint64_t)Tp, (uint64_t)n))
    return fail(h, FMD_EIO, "tensor map of the qkv buffer could not be encoded");

  cudaStream_t s = h->stream;
  launch_im2col_mel(h->at, mel, mel_dt, n, h->n_mels, F, h->kp1, h->bufA, s);
  ++*kernels;
  gemm(h, kEpiGelu, a1_m, h->conv1_m, M1, D, h->kp1, epi_args(h->bufB, h->conv1_b), kernels);
  launch_im2col_conv2(h->at, h->bufB, n, F, D, h->bufC, s);
  ++*kernels;
  {
    EncEpiArgs e = epi_args(h->x, h->conv2_b);
    e.pos = h->pos;
    e.period = Tp;
    gemm(h, kEpiGeluPos, a2_m, h->conv2_m, M2, D, 3 * D, e, kernels);
  }
  // head_dim^-1/4 on q and on k (whisper_encoder.rs:40, :52-55); q also carries
  // log2(e), so the attention kernel's scores are already in the exp2 domain
  const float qk_scale = std::pow(64.f, -0.25f), log2e = 1.4426950408889634f;
  for (const EncLayer& L : h->layers) {
    launch_layernorm(h->at, h->x, nullptr, M2, D, L.ln1_w, L.ln1_b, kLnEps, h->hbuf, s);
    EncEpiArgs e = epi_args(h->bufB, L.qkv_b);
    e.q_cols = D;
    e.scale_cols = 2 * D;
    e.scale_q = qk_scale * log2e;
    e.scale = qk_scale;
    gemm(h, kEpiQkv, h_m, L.qkv_m, M2, 3 * D, D, e, kernels);
    launch_enc_attn(h->at, qkv3_m, n, Tp, D, h->H, h->bufA, h->d_status, s);
    gemm(h, kEpiResid, ctx_m, L.o_m, M2, D, D, epi_args(h->x, L.o_b), kernels);
    launch_layernorm(h->at, h->x, nullptr, M2, D, L.ln2_w, L.ln2_b, kLnEps, h->hbuf, s);
    gemm(h, kEpiGelu, h_m, L.fc1_m, M2, FF, D, epi_args(h->bufC, L.fc1_b), kernels);
    gemm(h, kEpiResid, ff_m, L.fc2_m, M2, D, FF, epi_args(h->x, L.fc2_b), kernels);
    *kernels += 3;
  }
  launch_layernorm(h->at, h->x, nullptr, M2, D, h->lnf_w, h->lnf_b, kLnEps, out, s);
  ++*kernels;
  ACK(cudaGetLastError());
  return FMD_OK;
}

// Adaptor over the frames of n chunks in h->enc; rowmap (device) places
// `rows` kept tokens in `out`.
int run_adaptor(fmd_audio* h, int n, int rows, const int2* rowmap, void* out, int64_t* kernels) {
  const int Mg = n * h->Tp / h->merge, hid = h->hid, K = h->merge * h->D;
  alignas(64) CUtensorMap e_m, ah_m;
  int rc;
  if ((rc = amap(h, &e_m, h->enc, K, Mg)) || (rc = amap(h, &ah_m, h->ah, hid, Mg))) return rc;
  gemm(h, kEpiSilu, e_m, h->ad1_m, Mg, hid, K, epi_args(h->ah, h->ad1_b), kernels);
  gemm(h, kEpiF32, ah_m, h->ad2_m, Mg, hid, hid, epi_args(h->af, h->ad2_b), kernels);
  if (rows > 0) {
    launch_layernorm(h->at, h->af, rowmap, rows, hid, h->adn_w, h->adn_b, h->cfg.adaptor_norm_eps, out, h->stream);
    ++*kernels;
  }
  ACK(cudaGetLastError());
  return FMD_OK;
}

// Chunks [start, start + n) of `mel` (encoder batch `batch` of the call) to a
// device pointer the im2col kernel can read. Host mel goes through slot
// batch % 2: wait until the slot's previous copy has landed, fill the pinned
// buffer, copy on the copy stream once the device slot's previous reader has
// run, and make the compute stream wait for the copy.
int stage_mel(fmd_audio* h, const void* mel, int32_t mel_dt, bool dev, int start, int n, int batch,
              const void** out) {
  const size_t per = (size_t)h->n_mels * h->F * dt_size(mel_dt);
  const uint8_t* src = static_cast<const uint8_t*>(mel) + (size_t)start * per;
  if (dev) {
    *out = src;
    return FMD_OK;
  }
  const int s = batch & 1;
  ACK(cudaEventSynchronize(h->ev_copied[s]));
  std::memcpy(h->pinned[s], src, (size_t)n * per);
  ACK(cudaStreamWaitEvent(h->copy_stream, h->ev_consumed[s], 0));
  ACK(cudaMemcpyAsync(h->mel_dev[s], h->pinned[s], (size_t)n * per, cudaMemcpyHostToDevice, h->copy_stream));
  ACK(cudaEventRecord(h->ev_copied[s], h->copy_stream));
  ACK(cudaStreamWaitEvent(h->stream, h->ev_copied[s], 0));
  *out = h->mel_dev[s];
  return FMD_OK;
}

// After the batch that read slot batch % 2 has been launched.
int release_mel(fmd_audio* h, bool dev, int batch) {
  if (!dev) ACK(cudaEventRecord(h->ev_consumed[batch & 1], h->stream));
  return FMD_OK;
}

int check_mel(fmd_audio* h, const void* mel, int32_t mel_dt, int32_t n_chunks, bool* dev) {
  if (n_chunks < 0) return fail(h, FMD_EINVAL, "n_chunks < 0");
  if (n_chunks > 0 && mel == nullptr) return fail(h, FMD_EINVAL, "mel is NULL");
  const int32_t act_dt = h->at == kBF16 ? FMD_DT_BF16 : FMD_DT_F16;
  if (mel_dt != FMD_DT_F32 && mel_dt != act_dt)
    return fail(h, FMD_EINVAL, "mel dtype must be FMD_DT_F32 or the activation dtype");
  *dev = n_chunks > 0 && on_device(mel);
  return FMD_OK;
}

// Output rows of every audio (fmd_audio_token_offsets); `err` gets the reason of a failure.
int token_offsets(int per_chunk, int32_t n_chunks, const int32_t* tokens, const int32_t* mapping,
                  int32_t num_audios, int64_t* offsets, std::string* err) {
  if (num_audios < 0 || offsets == nullptr || n_chunks < 0) {
    *err = "bad n_chunks, num_audios or audio_offsets";
    return FMD_EINVAL;
  }
  if (n_chunks > 0 && (tokens == nullptr || mapping == nullptr)) {
    *err = "chunk_token_lengths / chunk_mapping is NULL";
    return FMD_EINVAL;
  }
  std::vector<int64_t> count(num_audios, 0), chunks(num_audios, 0);
  for (int i = 0; i < n_chunks; ++i) {
    if (mapping[i] < 0 || mapping[i] >= num_audios) {
      *err = "chunk_mapping[" + std::to_string(i) + "] is out of range";
      return FMD_EINVAL;
    }
    if (tokens[i] < 0) {
      *err = "negative chunk_token_lengths";
      return FMD_EINVAL;
    }
    count[mapping[i]] += std::min(tokens[i], per_chunk);
    ++chunks[mapping[i]];
  }
  offsets[0] = 0;
  for (int a = 0; a < num_audios; ++a) {
    if (chunks[a] == 0) {
      *err = "audio " + std::to_string(a) + " has no chunks";
      return FMD_EINVAL;
    }
    offsets[a + 1] = offsets[a] + count[a];
  }
  return FMD_OK;
}

int begin(fmd_audio* h) {
  ACK(cudaSetDevice(h->device));
  ACK(cudaMemsetAsync(h->d_status, 0, sizeof(int), h->stream));
  ACK(cudaEventRecord(h->ev0, h->stream));
  h->last_kernels = 0;
  return FMD_OK;
}

int finish(fmd_audio* h) {
  ACK(cudaEventRecord(h->ev1, h->stream));
  ACK(cudaStreamSynchronize(h->stream));
  float ms = 0.f;
  ACK(cudaEventElapsedTime(&ms, h->ev0, h->ev1));
  h->last_ms = ms;
  int st = 0;
  ACK(cudaMemcpy(&st, h->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st != 0) return fail(h, FMD_ETIMEDOUT, "a bounded device-side wait of the audio encoder gave up");
  return FMD_OK;
}

}  // namespace

extern "C" {

int fmd_audio_create(const fmd_audio_config* cfg, const fmd_audio_weights* w, int32_t precision, int32_t device,
                     int32_t max_batch, fmd_audio** out) {
  if (out == nullptr || cfg == nullptr || w == nullptr) return FMD_EINVAL;
  *out = nullptr;
  if (precision == FMD_PREC_F32) return FMD_ENOTSUP;
  if (precision != FMD_PREC_F16 && precision != FMD_PREC_BF16 && precision != FMD_PREC_INT8 &&
      precision != FMD_PREC_INT8_BF16)
    return FMD_EINVAL;
  const fmd_audio_config& c = *cfg;
  if (c.num_mel_bins < 1 || c.d_model < 1 || c.encoder_layers < 0 || c.encoder_attention_heads < 1 ||
      c.encoder_ffn_dim < 1 || c.max_source_positions < 1 || c.audio_merge_size < 1 || c.hidden_size < 1 ||
      max_batch < 1)
    return FMD_EINVAL;
  if (c.d_model % 128 || c.d_model > 2048 || c.d_model != c.encoder_attention_heads * 64 ||
      c.encoder_ffn_dim % 128 || c.num_mel_bins > 128 || c.max_source_positions % c.audio_merge_size ||
      c.adaptor_input_dim != c.audio_merge_size * c.d_model || c.hidden_size % 128 || c.hidden_size > 2048)
    return FMD_ENOTSUP;

  fmd_audio* h = new fmd_audio();
  h->cfg = c;
  h->at = (precision == FMD_PREC_BF16 || precision == FMD_PREC_INT8_BF16) ? kBF16 : kF16;
  h->device = device;
  h->D = c.d_model;
  h->Tp = c.max_source_positions;
  h->F = 2 * c.max_source_positions;
  h->H = c.encoder_attention_heads;
  h->FF = c.encoder_ffn_dim;
  h->n_mels = c.num_mel_bins;
  h->kp1 = (3 * c.num_mel_bins + 63) / 64 * 64;
  h->hid = c.hidden_size;
  h->merge = c.audio_merge_size;
  h->max_batch = max_batch;
  *out = h;

  const int D = h->D, FF = h->FF, Tp = h->Tp, F = h->F, hid = h->hid, Kad = c.adaptor_input_dim;
  ACK(cudaSetDevice(device));
  ACK(init_enc_kernels());
  ACK(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
  ACK(cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking));
  ACK(cudaEventCreate(&h->ev0));
  ACK(cudaEventCreate(&h->ev1));
  for (int s = 0; s < 2; ++s) {
    ACK(cudaEventCreateWithFlags(&h->ev_copied[s], cudaEventDisableTiming));
    ACK(cudaEventCreateWithFlags(&h->ev_consumed[s], cudaEventDisableTiming));
  }
  int rc = encoder_fn(h);
  if (rc) return rc;

  // staging for the largest host tensor (f32)
  const size_t largest = std::max({(size_t)D * c.num_mel_bins * 3, (size_t)D * D * 3, (size_t)Tp * D,
                                   (size_t)FF * D, (size_t)hid * Kad, (size_t)hid * hid});
  h->stage_bytes = largest * 4;
  if ((rc = alloc(h, h->stage_bytes, &h->stage, &h->work_bytes))) return rc;

  // front convolutions + positions
  if ((rc = alloc(h, (size_t)D * h->kp1 * 2, &h->conv1_w, &h->weight_bytes))) return rc;
  if ((rc = alloc(h, (size_t)D * 3 * D * 2, &h->conv2_w, &h->weight_bytes))) return rc;
  for (int which = 0; which < 2; ++which) {
    const fmd_tensor& t = which ? w->conv2_w : w->conv1_w;
    const int C = which ? D : c.num_mel_bins, kp = which ? 3 * D : h->kp1;
    const size_t n = (size_t)D * C * 3;
    if (t.data == nullptr || !dense_dt(t.dtype)) return fail(h, FMD_EINVAL, "conv weights must be dense host tensors");
    ACK(cudaMemcpyAsync(h->stage, t.data, n * dt_size(t.dtype), cudaMemcpyHostToDevice, h->stream));
    launch_conv_weight(h->at, h->stage, t.dtype, D, C, kp, which ? h->conv2_w : h->conv1_w, h->stream);
    ACK(cudaGetLastError());
  }
  if ((rc = weight_f32(h, w->conv1_b, D, &h->conv1_b, "conv1.bias")) ||
      (rc = weight_f32(h, w->conv2_b, D, &h->conv2_b, "conv2.bias")) ||
      (rc = weight_f32(h, w->embed_positions, (size_t)Tp * D, &h->pos, "embed_positions.weight")) ||
      (rc = weight_f32(h, w->layer_norm_w, D, &h->lnf_w, "layer_norm.weight")) ||
      (rc = weight_f32(h, w->layer_norm_b, D, &h->lnf_b, "layer_norm.bias")))
    return rc;
  if ((rc = wmap(h, &h->conv1_m, h->conv1_w, D, h->kp1)) || (rc = wmap(h, &h->conv2_m, h->conv2_w, D, 3 * D)))
    return rc;

  // layers
  if (c.encoder_layers > 0 && w->layers == nullptr) return fail(h, FMD_EINVAL, "layers is NULL");
  h->layers.resize(c.encoder_layers);
  for (int i = 0; i < c.encoder_layers; ++i) {
    const fmd_encoder_layer_weights& lw = w->layers[i];
    EncLayer& L = h->layers[i];
    const size_t DD = (size_t)D * D;
    if ((rc = alloc(h, 3 * DD * 2, &L.qkv_w, &h->weight_bytes))) return rc;
    uint8_t* qkv = static_cast<uint8_t*>(L.qkv_w);
    if ((rc = put(h, lw.q_proj_w, DD, qkv, false, "q_proj.weight")) ||
        (rc = put(h, lw.k_proj_w, DD, qkv + DD * 2, false, "k_proj.weight")) ||
        (rc = put(h, lw.v_proj_w, DD, qkv + 2 * DD * 2, false, "v_proj.weight")))
      return rc;
    if ((rc = alloc(h, (size_t)3 * D * 4, &L.qkv_b, &h->weight_bytes))) return rc;
    ACK(cudaMemsetAsync(L.qkv_b, 0, (size_t)3 * D * 4, h->stream));  // k_proj has no bias
    if ((rc = put(h, lw.q_proj_b, D, L.qkv_b, true, "q_proj.bias")) ||
        (rc = put(h, lw.v_proj_b, D, L.qkv_b + 2 * D, true, "v_proj.bias")))
      return rc;
    if ((rc = weight_act(h, lw.out_proj_w, DD, &L.o_w, "out_proj.weight")) ||
        (rc = weight_f32(h, lw.out_proj_b, D, &L.o_b, "out_proj.bias")) ||
        (rc = weight_f32(h, lw.self_attn_layer_norm_w, D, &L.ln1_w, "self_attn_layer_norm.weight")) ||
        (rc = weight_f32(h, lw.self_attn_layer_norm_b, D, &L.ln1_b, "self_attn_layer_norm.bias")) ||
        (rc = weight_act(h, lw.fc1_w, (size_t)FF * D, &L.fc1_w, "fc1.weight")) ||
        (rc = weight_f32(h, lw.fc1_b, FF, &L.fc1_b, "fc1.bias")) ||
        (rc = weight_act(h, lw.fc2_w, (size_t)D * FF, &L.fc2_w, "fc2.weight")) ||
        (rc = weight_f32(h, lw.fc2_b, D, &L.fc2_b, "fc2.bias")) ||
        (rc = weight_f32(h, lw.final_layer_norm_w, D, &L.ln2_w, "final_layer_norm.weight")) ||
        (rc = weight_f32(h, lw.final_layer_norm_b, D, &L.ln2_b, "final_layer_norm.bias")))
      return rc;
    if ((rc = wmap(h, &L.qkv_m, L.qkv_w, 3 * D, D)) || (rc = wmap(h, &L.o_m, L.o_w, D, D)) ||
        (rc = wmap(h, &L.fc1_m, L.fc1_w, FF, D)) || (rc = wmap(h, &L.fc2_m, L.fc2_w, D, FF)))
      return rc;
  }

  // adaptor (adaptor.rs:18-36)
  if ((rc = weight_act(h, w->adaptor_fc1_w, (size_t)hid * Kad, &h->ad1_w, "vq_adaptor.layers.0.weight")) ||
      (rc = weight_f32(h, w->adaptor_fc1_b, hid, &h->ad1_b, "vq_adaptor.layers.0.bias")) ||
      (rc = weight_act(h, w->adaptor_fc2_w, (size_t)hid * hid, &h->ad2_w, "vq_adaptor.layers.2.weight")) ||
      (rc = weight_f32(h, w->adaptor_fc2_b, hid, &h->ad2_b, "vq_adaptor.layers.2.bias")) ||
      (rc = weight_f32(h, w->adaptor_norm_w, hid, &h->adn_w, "vq_adaptor.layers.3.weight")) ||
      (rc = weight_f32(h, w->adaptor_norm_b, hid, &h->adn_b, "vq_adaptor.layers.3.bias")))
    return rc;
  if ((rc = wmap(h, &h->ad1_m, h->ad1_w, hid, Kad)) || (rc = wmap(h, &h->ad2_m, h->ad2_w, hid, hid))) return rc;

  // work buffers (zeroed once so no tile ever reads uninitialised bits)
  const size_t mb = (size_t)max_batch, rows = mb * Tp, groups = rows / h->merge;
  const size_t szA = std::max(rows * D, mb * F * h->kp1) * 2;      // ctx | conv1 operand
  const size_t szB = std::max(rows * 3 * D, mb * F * D) * 2;       // qkv | conv1 output
  const size_t szC = std::max(rows * FF, rows * 3 * D) * 2;        // fc1 output | conv2 operand
  h->mel_stage_bytes = mb * c.num_mel_bins * F * 4;
  struct B {
    void** p;
    size_t n;
  } bufs[] = {{&h->bufA, szA},
              {&h->bufB, szB},
              {&h->bufC, szC},
              {&h->hbuf, rows * D * 2},
              {&h->enc, rows * D * 2},
              {reinterpret_cast<void**>(&h->x), rows * D * 4},
              {&h->ah, groups * hid * 2},
              {reinterpret_cast<void**>(&h->af), groups * hid * 4},
              {reinterpret_cast<void**>(&h->d_status), 16},
              {&h->mel_dev[0], h->mel_stage_bytes},
              {&h->mel_dev[1], h->mel_stage_bytes}};
  for (B& b : bufs) {
    if ((rc = alloc(h, b.n, b.p, &h->work_bytes))) return rc;
    ACK(cudaMemsetAsync(*b.p, 0, b.n, h->stream));
  }
  for (int s = 0; s < 2; ++s) ACK(cudaHostAlloc(&h->pinned[s], h->mel_stage_bytes, cudaHostAllocDefault));
  ACK(cudaStreamSynchronize(h->stream));
  return FMD_OK;
}

int fmd_audio_destroy(fmd_audio* h) {
  if (h == nullptr) return FMD_OK;
  cudaSetDevice(h->device);
  if (h->stream) cudaStreamSynchronize(h->stream);
  if (h->copy_stream) cudaStreamSynchronize(h->copy_stream);
  for (void* p : h->allocs) cudaFree(p);
  if (h->rowmap_all) cudaFree(h->rowmap_all);
  for (int s = 0; s < 2; ++s) {
    if (h->pinned[s]) cudaFreeHost(h->pinned[s]);
    if (h->ev_copied[s]) cudaEventDestroy(h->ev_copied[s]);
    if (h->ev_consumed[s]) cudaEventDestroy(h->ev_consumed[s]);
  }
  if (h->ev0) cudaEventDestroy(h->ev0);
  if (h->ev1) cudaEventDestroy(h->ev1);
  if (h->copy_stream) cudaStreamDestroy(h->copy_stream);
  if (h->stream) cudaStreamDestroy(h->stream);
  delete h;
  return FMD_OK;
}

const char* fmd_audio_last_error(const fmd_audio* h) { return h ? h->err.c_str() : ""; }

int fmd_audio_memory_bytes(const fmd_audio* h, int64_t* weights, int64_t* workspace) {
  if (h == nullptr) return FMD_EINVAL;
  if (weights) *weights = h->weight_bytes;
  if (workspace) *workspace = h->work_bytes;
  return FMD_OK;
}

int fmd_audio_token_offsets(const fmd_audio_config* cfg, int32_t n_chunks, const int32_t* chunk_token_lengths,
                            const int32_t* chunk_mapping, int32_t num_audios, int64_t* audio_offsets) {
  if (cfg == nullptr || cfg->audio_merge_size < 1 || cfg->max_source_positions < 1) return FMD_EINVAL;
  std::string err;
  return token_offsets(cfg->max_source_positions / cfg->audio_merge_size, n_chunks, chunk_token_lengths,
                       chunk_mapping, num_audios, audio_offsets, &err);
}

int fmd_audio_last_timing(const fmd_audio* h, double* device_ms, int64_t* kernels) {
  if (h == nullptr) return FMD_EINVAL;
  if (device_ms) *device_ms = h->last_ms;
  if (kernels) *kernels = h->last_kernels;
  return FMD_OK;
}

int fmd_audio_encode(fmd_audio* h, const void* mel, int32_t mel_dtype, int32_t n_chunks, void* frames_out) {
  if (h == nullptr) return FMD_EINVAL;
  h->err.clear();
  bool dev = false;
  int rc = check_mel(h, mel, mel_dtype, n_chunks, &dev);
  if (rc) return rc;
  if (n_chunks == 0) return FMD_OK;
  if (frames_out == nullptr || (reinterpret_cast<uintptr_t>(frames_out) & 15) || !on_device(frames_out))
    return fail(h, FMD_EINVAL, "frames_out must be 16-byte aligned device memory");
  if ((rc = begin(h))) return rc;
  const size_t per_chunk = (size_t)h->Tp * h->D * 2;
  for (int start = 0, batch = 0; start < n_chunks; start += h->max_batch, ++batch) {
    const int n = std::min(h->max_batch, n_chunks - start);
    const void* src = nullptr;
    if ((rc = stage_mel(h, mel, mel_dtype, dev, start, n, batch, &src))) return rc;
    void* out = static_cast<uint8_t*>(frames_out) + (size_t)start * per_chunk;
    if ((rc = run_encoder(h, src, mel_dtype, n, out, &h->last_kernels))) return rc;
    if ((rc = release_mel(h, dev, batch))) return rc;
  }
  return finish(h);
}

int fmd_audio_encode_audio(fmd_audio* h, const void* mel, int32_t mel_dtype, int32_t n_chunks,
                           const int32_t* chunk_token_lengths, const int32_t* chunk_mapping, int32_t num_audios,
                           int32_t encoder_batch, void* out, int64_t* audio_offsets) {
  if (h == nullptr) return FMD_EINVAL;
  h->err.clear();
  // Rows kept per chunk: tokens * merge frames, at most the chunk's frames
  // (mod.rs:110-116), merged back into min(tokens, Tp / merge) rows.
  const int per_chunk = h->Tp / h->merge;
  int rc0 = token_offsets(per_chunk, n_chunks, chunk_token_lengths, chunk_mapping, num_audios, audio_offsets,
                          &h->err);
  if (rc0) return rc0;
  if (out == nullptr || n_chunks == 0) return FMD_OK;
  bool dev = false;
  int rc = check_mel(h, mel, mel_dtype, n_chunks, &dev);
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || !on_device(out))
    return fail(h, FMD_EINVAL, "out must be 16-byte aligned device memory");

  const int eb = std::min(std::max(encoder_batch, 1), h->max_batch);
  // the adaptor row maps of every batch, uploaded once: entry {row of the
  // batch's merged frames, output row}
  std::vector<int64_t> next(audio_offsets, audio_offsets + num_audios);
  std::vector<int2> map;
  std::vector<size_t> batch_at;
  for (int start = 0; start < n_chunks; start += eb) {
    batch_at.push_back(map.size());
    const int n = std::min(eb, n_chunks - start);
    for (int b = 0; b < n; ++b) {
      const int g = start + b, a = chunk_mapping[g];
      const int keep = std::min(chunk_token_lengths[g], per_chunk);
      for (int j = 0; j < keep; ++j) map.push_back(make_int2(b * per_chunk + j, (int)(next[a] + j)));
      next[a] += keep;
    }
  }
  batch_at.push_back(map.size());
  if ((rc = begin(h))) return rc;
  if (map.size() > h->rowmap_cap) {
    ACK(cudaStreamSynchronize(h->stream));
    if (h->rowmap_all) cudaFree(h->rowmap_all);
    h->rowmap_all = nullptr;
    h->rowmap_cap = 0;
    ACK(cudaMalloc(&h->rowmap_all, map.size() * sizeof(int2)));
    h->rowmap_cap = map.size();
  }
  if (!map.empty())
    ACK(cudaMemcpyAsync(h->rowmap_all, map.data(), map.size() * sizeof(int2), cudaMemcpyHostToDevice, h->stream));
  for (int start = 0, batch = 0; start < n_chunks; start += eb, ++batch) {
    const int n = std::min(eb, n_chunks - start);
    const void* src = nullptr;
    if ((rc = stage_mel(h, mel, mel_dtype, dev, start, n, batch, &src))) return rc;
    if ((rc = run_encoder(h, src, mel_dtype, n, h->enc, &h->last_kernels))) return rc;
    if ((rc = release_mel(h, dev, batch))) return rc;
    const int rows = (int)(batch_at[batch + 1] - batch_at[batch]);
    if ((rc = run_adaptor(h, n, rows, h->rowmap_all + batch_at[batch], out, &h->last_kernels))) return rc;
  }
  return finish(h);
}

}  // extern "C"
