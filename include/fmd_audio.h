/*
 * fmd_audio.h -- C ABI of the B200-native audio encoder: the Whisper encoder
 * and the VQ adaptor that turn 30 s log-mel chunks into the audio embeddings
 * spliced into a Moss prompt.
 *
 * It replaces, in cnmoro/fast-moss-diarization:
 *   - `WhisperEncoder::{load, forward}`
 *     (`crates/fmd-core/src/model/whisper_encoder.rs:114-163`),
 *   - `VqAdaptor::{load, time_merge, forward, merge_and_project}`
 *     (`crates/fmd-core/src/model/adaptor.rs:18-64`),
 *   - `MossModel::encode_audio` (`crates/fmd-core/src/model/mod.rs:75-126`):
 *     batched encoder passes over every chunk of a request set, per-chunk
 *     trimming to the chunk's audio tokens and per-file reassembly.
 * Conventions are those of fmd_decoder.h: `extern "C"`, plain pointers and
 * sizes, an `int` status (FMD_OK or a negative FMD_E* code) and a message in
 * `fmd_audio_last_error`. A handle is bound to one CUDA device, owns all of its
 * device memory, and is not thread-safe (the reference serialises calls behind
 * `Mutex<Engine>`, crates/fmd-py/src/lib.rs:176-183).
 *
 * Every projection stays dense in the activation dtype, as in the reference
 * (`linear_dense`, whisper_encoder.rs:31-39, adaptor.rs:27-33): the int8
 * precisions only select f16 activations (precision.rs:32-41).
 */
#ifndef FMD_AUDIO_H
#define FMD_AUDIO_H

#include <stddef.h>
#include <stdint.h>

#include "fmd_decoder.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct fmd_audio fmd_audio;

/* `AudioConfig` (crates/fmd-core/src/config.rs:61-75) plus the adaptor's
 * fields of `ModelConfig` (config.rs:78-90) and the text width it projects to. */
typedef struct fmd_audio_config {
  int32_t num_mel_bins;            /* 80 (Whisper-Medium)                         */
  int32_t d_model;                 /* 1024; a multiple of 128                      */
  int32_t encoder_layers;          /* 24                                           */
  int32_t encoder_attention_heads; /* 16; head_dim = d_model / heads must be 64    */
  int32_t encoder_ffn_dim;         /* 4096; a multiple of 128                      */
  int32_t max_source_positions;    /* 1500 = encoder frames per 30 s chunk         */
  int32_t audio_merge_size;        /* 4 (adaptor time merge)                       */
  int32_t adaptor_input_dim;       /* d_model * audio_merge_size                   */
  int32_t hidden_size;             /* text hidden size (adaptor output width)      */
  float adaptor_norm_eps;          /* text rms_norm_eps (mod.rs:49-55)             */
} fmd_audio_config;

/* One encoder layer, named as in the checkpoint under
 * `model.whisper_encoder.layers.{i}` (whisper_encoder.rs:28-41, :74-83).
 * Projections are row-major (out, in); k_proj has no bias. */
typedef struct fmd_encoder_layer_weights {
  fmd_tensor q_proj_w, q_proj_b;
  fmd_tensor k_proj_w;
  fmd_tensor v_proj_w, v_proj_b;
  fmd_tensor out_proj_w, out_proj_b;
  fmd_tensor self_attn_layer_norm_w, self_attn_layer_norm_b;
  fmd_tensor fc1_w, fc1_b;
  fmd_tensor fc2_w, fc2_b;
  fmd_tensor final_layer_norm_w, final_layer_norm_b;
} fmd_encoder_layer_weights;

/* Host tensors of the audio tower (whisper_encoder.rs:115-131, adaptor.rs:18-36):
 * conv1 (d_model, num_mel_bins, 3), conv2 (d_model, d_model, 3), positions
 * (max_source_positions, d_model), the final encoder layer_norm, and the
 * adaptor's `layers.0` (hidden, adaptor_input_dim), `layers.2`
 * (hidden, hidden), `layers.3` layer norm (hidden). */
typedef struct fmd_audio_weights {
  fmd_tensor conv1_w, conv1_b;
  fmd_tensor conv2_w, conv2_b;
  fmd_tensor embed_positions;
  const fmd_encoder_layer_weights* layers; /* encoder_layers entries */
  fmd_tensor layer_norm_w, layer_norm_b;
  fmd_tensor adaptor_fc1_w, adaptor_fc1_b;
  fmd_tensor adaptor_fc2_w, adaptor_fc2_b;
  fmd_tensor adaptor_norm_w, adaptor_norm_b;
} fmd_audio_weights;

/* `WhisperEncoder::load` + `VqAdaptor::load`: validates the shape, copies the
 * weights to `device` in the activation dtype of `precision` (FMD_PREC_*;
 * FMD_PREC_F32 is FMD_ENOTSUP), and reserves work buffers for batches of up to
 * `max_batch` chunks. Out-of-shape configurations are FMD_ENOTSUP. When a
 * failure happens after the handle was made, `*out` still holds it so that
 * fmd_audio_last_error can report the cause; release it with
 * fmd_audio_destroy. */
int fmd_audio_create(const fmd_audio_config* cfg, const fmd_audio_weights* w, int32_t precision, int32_t device,
                     int32_t max_batch, fmd_audio** out);
int fmd_audio_destroy(fmd_audio* h);
const char* fmd_audio_last_error(const fmd_audio* h);
/* Device bytes held: weights and work buffers. */
int fmd_audio_memory_bytes(const fmd_audio* h, int64_t* weights, int64_t* workspace);

/* `WhisperEncoder::forward` (whisper_encoder.rs:142-163) over `n_chunks` log-mel
 * chunks `mel` (n_chunks, num_mel_bins, 2 * max_source_positions), row-major,
 * dtype `mel_dtype` (FMD_DT_F32, or the activation dtype), in host or device
 * memory. Writes `frames_out` (device, n_chunks x max_source_positions x
 * d_model, activation dtype). Chunks are processed `max_batch` at a time. */
int fmd_audio_encode(fmd_audio* h, const void* mel, int32_t mel_dtype, int32_t n_chunks, void* frames_out);

/* `MossModel::encode_audio` (mod.rs:75-126): encoder passes over the chunks
 * `encoder_batch` at a time (capped at the handle's max_batch), each chunk
 * trimmed to `chunk_token_lengths[i] * audio_merge_size` frames, the parts of
 * audio `chunk_mapping[i]` joined in chunk order, merged and projected by the
 * adaptor. `audio_offsets` (host, num_audios + 1 entries) receives the first
 * output row of every audio (audio a owns rows [offsets[a], offsets[a+1])).
 * `out` (device, offsets[num_audios] x hidden_size, activation dtype, 16-byte
 * aligned) may be NULL to query the offsets only. An audio without chunks is
 * FMD_EINVAL (the reference fails to join an empty list). */
int fmd_audio_encode_audio(fmd_audio* h, const void* mel, int32_t mel_dtype, int32_t n_chunks,
                           const int32_t* chunk_token_lengths, const int32_t* chunk_mapping, int32_t num_audios,
                           int32_t encoder_batch, void* out, int64_t* audio_offsets);

/* The output layout of fmd_audio_encode_audio without a handle or a device:
 * audio a owns rows [offsets[a], offsets[a+1]) where each chunk i of audio
 * chunk_mapping[i] contributes min(chunk_token_lengths[i],
 * max_source_positions / audio_merge_size) rows, in chunk order
 * (mod.rs:108-125). `audio_offsets` has num_audios + 1 entries. Same errors as
 * fmd_audio_encode_audio (FMD_EINVAL for an audio without chunks). Host only. */
int fmd_audio_token_offsets(const fmd_audio_config* cfg, int32_t n_chunks, const int32_t* chunk_token_lengths,
                            const int32_t* chunk_mapping, int32_t num_audios, int64_t* audio_offsets);

/* CUDA-event time (ms) of the device work of the last encode call, and the
 * number of kernels it launched. */
int fmd_audio_last_timing(const fmd_audio* h, double* device_ms, int64_t* kernels);

/* ---- log-mel frontend ----------------------------------------------------
 * `MelFrontend` (crates/fmd-core/src/audio/mel.rs:29-133): periodic Hann
 * window, centred STFT with reflect padding, power spectrum, Slaney mel
 * filterbank, log10 with a 1e-10 floor, the per-chunk clamp at peak - 8 and
 * the (v + 4) / 4 rescale. `extract_features` (audio/mod.rs:47-116) runs it
 * on every zero-padded 30 s chunk; the chunk planning stays on the host. */

typedef struct fmd_mel fmd_mel;

/* `FeatureConfig` (crates/fmd-core/src/config.rs:121-166). */
typedef struct fmd_feature_config {
  int32_t feature_size;  /* n_mels: 80                                        */
  int32_t sampling_rate; /* 16000                                             */
  int32_t hop_length;    /* 160                                               */
  int32_t n_fft;         /* 400; n_fft / 2 + 1 <= 256 frequency bins          */
  int32_t n_samples;     /* 480000 samples per chunk (30 s)                   */
  int32_t nb_max_frames; /* 3000 = n_samples / hop_length                     */
} fmd_feature_config;

/* `MelFrontend::new`: the window, the DFT basis and the filterbank on
 * `device`. Unsupported shapes are FMD_ENOTSUP. On a failure after the handle
 * was made, `*out` holds it for fmd_mel_last_error; release it with
 * fmd_mel_destroy. */
int fmd_mel_create(const fmd_feature_config* cfg, int32_t device, fmd_mel** out);
int fmd_mel_destroy(fmd_mel* h);
const char* fmd_mel_last_error(const fmd_mel* h);

/* `MelFrontend::log_mel` of `n_chunks` windows of n_samples f32 samples each
 * (host or device memory, each already zero-padded to the window as
 * extract_features does, audio/mod.rs:100-106) -> `out` (device, f32,
 * n_chunks x feature_size x nb_max_frames), the encoder's mel input. */
int fmd_mel_log_mel(fmd_mel* h, const float* samples, int32_t n_chunks, float* out);

/* The Slaney filterbank `mel_filter_bank` (mel.rs:183-240) as a dense host
 * matrix (feature_size x (n_fft / 2 + 1)) f32. Host only. */
int fmd_mel_filters(const fmd_feature_config* cfg, float* out);

#ifdef __cplusplus
}
#endif

#endif /* FMD_AUDIO_H */
