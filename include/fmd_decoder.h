/*
 * fmd_decoder.h -- C ABI of the B200-native batched Qwen3 decoder step.
 *
 * This library replaces the candle decoder of cnmoro/fast-moss-diarization
 * (`crates/fmd-core/src/model/qwen3.rs`, `crates/fmd-core/src/model/linear.rs`)
 * and the greedy micro-batch loop that drives it
 * (`crates/fmd-core/src/engine.rs:382-424`, `:463-541`). Every entry point is
 * `extern "C"` with plain pointers and sizes; host buffers are borrowed for
 * the duration of the call only. All device memory is owned by the handle.
 *
 * Conventions
 *  - Every function returns an `int` status: 0 on success, a negative
 *    errno-style code otherwise (FMD_E*). `fmd_last_error(h)` returns the
 *    message of the last failure on that handle. The reference surfaces the
 *    same failures as `crate::error::Error` (`error.rs:9-49`); KV overflow maps
 *    `KvCache::append`'s error (`qwen3.rs:88-94`) to FMD_EOVERFLOW, and an
 *    allocation failure maps the batch-level failure of `engine.rs:414-421`
 *    to FMD_ENOMEM.
 *  - A handle is bound to one CUDA device and is NOT thread-safe: callers
 *    serialise calls, as the reference's Python binding does with
 *    `Mutex<Engine>` (`crates/fmd-py/src/lib.rs:176-183`).
 *  - Activation buffers passed in or out use the handle's activation dtype
 *    (bf16 or f16 raw bits) unless a dtype argument says otherwise; logits are
 *    always f32 (`qwen3.rs:459-463`).
 */
#ifndef FMD_DECODER_H
#define FMD_DECODER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define FMD_OK 0
#define FMD_EINVAL (-22)     /* bad argument (shape, slot, dtype ...)            */
#define FMD_ENOMEM (-12)     /* device allocation / KV pool exhausted            */
#define FMD_EIO (-5)         /* CUDA runtime error                               */
#define FMD_EBUSY (-16)      /* wrong state: no weights loaded, no KV reserved   */
#define FMD_EOVERFLOW (-75)  /* KV cache capacity of a slot exceeded             */
#define FMD_ENOTSUP (-95)    /* configuration not supported by these kernels     */
#define FMD_ETIMEDOUT (-110) /* a bounded device-side wait gave up               */

/* ---- precisions (precision.rs:11-17, :32-41) ----------------------------- */
#define FMD_PREC_F32 0       /* not supported on the GPU path: FMD_ENOTSUP       */
#define FMD_PREC_F16 1       /* dense f16 weights, f16 activations               */
#define FMD_PREC_BF16 2      /* dense bf16 weights, bf16 activations (default)   */
#define FMD_PREC_INT8 3      /* Q8_0 weights, f16 activations (reference Int8)   */
#define FMD_PREC_INT8_BF16 4 /* Q8_0 weights, bf16 activations                   */

/* ---- host tensor dtypes -------------------------------------------------- */
#define FMD_DT_F32 0
#define FMD_DT_F16 1
#define FMD_DT_BF16 2
#define FMD_DT_Q8_0 3 /* GGML blocks of 34 bytes {f16 d; int8 qs[32]} along the input axis */

/* ---- finish reasons (engine.rs:132-137) -------------------------------- */
#define FMD_FINISH_STOP 0   /* end-of-turn token (or the forced stop step)      */
#define FMD_FINISH_LENGTH 1 /* max_new_tokens budget ran out                    */

typedef struct fmd_handle fmd_handle;

/* Qwen3 text backbone shape (`TextConfig`, config.rs:8-58). */
typedef struct fmd_config {
  int32_t vocab_size;
  int32_t hidden_size;
  int32_t intermediate_size;
  int32_t num_hidden_layers;
  int32_t num_attention_heads;
  int32_t num_key_value_heads;
  int32_t head_dim;                /* only 128 is supported                      */
  float rms_norm_eps;
  double rope_theta;
  int32_t max_position_embeddings; /* RoPE table = min(this, 65536), engine.rs:238-243 */
  int32_t eos_token_id;            /* 151645 in the reference, engine.rs:246       */
} fmd_config;

/* A host tensor: `data` points at row-major values of dtype FMD_DT_*. */
typedef struct fmd_tensor {
  const void* data;
  int32_t dtype;
} fmd_tensor;

/* One decoder layer, named as in the checkpoint (qwen3.rs:177-193, :268-285,
 * :306-318). Projections are row-major (out, in). */
typedef struct fmd_layer_weights {
  fmd_tensor input_layernorm;
  fmd_tensor post_attention_layernorm;
  fmd_tensor q_norm;
  fmd_tensor k_norm;
  fmd_tensor q_proj;
  fmd_tensor k_proj;
  fmd_tensor v_proj;
  fmd_tensor o_proj;
  fmd_tensor gate_proj;
  fmd_tensor up_proj;
  fmd_tensor down_proj;
} fmd_layer_weights;

typedef struct fmd_weights {
  fmd_tensor embed_tokens;          /* (vocab, hidden); lookups stay dense (qwen3.rs:360) */
  fmd_tensor norm;                  /* (hidden)                                           */
  fmd_tensor lm_head;               /* (vocab, hidden); data == NULL => tied (qwen3.rs:366-372) */
  const fmd_layer_weights* layers;  /* num_hidden_layers entries                          */
} fmd_weights;

/* One generation request for the continuous-batching engine: the prompt is
 * `prompt_len` rows of the embedding arena starting at `embed_row` (the
 * output of the reference's `MossModel::splice_audio`, model/mod.rs:134-180). */
typedef struct fmd_request {
  int32_t prompt_len;
  int32_t max_new_tokens;  /* generation budget (engine.rs:466-469)                */
  int32_t forced_stop;     /* -1, or: the n-th generated token ends the turn        */
  int32_t reserved;
  int64_t embed_row;
} fmd_request;

typedef struct fmd_result {
  int32_t n_tokens;        /* tokens emitted (EOS is not emitted, engine.rs:513-518) */
  int32_t finish_reason;   /* FMD_FINISH_*                                           */
} fmd_result;

typedef struct fmd_stats {
  int64_t steps;            /* device steps run since fmd_engine_start           */
  int64_t generated_tokens; /* engine.rs:395 BatchStats::generated_tokens        */
  int64_t prefill_tokens;
  int64_t requests_done;
  double generate_seconds;  /* wall time of the call (engine.rs:424)             */
  int32_t device_status;    /* 0, or a FMD_E* code raised on the device          */
  int32_t reserved;
  /* the window advanced by this call (fmd_engine_step / fmd_engine_run) */
  int64_t window_steps;     /* device steps launched                             */
  int64_t window_tokens;    /* tokens emitted                                    */
  double window_device_ms;  /* CUDA-event time on the engine stream              */
  /* decode attention of the window's last step (CUDA events around each of
   * its per-layer launches inside the step graph) */
  double attn_decode_ms;    /* duration of the middle layer's launch in the last step */
  int64_t attn_kv_tokens;   /* sum of key positions read by one launch           */
  int64_t attn_rows;        /* decode rows in that step                          */
  int64_t window_mixed_steps; /* steps of the window that could carry prefill rows */
  int64_t graph_kernels_mixed;  /* kernels in one replay of the step graph that may carry prefill rows */
  int64_t graph_kernels_decode; /* kernels in one replay of the decode-only step graph */
  double lm_head_ms;        /* duration of the lm_head launch of the window's last step */
} fmd_stats;

/* ---- handle ------------------------------------------------------------- */

/* Replaces `Engine::new` / `Qwen3::load` construction (engine.rs:189-259,
 * qwen3.rs:354-390): validates the shape and precision and binds `device`. */
int fmd_create(const fmd_config* cfg, int32_t precision, int32_t device, fmd_handle** out);
int fmd_destroy(fmd_handle* h);
const char* fmd_last_error(const fmd_handle* h);
const char* fmd_status_string(int32_t status);
int fmd_version(void);

/* Replaces `Loader::{linear_with, fused_linear}` + `Qwen3::load`
 * (linear.rs:179-265, qwen3.rs:354-390): copies host weights to the device,
 * converting dense tensors to the activation dtype and, for the int8
 * precisions, quantising f32/bf16/f16 projections to Q8_0 exactly as the
 * reference does (from the f32 value). Q8_0 sources are repacked as-is. */
int fmd_load_weights(fmd_handle* h, const fmd_weights* w);

/* Replaces `Qwen3::new_caches` (qwen3.rs:415-428): reserves a paged KV pool of
 * `max_tokens_total` token positions shared by `max_slots` sequences, and work
 * buffers for up to `max_rows_per_step` token rows per forward pass. Returns
 * FMD_ENOMEM instead of aborting when the device cannot hold it. */
int fmd_kv_reserve(fmd_handle* h, int32_t max_slots, int64_t max_tokens_total, int32_t max_rows_per_step);

/* `Qwen3::cache_bytes` (qwen3.rs:431-440) for a dense (batch, capacity) cache. */
int64_t fmd_cache_bytes(const fmd_config* cfg, int32_t precision, int64_t batch, int64_t capacity);
/* Device bytes held by the handle: weights, KV pool, work buffers. */
int fmd_memory_bytes(const fmd_handle* h, int64_t* weights, int64_t* kv_pool, int64_t* workspace);

/* ---- decoder-forward operator surface ----------------------------------- */

/* `Qwen3::embed` (qwen3.rs:405-412): `n` ids -> n x hidden rows (act dtype). */
int fmd_embed(fmd_handle* h, const int32_t* ids, int64_t n, void* out);

/* `MossModel::splice_audio` (crates/fmd-core/src/model/mod.rs:134-180): the
 * prompt embedding of one sequence, assembled on the GPU. `token_ids` (host,
 * `n_ids` ids) is the prompt with `audio_token_id` at every audio position;
 * text ids are looked up in the embedding table and the audio positions take
 * the rows of `audio_embeds` (device, `n_audio` x hidden, FMD_DT_F32 or the
 * activation dtype) in order. `out` (device, n_ids x hidden, activation dtype)
 * can be the caller's prompt arena, e.g. the buffer later passed to
 * fmd_engine_load. Both device buffers must be 16-byte aligned memory of the
 * handle's device. A placeholder count different from `n_audio` is
 * FMD_EINVAL, as in the reference (mod.rs:143-150). Needs weights, not a KV
 * reservation. */
int fmd_splice_audio(fmd_handle* h, const int32_t* token_ids, int64_t n_ids, const void* audio_embeds,
                     int64_t n_audio, int32_t audio_dtype, int32_t audio_token_id, void* out);

/* Open a sequence slot with room for `capacity` positions: the per-sequence
 * analogue of `KvCache::new` (qwen3.rs:41-55). Fails with FMD_ENOMEM when the
 * pool has too few free pages. */
int fmd_slot_open(fmd_handle* h, int32_t slot, int32_t capacity);
/* Release a slot's pages (`KvCache::truncate(0)` + drop, qwen3.rs:105-107). */
int fmd_slot_release(fmd_handle* h, int32_t slot);
/* Current cached length of a slot (`KvCache::len`, qwen3.rs:57-59). */
int fmd_slot_len(fmd_handle* h, int32_t slot, int32_t* len);

/* `Qwen3::prefill` + `Qwen3::logits` (qwen3.rs:475-496, :459-463) over a
 * ragged batch: sequence i appends `lens[i]` prompt rows to slot `slots[i]`.
 * `embeds` holds sum(lens) x hidden rows of dtype `embeds_dtype`
 * (FMD_DT_F32 or the activation dtype) back to back, in sequence order (the
 * reference passes the same rows left-padded, engine.rs:476-491). Outputs are
 * the last position's f32 logits (n x vocab) and/or greedy ids (n); either
 * may be NULL. */
int fmd_prefill(fmd_handle* h, int32_t n, const int32_t* slots, const int32_t* lens,
                const void* embeds, int32_t embeds_dtype, float* logits, int32_t* next_ids);

/* `Qwen3::decode_step` + `argmax_rows` (qwen3.rs:499-511, engine.rs:550-559):
 * one token per slot. Outputs as for fmd_prefill. Each slot's position is its
 * own cached length, so no shared offset / pad_lengths are needed. */
int fmd_decode_step(fmd_handle* h, int32_t n, const int32_t* slots, const int32_t* ids,
                    float* logits, int32_t* next_ids);

/* ---- continuous-batching engine (engine.rs:382-424, :463-541) ----------- */

/* Copy a request queue and its prompt-embedding arena (`embed_rows` x hidden,
 * dtype `embeds_dtype`) into device memory. Requests are served in the given
 * order; sort them by prompt length first to mirror engine.rs:385. The arena
 * may be host memory, or device memory of the handle's device in the
 * activation dtype (e.g. rows written by fmd_splice_audio), which is copied on
 * the device. */
int fmd_engine_load(fmd_handle* h, const fmd_request* reqs, int32_t n_reqs,
                    const void* embeds, int64_t embed_rows, int32_t embeds_dtype);

/* Reset the engine onto the loaded queue (all slots free, all KV pages free)
 * and build the CUDA graph of one step for (`max_batch`, `prefill_chunk`). */
int fmd_engine_start(fmd_handle* h, int32_t max_batch, int32_t prefill_chunk);

/* Advance the started engine by up to `max_steps` device steps (fewer if the
 * queue drains). `stats` is cumulative since fmd_engine_start, plus the window
 * fields for this call. */
int fmd_engine_step(fmd_handle* h, int64_t max_steps, fmd_stats* stats);

/* fmd_engine_start + fmd_engine_step until the queue drains: up to
 * `max_batch` sequences decode together; finished slots are refilled from the
 * queue on the GPU; prompts are prefilled in chunks of up to `prefill_chunk`
 * rows mixed into decode steps. Returns when every request is done or
 * `max_steps` steps ran. */
int fmd_engine_run(fmd_handle* h, int32_t max_batch, int32_t prefill_chunk, int64_t max_steps,
                   fmd_stats* stats);

/* Copy results back: `tokens` is n_reqs x `token_stride` int32 (row i holds
 * request i's emitted ids), `results` is n_reqs entries. Either may be NULL. */
int fmd_engine_fetch(fmd_handle* h, int32_t* tokens, int32_t token_stride, fmd_result* results);

/* load + run + fetch in one call: the host-buffer entry point that replaces
 * `Engine::generate_batch` over a whole request list. */
int fmd_generate(fmd_handle* h, const fmd_request* reqs, int32_t n_reqs, const void* embeds,
                 int64_t embed_rows, int32_t embeds_dtype, int32_t max_batch, int32_t prefill_chunk,
                 int32_t* tokens, int32_t token_stride, fmd_result* results, fmd_stats* stats);

/* ---- inspection (tests) -------------------------------------------------- */

/* Dequantise (or widen) one stored projection back to f32 on the device and
 * copy it out: `which` = 0 qkv, 1 o, 2 gate_up, 3 down, 4 lm_head (`layer`
 * ignored). `out` holds rows x cols f32. */
int fmd_debug_weight(fmd_handle* h, int32_t layer, int32_t which, float* out, int64_t out_elems);

/* Copy `n` cached K and V rows (kv_heads x head_dim each, act dtype) of one
 * layer of one slot, starting at position `pos`. */
int fmd_debug_kv(fmd_handle* h, int32_t slot, int32_t layer, int32_t pos, int32_t n, void* k_out,
                 void* v_out);

/* Failure detection check (no reference counterpart; the reference has no
 * device-side waits): runs one bounded mbarrier wait, the wait every ring
 * kernel of this library uses, on a barrier nothing arrives on, with at most
 * `limit` tries. The wait gives up, the device status word is set and the
 * call returns FMD_ETIMEDOUT as a step whose wait ran out would; no copy is
 * in flight, so the context and the handle stay usable. */
int fmd_debug_wait_timeout(fmd_handle* h, int32_t limit);

/* Issue cost of a tcgen05.mma (no reference counterpart; a hardware check
 * behind the kernels' design): one CTA issues `iters` MMAs of M 128 x N `n`
 * x K 16 (f16, operands in shared memory) in a bare loop, either from one
 * thread of a diverged warp (`form` 0) or from the elected lane of a warp
 * that runs the loop converged (`form` 1, the form the library's tensor-core
 * kernels use), and *cycles_per_mma receives the SM cycles per MMA from the
 * first issue to the completion of the last: the per-instruction floor that
 * small-N MMAs (the lm_head's 32 rows, attention's 64 keys) run into, and the
 * tensor peak at N 256 (128 cycles). n: a multiple of 16 in [16, 256];
 * iters: a multiple of 8 in [8, 2^20]; the handle must have weights loaded and
 * a KV pool reserved, as for the other debug calls. */
int fmd_debug_mma_issue(fmd_handle* h, int32_t form, int32_t n, int32_t iters, double* cycles_per_mma);

/* Which kernels serve this handle's steps after fmd_kv_reserve (no reference
 * counterpart): bit 0 = decode steps run the persistent layer tail
 * (FMD_LAYER_TAIL=1, Q8_0 weights, max_slots <= 32), bit 1 = mixed steps run
 * the persistent projection GEMM k_proj_tc, bit 2 = the last lm_head launch
 * (or step-graph capture) ran on the tensor cores (Q8_0 lm_head, max_slots
 * <= 64; opt-in with FMD_LM_HEAD_TC=1),
 * bit 3 = prefill attention on persistent CTAs with two query tiles each
 * (FMD_PREFILL_PP=0 selects one CTA per prefill block and kv head), bit 4 =
 * decode-only steps run each half of their rows on its own stream
 * (FMD_DECODE_SPLIT=1, even max_slots >= 16, layer tail off). */
#define FMD_PATH_LAYER_TAIL 1
#define FMD_PATH_PROJ_TC 2
#define FMD_PATH_LM_HEAD_TC 4
#define FMD_PATH_PREFILL_PP 8
#define FMD_PATH_DECODE_SPLIT 16
int fmd_debug_paths(const fmd_handle* h, int32_t* flags);

/* ---- greedy pick without allocation -------------------------------------- */

/* No counterpart in the reference. Greedy ids (per-row argmax, lowest index
 * among equal maxima) of `n_rows` x `vocab` f32 logits that the caller already
 * holds on the current device, written to the caller's device buffer
 * `next_ids` on `stream` (a cudaStream_t; NULL = legacy default stream). No
 * handle, no synchronisation.
 *
 * Who it is for: callers that can't let a library call cudaMalloc or cudaFree,
 * such as a host engine that sizes and owns every device byte itself, or code
 * that must not stall behind the device synchronisation those calls can imply.
 * This entry point allocates nothing. Its scratch is a fixed 128 KiB array
 * compiled into the library, which every GPU that loads the library holds
 * until the process exits.
 *
 * Limits: 1 <= n_rows <= 64 and 1 <= vocab <= 1048576; larger sizes return
 * FMD_EINVAL without launching anything. The first call on each device looks
 * up the scratch's device address with that device current, so make that
 * first call before any stream capture on that device (a call after
 * cudaDeviceReset looks it up again, so the same applies to it). All calls
 * share the one scratch array, which keeps the last call's contents. Each
 * call writes every entry it reads, so nothing needs clearing, but calls
 * whose kernels overlap on the GPU (different streams or host threads) race.
 *
 * Values: NaN logits are never picked. A row whose logits are all -inf gets
 * its first column (0), as np.argmax does; a row with no non-NaN logit gets
 * the id -1, which no vocabulary id equals (the call does not synchronise,
 * so it cannot report this as a status).
 *
 * Errors: if a CUDA error from earlier work is already pending in the calling
 * thread, the call launches nothing, returns FMD_EIO and leaves that error
 * pending for its owner. A failure of the call's own launches returns
 * FMD_EIO and is consumed (cleared) by the call. */
int fmd_greedy_pick_noalloc(const float* logits, int32_t n_rows, int32_t vocab, int32_t* next_ids, void* stream);

/* Host-side GGML Q8_0 quantiser (the `QTensor::quantize` step of
 * linear.rs:197): rows x cols f32 -> rows x cols/32 34-byte blocks. */
int fmd_q8_0_quantize(const float* src, int64_t rows, int64_t cols, void* blocks);

/* The same quantisation on the GPU, for weights already in device memory (a
 * checkpoint uploaded as stored): `src` is rows x cols of FMD_DT_F32, F16 or
 * BF16 (each value taken as its exact f32), `qs` receives rows x cols int8 and
 * `d` rows x cols/32 f16 scales (bit patterns), the structure-of-arrays form of
 * the 34-byte blocks; bit-identical to fmd_q8_0_quantize. All three pointers
 * are device memory; the work is queued on `stream` (a cudaStream_t, NULL =
 * legacy default stream) and the call does not synchronise. cols must be a
 * multiple of 32. */
int fmd_q8_0_quantize_device(const void* src, int32_t src_dtype, int64_t rows, int64_t cols, int8_t* qs,
                             uint16_t* d, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FMD_DECODER_H */
