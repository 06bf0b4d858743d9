// Launchers of the audio tower (Whisper encoder + VQ adaptor) kernels.
#pragma once

#include <cuda.h>

#include "fmd_kernels.cuh"

namespace fmd {

// Fused epilogues of the encoder GEMM, v = acc + bias[n]:
enum EncEpi : int {
  kEpiQkv = 0,      // out_T = v * (n < q_cols ? scale_q : n < scale_cols ? scale : 1)  (q, k scaling)
  kEpiGelu = 1,     // out_T = gelu_erf(v)                         (conv1, fc1)
  kEpiResid = 2,    // out_f32 += v                                (out_proj, fc2: residual adds)
  kEpiGeluPos = 3,  // out_f32 = gelu_erf(v) + pos[m % period][n]  (conv2 + learned positions)
  kEpiSilu = 4,     // out_T = silu(v)                             (adaptor layers.0)
  kEpiF32 = 5,      // out_f32 = v                                 (adaptor layers.2, before its norm)
};

struct EncEpiArgs {
  const float* bias = nullptr;  // [N] or null
  void* out = nullptr;          // [M][N], act dtype or f32 by epilogue
  const float* pos = nullptr;   // [period][N] (kEpiGeluPos)
  int period = 1;
  int q_cols = 0;
  int scale_cols = 0;
  float scale_q = 1.f;
  float scale = 1.f;
};

cudaError_t init_enc_kernels();

// Tile width of the encoder GEMM for N output features (0: unsupported N).
int enc_gemm_bn(int N);
// 2D map over a row-major [rows][cols] 16-bit matrix with the 128-byte
// swizzle, box {64, box_rows}.
bool enc_make_map2(void* encode_fn, CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                   uint32_t box_rows);
// 3D map over [chunks][rows][cols] (16-bit), box {64, 64, 1}: reads past a
// chunk's last row are zero-filled instead of reaching the next chunk.
bool enc_make_map3(void* encode_fn, CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                   uint64_t chunks);

// out = epilogue(A[M][K] . B[N][K]^T); amap box {64, 128}, bmap box {64, bn}.
// K a multiple of 64, N a multiple of bn.
void launch_enc_gemm(ActType at, int epi, const CUtensorMap& amap, const CUtensorMap& bmap, int bn, int M, int N,
                     int K, const EncEpiArgs& ep, int* status, cudaStream_t s);

// Bidirectional attention of every (chunk, head): qkv [chunks * frames][3 D]
// (q | k | v; k pre-scaled by head_dim^-1/4, q by head_dim^-1/4 x log2(e), so the
// scores come out in the exp2 domain), through `qkv_map` (enc_make_map3 over it);
// ctx [chunks * frames][D]. head_dim 64.
void launch_enc_attn(ActType at, const CUtensorMap& qkv_map, int n_chunks, int frames, int D, int heads, void* ctx,
                     int* status, cudaStream_t s);

// conv1 operand: a1[b * F + t][k * n_mels + c] = mel[b][c][t + k - 1] (0 off
// the ends), columns [3 n_mels, kp) zero. mel_dt FMD_DT_F32 or the act dtype.
void launch_im2col_mel(ActType at, const void* mel, int mel_dt, int n_chunks, int n_mels, int n_frames, int kp,
                       void* a1, cudaStream_t s);
// conv2 operand: a2[b * F/2 + t][k * D + c] = x1[b * F + 2 t + k - 1][c] (0 off the ends).
void launch_im2col_conv2(ActType at, const void* x1, int n_chunks, int n_frames, int D, void* a2, cudaStream_t s);

// out[dst] = layer_norm(x[src]) * w + b over rows of D (a multiple of 128,
// <= 2048) f32 values; rowmap[i] = {src, dst} (null: row i -> row i).
void launch_layernorm(ActType at, const float* x, const int2* rowmap, int rows, int D, const float* w,
                      const float* b, float eps, void* out, cudaStream_t s);

// Host dtype (FMD_DT_F32 / F16 / BF16) -> act dtype or f32, on the device.
void launch_convert_act(ActType at, const void* src, int src_dt, size_t n, void* dst, cudaStream_t s);
void launch_convert_f32(const void* src, int src_dt, size_t n, float* dst, cudaStream_t s);
// conv weight (O, C, 3) -> act [O][kp] with column k * C + c = w[o][c][k], zero pad.
void launch_conv_weight(ActType at, const void* src, int src_dt, int O, int C, int kp, void* dst, cudaStream_t s);

}  // namespace fmd
