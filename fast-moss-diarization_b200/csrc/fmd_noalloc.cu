// Greedy pick over logits the caller already holds on the device, without
// allocating any device memory.
//
// Some callers can't let a library call cudaMalloc/cudaFree. A host engine
// that sizes and owns every device byte itself has that rule, and so does
// code that must not stall behind the device synchronisation those calls can
// imply. This entry point serves them: it needs only the caller's logits and
// output buffers plus a fixed scratch array that lives in the library's
// device image for as long as the process runs.
//
// Each row is split across up to kMaxParts CTAs. Each CTA writes its best
// (value, index) candidate into the scratch array, and a second kernel
// reduces the candidates of each row. Ties resolve to the lowest index, as
// in the decode step's greedy pick. NaN logits are never picked; a row of
// -inf values picks its first column (as np.argmax does); a row with no
// non-NaN value gets the id -1.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>

#include <mutex>

#include "../../include/fmd_decoder.h"

namespace {

constexpr int kMaxRows = 64;        // rows per call
constexpr int kMaxParts = 256;      // candidate CTAs per row
constexpr int kSliceCols = 4096;    // logits scanned by one candidate CTA
constexpr int kMaxVocab = kMaxParts * kSliceCols;  // 1,048,576 columns
constexpr int kMaxDevices = 64;
constexpr int kNone = 0x7fffffff;   // candidate index of "no non-NaN value seen"

struct Candidate {
  float value;
  int index;
};

// The scratch: kMaxRows x kMaxParts candidates = 128 KiB on every GPU that
// loads the library, held until the process exits. Each call writes every
// entry it later reads, so nothing needs clearing between calls.
static __device__ __align__(256) Candidate g_pick_scratch[kMaxRows * kMaxParts];

// Device address of g_pick_scratch per device ordinal, looked up with that
// device current, together with the unique id of the CUDA context it belongs
// to. In host code the symbol's name is only a host-side stand-in, so kernels
// always receive this looked-up address. A new context on the device (after
// cudaDeviceReset) has a new id, which triggers a fresh lookup.
struct ScratchEntry {
  Candidate* addr = nullptr;
  unsigned long long ctx_id = 0;
};
ScratchEntry g_scratch[kMaxDevices];
std::mutex g_scratch_mutex;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__global__ void __launch_bounds__(256) k_pick_partial(const float* __restrict__ logits, int vocab, int parts,
                                                      Candidate* __restrict__ scratch) {
  __shared__ Candidate red[8];
  const int row = blockIdx.y, part = blockIdx.x;
  const float* x = logits + (size_t)row * vocab;
  const int c0 = part * kSliceCols;
  const int c1 = min(vocab, c0 + kSliceCols);
  float best = -INFINITY;
  int bi = kNone;
  for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
    const float v = x[c];
    // columns ascend per thread: strict > keeps the first maximum; the first
    // non-NaN value is always taken, so a row of -inf keeps its first column
    if (v > best || (bi == kNone && v == v)) {
      best = v;
      bi = c;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = Candidate{best, bi};
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (better(red[w].value, red[w].index, best, bi)) {
        best = red[w].value;
        bi = red[w].index;
      }
    scratch[row * parts + part] = Candidate{best, bi};
  }
}

__global__ void __launch_bounds__(32) k_pick_final(const Candidate* __restrict__ scratch, int parts,
                                                   int32_t* __restrict__ next_ids) {
  const int row = blockIdx.x;
  float best = -INFINITY;
  int bi = kNone;
  for (int p = threadIdx.x; p < parts; p += 32) {
    const Candidate c = scratch[row * parts + p];
    if (better(c.value, c.index, best, bi)) {
      best = c.value;
      bi = c.index;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  // every value of the row was NaN: a sentinel no vocabulary id can equal
  if (threadIdx.x == 0) next_ids[row] = bi == kNone ? -1 : bi;
}

// Driver entry points used to tell one CUDA context of a device from the next.
bool ctx_fns(CtxGetCurrentFn* cur, CtxGetIdFn* id) {
  static CtxGetCurrentFn s_cur = nullptr;
  static CtxGetIdFn s_id = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* f = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      s_cur = reinterpret_cast<CtxGetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      s_id = reinterpret_cast<CtxGetIdFn>(f);
  }
  *cur = s_cur;
  *id = s_id;
  return s_cur != nullptr && s_id != nullptr;
}

// Unique id of the context current on this thread, 0 if there is none.
unsigned long long current_ctx_id(CtxGetCurrentFn cur, CtxGetIdFn id) {
  CUcontext c = nullptr;
  if (cur(&c) != CUDA_SUCCESS || c == nullptr) return 0;
  unsigned long long v = 0;
  return id(c, &v) == CUDA_SUCCESS ? v : 0;
}

// The device address of the scratch array for the current device and
// context: looked up once per context (with that device current), then
// served from the cache.
int scratch_for_current_device(Candidate** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return FMD_EIO;
  if (dev < 0 || dev >= kMaxDevices) return FMD_EINVAL;
  CtxGetCurrentFn cur;
  CtxGetIdFn idf;
  if (!ctx_fns(&cur, &idf)) return FMD_EIO;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchEntry& e = g_scratch[dev];
  const unsigned long long now = current_ctx_id(cur, idf);
  if (e.addr == nullptr || now == 0 || now != e.ctx_id) {
    void* p = nullptr;
    // creates the device's primary context if this thread has none yet
    if (cudaGetSymbolAddress(&p, g_pick_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // the lookup's own failure; nothing else was pending
      return FMD_EIO;
    }
    e.addr = static_cast<Candidate*>(p);
    e.ctx_id = current_ctx_id(cur, idf);
  }
  *out = e.addr;
  return FMD_OK;
}

}  // namespace

extern "C" int fmd_greedy_pick_noalloc(const float* logits, int32_t n_rows, int32_t vocab, int32_t* next_ids,
                                       void* stream) {
  if (logits == nullptr || next_ids == nullptr) return FMD_EINVAL;
  if (n_rows < 1 || n_rows > kMaxRows || vocab < 1 || vocab > kMaxVocab) return FMD_EINVAL;
  // An error left pending by earlier work in this thread is not this call's:
  // refuse to launch and leave it in place for its owner.
  if (cudaPeekAtLastError() != cudaSuccess) return FMD_EIO;
  Candidate* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != FMD_OK) return rc;
  const int parts = (vocab + kSliceCols - 1) / kSliceCols;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  k_pick_partial<<<dim3(parts, n_rows), 256, 0, s>>>(logits, vocab, parts, scratch);
  if (cudaGetLastError() != cudaSuccess) return FMD_EIO;  // this launch's error, consumed
  k_pick_final<<<n_rows, 32, 0, s>>>(scratch, parts, next_ids);
  if (cudaGetLastError() != cudaSuccess) return FMD_EIO;
  return FMD_OK;
}
