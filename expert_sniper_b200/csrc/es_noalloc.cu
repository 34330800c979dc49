// es_moe_forward_noalloc: the MoE block forward for callers that cannot
// allocate device memory.
//
// Some hosts of this library own all of the GPU's memory themselves -- an
// inference runtime with a fixed arena, a plugin loaded into a process whose
// allocator forbids outside allocations, or a real-time loop where a
// cudaMalloc (which may synchronise the device) is not allowed. They can pass
// inputs and outputs but not a workspace. This entry point uses a scratch
// buffer that is part of the library image instead: a file-scope __device__
// array, created when the library's module is loaded on a device and held
// there until the process exits.
//
// Limits and behaviour:
//   - the scratch is kNoallocScratchBytes (64 MiB); a call whose workspace
//     (es_moe_workspace_bytes) would exceed it returns ES_ERR_WORKSPACE;
//   - the first call in each CUDA context looks up the array's device
//     address (cudaGetSymbolAddress, with that context's device current) and
//     caches it keyed by the context: a __device__ array's address belongs
//     to the context the module was loaded in, so a host that switches to
//     its own driver-API context, or resets the device, gets the address
//     resolved again rather than a stale one; make the first call in a
//     context before any stream capture on its device;
//   - every call on a device shares the one array and leaves its contents
//     there; the counters that must start at zero are cleared at the start of
//     each call, so calls that overlap on the GPU (different streams, or
//     different host threads) race -- order them on one stream;
//   - device-side error flags land in the shared scratch; each call clears
//     them first, and es_moe_noalloc_read_error reads those of the last call
//     on the current device;
//   - the counters are cleared with three cudaMemsetAsync calls per call
//     (a few microseconds of launch work ahead of the block's kernels);
//   - nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "es_layout.h"
#include "es_moe.h"

namespace {

constexpr size_t kNoallocScratchBytes = size_t(64) << 20;
constexpr int kMaxContexts = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// cuCtxGetCurrent from the driver, looked up once through the runtime.
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

std::mutex g_setup_mu;
CUcontext g_ctx[kMaxContexts] = {};
void* g_scratch_ptr[kMaxContexts] = {};
int g_n_ctx = 0;

// Device address of the scratch array in the current context (resolved once
// per context, after making sure a context is current on this thread).
es_status scratch_in_current_context(void** out) {
  // a thread that has not touched the runtime yet has no current context:
  // cudaSetDevice makes the device's primary context current (it allocates
  // nothing)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ES_ERR_CUDA;
  CtxGetCurrentFn get = ctx_get_current();
  if (!get) return ES_ERR_CUDA;
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS) return ES_ERR_CUDA;
  if (!ctx) {
    if (cudaSetDevice(dev) != cudaSuccess) return ES_ERR_CUDA;
    if (get(&ctx) != CUDA_SUCCESS || !ctx) return ES_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_setup_mu);
  for (int i = 0; i < g_n_ctx; ++i)
    if (g_ctx[i] == ctx) {
      *out = g_scratch_ptr[i];
      return ES_OK;
    }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return ES_ERR_CUDA;
  // a full table (more contexts than kMaxContexts over the process's life)
  // recycles the oldest entry: a context seen again is simply resolved again
  const int slot = g_n_ctx < kMaxContexts ? g_n_ctx++ : 0;
  g_ctx[slot] = ctx;
  g_scratch_ptr[slot] = p;
  *out = p;
  return ES_OK;
}

}  // namespace

extern "C" {

es_status es_moe_forward_noalloc(const es_moe_cfg* cfg, const void* x, const void* logits,
                                 int32_t logits_dtype, const float* cache_bias,
                                 const void* shared_gate_w, const void* packed, void* out,
                                 int32_t out_dtype, int32_t* topk_idx, float* topk_w, int32_t T,
                                 es_stream_t stream) {
  if (!cfg) return ES_ERR_INVALID_ARG;
  size_t need = 0;
  es_status s = es_moe_workspace_bytes(cfg, T, &need);
  if (s != ES_OK) return s;
  if (need > kNoallocScratchBytes) return ES_ERR_WORKSPACE;
  if (T == 0) return ES_OK;
  void* ws = nullptr;
  if ((s = scratch_in_current_context(&ws)) != ES_OK) return s;
  // zero what the kernels expect at zero (the error word, the front-end
  // ticket and work counters, the token bitmaps, the split-K counters): a
  // previous call that stopped early could have left them set. The region
  // sizes come from the workspace carving itself.
  const es::Workspace w = es::carve_workspace(ws, cfg->hidden, cfg->num_experts, cfg->top_k,
                                              cfg->inter, cfg->shared_inter > 0, T);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(w.err, 0, w.zero_ctl_bytes, st) != cudaSuccess ||
      cudaMemsetAsync(w.bitmap, 0, w.zero_bitmap_bytes, st) != cudaSuccess ||
      cudaMemsetAsync(w.counters, 0, w.zero_counter_bytes, st) != cudaSuccess)
    return ES_ERR_CUDA;
  return es_moe_forward(cfg, x, logits, logits_dtype, cache_bias, shared_gate_w, packed, out,
                        out_dtype, topk_idx, topk_w, T, ws, kNoallocScratchBytes, stream);
}

es_status es_moe_noalloc_read_error(int32_t clear, uint32_t* flags_out, es_stream_t stream) {
  if (!flags_out) return ES_ERR_INVALID_ARG;
  void* ws = nullptr;
  const es_status s = scratch_in_current_context(&ws);
  if (s != ES_OK) return s;
  return es_moe_read_error(ws, clear, flags_out, stream);
}

}  // extern "C"
