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
//   - the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current); make that first call
//     before any stream capture on the device;
//   - every call on a device shares the one array and leaves its contents
//     there; the counters that must start at zero are cleared at the start of
//     each call, so calls that overlap on the GPU (different streams, or
//     different host threads) race -- order them on one stream;
//   - device-side error flags land in the shared scratch and are not
//     reported by this entry point;
//   - nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda_runtime.h>

#include <mutex>

#include "es_layout.h"
#include "es_moe.h"

namespace {

constexpr size_t kNoallocScratchBytes = size_t(64) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up once).
es_status scratch_on_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ES_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return ES_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return ES_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
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
  if ((s = scratch_on_current_device(&ws)) != ES_OK) return s;
  // zero what the kernels expect at zero (the error word, the front-end
  // ticket and work counters, the token bitmaps, the split-K counters): a
  // previous call that stopped early could have left them set
  const es::Workspace w = es::carve_workspace(ws, cfg->hidden, cfg->num_experts, cfg->top_k,
                                              cfg->inter, cfg->shared_inter > 0, T);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t ctl = reinterpret_cast<char*>(w.bitmap) - reinterpret_cast<char*>(w.err);
  const size_t bitmap_bytes = (size_t)w.E1 * w.W * 4;
  const long long routed = (long long)T * cfg->top_k < cfg->num_experts
                               ? (long long)T * cfg->top_k
                               : cfg->num_experts;
  const size_t A = (size_t)(routed + (cfg->shared_inter > 0 ? 1 : 0));
  const size_t cnt_gu = A * (cfg->inter / 32), cnt_dn = A * (cfg->hidden / 64);
  const size_t counter_bytes = (cnt_gu > cnt_dn ? cnt_gu : cnt_dn) * 4;
  if (cudaMemsetAsync(w.err, 0, ctl, st) != cudaSuccess ||
      cudaMemsetAsync(w.bitmap, 0, bitmap_bytes, st) != cudaSuccess ||
      cudaMemsetAsync(w.counters, 0, counter_bytes, st) != cudaSuccess)
    return ES_ERR_CUDA;
  return es_moe_forward(cfg, x, logits, logits_dtype, cache_bias, shared_gate_w, packed, out,
                        out_dtype, topk_idx, topk_w, T, ws, kNoallocScratchBytes, stream);
}

}  // extern "C"
