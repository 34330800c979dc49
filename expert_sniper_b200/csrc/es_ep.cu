// Expert-parallel helpers: per-destination routing masks and the fixed-order
// sum of per-owner partials.
//
// The reference's Expert Network broadcasts each layer's request to every
// node; a node masks the top-k weights to its own partition and returns a
// partial (src/expert_network/node.py:142-172), and the driver sums the
// partials in fixed node order in fp32 (src/expert_network/reader.py:
// 278-286). Here the home GPU computes each destination's mask once
// (es_ep_mask), the owners run es_moe_expert_ffn on the rows they receive,
// and es_ep_combine adds the returned partials in rank order.
#include "es_common.cuh"
#include "es_kernels.cuh"
#include "es_moe.h"

#include <string.h>

namespace es {
namespace {

// one thread per (destination, token, slot)
__global__ void ep_mask_kernel(const int32_t* idx, const float* w, const int32_t* owner,
                               const int32_t* local_id, int E, int k, int T, int world,
                               int32_t* send_idx, float* send_w, uint32_t* err) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)world * T * k;
  pdl_wait();
  pdl_trigger();
  if (i >= total) return;
  const int d = (int)(i / ((long long)T * k));
  const long long tj = i - (long long)d * T * k;
  const int e = idx[tj];
  int l = -1;
  if (e >= 0 && e < E) {
    if (owner[e] == d) l = local_id[e];
  } else if (e != -1) {
    set_error(err, 0x1u);
  }
  send_idx[i] = l;
  send_w[i] = w[tj];
}

// out[t][c] = sum over ranks r in order of partials[r][t][c] (+ extra[t][c])
__global__ void ep_combine_kernel(const float* partials, const float* extra, int world, int T,
                                  int D, void* out, int out_f32) {
  const long long i4 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const long long n = (long long)T * D;
  pdl_wait();
  pdl_trigger();
  if (i4 >= n) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = 0; r < world; ++r) {
    const float4 p = *reinterpret_cast<const float4*>(partials + (size_t)r * n + i4);
    acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
  }
  if (extra) {
    const float4 p = *reinterpret_cast<const float4*>(extra + i4);
    acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
  }
  if (out_f32) {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + i4) = acc;
  } else {
    const uint32_t lo = (uint32_t)float_to_bf16_bits(acc.x) | ((uint32_t)float_to_bf16_bits(acc.y) << 16);
    const uint32_t hi = (uint32_t)float_to_bf16_bits(acc.z) | ((uint32_t)float_to_bf16_bits(acc.w) << 16);
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + i4) = make_uint2(lo, hi);
  }
}

// ---------------------------------------------------------------------------
// Peer-to-peer exchange (es_ep_dispatch / receive / return / combine_p2p).
// A rank writes into other ranks' windows with plain stores over NVLink
// (the windows are CUDA IPC mappings), then publishes a step number with a
// system-scope release store; the reader polls it with system-scope acquire
// loads. Producers of one flag are several CTAs: each makes its stores
// visible system-wide (fence) before taking a ticket, and the CTA that takes
// the last ticket fences again and releases the flag.
// ---------------------------------------------------------------------------
constexpr uint32_t kDevErrTimeout = 0x8u;
constexpr int kEpThreads = 256;
constexpr int kDispatchTok = 8;   // home tokens per dispatch CTA
constexpr int kRecvRows = 64;     // received rows per receive CTA
constexpr int kReturnRows = 4;    // rows per return CTA

struct EpArgs {
  int world, rank, cap, D, k, E;
  const int32_t* owner;
  const int32_t* local_id;
  void* const* peers;
  void* window;
  uint32_t* err;
};

ES_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
ES_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

// Waits until *flag has reached step e (wrap-safe), for about a second.
ES_DEV bool wait_step(const uint32_t* flag, uint32_t e) {
  if ((int)(ld_acquire_sys(flag) - e) >= 0) return true;
  const long long t0 = clock64();
  while ((int)(ld_acquire_sys(flag) - e) < 0) {
    if (clock64() - t0 > (1LL << 31)) return false;
    __nanosleep(256);
  }
  return true;
}

// Does token t have a slot owned by rank d?
ES_DEV bool token_uses(const EpArgs& a, const int32_t* idx, int t, int d) {
  for (int j = 0; j < a.k; ++j) {
    const int e = idx[(size_t)t * a.k + j];
    if (e >= 0 && e < a.E && a.owner[e] == d) return true;
  }
  return false;
}

// Last of `n` CTAs to arrive on `ticket` (called by one thread after its
// CTA's stores; the fence makes them visible system-wide first).
ES_DEV bool last_cta(int* ticket, int n) {
  __threadfence_system();
  const int tk = atomicAdd(ticket, 1);
  if (tk != n - 1) return false;
  __threadfence_system();
  *ticket = 0;
  return true;
}

// grid (world destinations, chunks of kDispatchTok home tokens)
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(EpArgs a, const uint16_t* x,
                                                                 const int32_t* idx,
                                                                 const float* w, int T) {
  __shared__ int s_before, s_total;
  __shared__ uint32_t s_bits;
  const int d = blockIdx.x, c = blockIdx.y, tid = threadIdx.x;
  EpWindow me = carve_ep_window(a.window, a.world, a.cap, a.D, a.k);
  EpWindow peer = carve_ep_window(a.peers[d], a.world, a.cap, a.D, a.k);
  const uint32_t e = *me.epoch + 1;
  const int t0 = c * kDispatchTok;
  // tokens of this destination before the chunk, and in total
  int before = 0, total = 0;
  for (int base = 0; base < T; base += kEpThreads) {
    const int t = base + tid;
    const bool use = t < T && token_uses(a, idx, t, d);
    before += __syncthreads_count(use && t < t0);
    total += __syncthreads_count(use);
  }
  if (tid < 32) {
    const int t = t0 + tid;
    const bool use = tid < kDispatchTok && t < T && token_uses(a, idx, t, d);
    const uint32_t bits = __ballot_sync(0xffffffffu, use);
    if (tid == 0) { s_bits = bits; s_before = before; s_total = total; }
  }
  __syncthreads();
  const uint32_t bits = s_bits;
  const size_t src_row0 = (size_t)a.rank * a.cap;
  const int chunks = a.D / 8;   // 16-byte pieces per row
  for (int i = 0; i < kDispatchTok; ++i) {
    if (!((bits >> i) & 1u)) continue;
    const int t = t0 + i;
    const int pos = s_before + __popc(bits & ((1u << i) - 1u));
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * a.D);
    uint4* dst = reinterpret_cast<uint4*>(peer.rows_in + (src_row0 + pos) * a.D);
    for (int q = tid; q < chunks; q += kEpThreads) dst[q] = src[q];
    if (tid < a.k) {
      const int eid = idx[(size_t)t * a.k + tid];
      const bool mine = eid >= 0 && eid < a.E && a.owner[eid] == d;
      peer.idx_in[(src_row0 + pos) * a.k + tid] = mine ? a.local_id[eid] : -1;
      peer.w_in[(src_row0 + pos) * a.k + tid] = w[(size_t)t * a.k + tid];
    }
    if (tid == 0) peer.tok_in[src_row0 + pos] = t;
  }
  __syncthreads();
  if (tid == 0 && last_cta(&me.tickets[d], gridDim.y)) {
    peer.cnt_in[a.rank] = s_total;
    __threadfence_system();
    st_release_sys(&peer.flags_in[a.rank], e);
  }
}

// grid (world sources, chunks of kRecvRows rows)
__global__ void __launch_bounds__(kEpThreads) ep_receive_kernel(EpArgs a, int32_t* idx_out,
                                                                float* w_out) {
  __shared__ int s_cnt;
  const int s = blockIdx.x, tid = threadIdx.x;
  EpWindow me = carve_ep_window(a.window, a.world, a.cap, a.D, a.k);
  const uint32_t e = *me.epoch + 1;
  if (tid == 0) {
    int cnt = 0;
    if (wait_step(&me.flags_in[s], e)) {
      cnt = __ldcg(&me.cnt_in[s]);
      cnt = cnt < 0 ? 0 : (cnt > a.cap ? a.cap : cnt);
    } else {
      atomicOr(a.err, kDevErrTimeout);
    }
    s_cnt = cnt;
  }
  __syncthreads();
  const int cnt = s_cnt;
  const int r0 = blockIdx.y * kRecvRows;
  for (int i = tid; i < kRecvRows * a.k; i += kEpThreads) {
    const int r = r0 + i / a.k, j = i % a.k;
    if (r >= a.cap) break;
    const size_t o = ((size_t)s * a.cap + r) * a.k + j;
    const bool live = r < cnt;
    idx_out[o] = live ? __ldcg(me.idx_in + o) : -1;
    w_out[o] = live ? __ldcg(me.w_in + o) : 0.f;
  }
}

// grid (world sources, chunks of kReturnRows rows): partials back home
__global__ void __launch_bounds__(kEpThreads) ep_return_kernel(EpArgs a, const float* y) {
  const int s = blockIdx.x, tid = threadIdx.x;
  EpWindow me = carve_ep_window(a.window, a.world, a.cap, a.D, a.k);
  EpWindow home = carve_ep_window(a.peers[s], a.world, a.cap, a.D, a.k);
  const uint32_t e = *me.epoch + 1;
  int cnt = __ldcg(&me.cnt_in[s]);
  cnt = cnt < 0 ? 0 : (cnt > a.cap ? a.cap : cnt);
  const int chunks = a.D / 4;
  for (int i = 0; i < kReturnRows; ++i) {
    const int r = blockIdx.y * kReturnRows + i;
    if (r >= cnt) break;
    const int t = __ldcg(&me.tok_in[(size_t)s * a.cap + r]);
    if (t < 0 || t >= a.cap) continue;
    const float4* src = reinterpret_cast<const float4*>(y + ((size_t)s * a.cap + r) * a.D);
    float4* dst = reinterpret_cast<float4*>(home.ret_in + ((size_t)a.rank * a.cap + t) * a.D);
    for (int q = tid; q < chunks; q += kEpThreads) dst[q] = src[q];
  }
  __syncthreads();
  if (tid == 0 && last_cta(&me.tickets[a.world + s], gridDim.y))
    st_release_sys(&home.flags_ret[a.rank], e);
}

// grid (T, column blocks of 4 * kEpThreads): fixed rank-order sum
__global__ void __launch_bounds__(kEpThreads) ep_combine_p2p_kernel(EpArgs a,
                                                                    const int32_t* idx,
                                                                    const float* extra, int T,
                                                                    void* out, int out_f32) {
  __shared__ uint32_t s_mask;
  __shared__ int s_ok;
  const int t = blockIdx.x, tid = threadIdx.x;
  EpWindow me = carve_ep_window(a.window, a.world, a.cap, a.D, a.k);
  const uint32_t e = *me.epoch + 1;
  if (tid == 0) {
    bool ok = true;
    for (int d = 0; d < a.world && ok; ++d) ok = wait_step(&me.flags_ret[d], e);
    if (!ok) atomicOr(a.err, kDevErrTimeout);
    uint32_t m = 0;
    for (int j = 0; j < a.k; ++j) {
      const int eid = idx[(size_t)t * a.k + j];
      if (eid >= 0 && eid < a.E) m |= 1u << a.owner[eid];
    }
    s_mask = m;
    s_ok = ok;
  }
  __syncthreads();
  const uint32_t m = s_ok ? s_mask : 0u;
  const int c4 = (blockIdx.y * kEpThreads + tid) * 4;
  if (c4 < a.D) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int d = 0; d < a.world; ++d) {
      if (!((m >> d) & 1u)) continue;
      const float4 p = __ldcg(reinterpret_cast<const float4*>(
          me.ret_in + ((size_t)d * a.cap + t) * a.D + c4));
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    if (extra) {
      const float4 p = *reinterpret_cast<const float4*>(extra + (size_t)t * a.D + c4);
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    if (out_f32) {
      *reinterpret_cast<float4*>(static_cast<float*>(out) + (size_t)t * a.D + c4) = acc;
    } else {
      const uint32_t lo = (uint32_t)float_to_bf16_bits(acc.x) | ((uint32_t)float_to_bf16_bits(acc.y) << 16);
      const uint32_t hi = (uint32_t)float_to_bf16_bits(acc.z) | ((uint32_t)float_to_bf16_bits(acc.w) << 16);
      *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + (size_t)t * a.D + c4) = make_uint2(lo, hi);
    }
  }
  __syncthreads();
  if (tid == 0 && last_cta(&me.tickets[2 * a.world], gridDim.x * gridDim.y)) *me.epoch = e;
}

}  // namespace
}  // namespace es

extern "C" {

es_status es_ep_mask(const int32_t* topk_idx, const float* topk_w, const int32_t* owner,
                     const int32_t* local_id, int32_t num_experts, int32_t top_k, int32_t T,
                     int32_t world, int32_t* send_idx, float* send_w, void* workspace,
                     es_stream_t stream) {
  if (T < 0 || world < 1 || top_k < 1 || top_k > 16 || num_experts < 1) return ES_ERR_INVALID_ARG;
  if (T == 0) return ES_OK;
  if (!topk_idx || !topk_w || !owner || !local_id || !send_idx || !send_w) return ES_ERR_INVALID_ARG;
  const long long total = (long long)world * T * top_k;
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  if (blocks > 0x7fffffffLL) return ES_ERR_UNSUPPORTED;
  uint32_t* err = static_cast<uint32_t*>(workspace);  // error word at offset 0, or NULL
  return es::launch_pdl(es::ep_mask_kernel, dim3((unsigned)blocks), dim3(threads), 0,
                        static_cast<cudaStream_t>(stream), topk_idx, topk_w, owner, local_id,
                        (int)num_experts, (int)top_k, (int)T, (int)world, send_idx, send_w, err) ==
                 cudaSuccess
             ? ES_OK
             : ES_ERR_CUDA;
}

es_status es_ep_combine(const float* partials, const float* extra, int32_t world, int32_t T,
                        int32_t D, void* out, int32_t out_dtype, es_stream_t stream) {
  if (world < 1 || T < 0 || D <= 0 || D % 4) return ES_ERR_INVALID_ARG;
  if (out_dtype != ES_DTYPE_BF16 && out_dtype != ES_DTYPE_F32) return ES_ERR_UNSUPPORTED;
  if (T == 0) return ES_OK;
  if (!partials || !out) return ES_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(partials) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(extra)) % 16)
    return ES_ERR_INVALID_ARG;
  const long long n4 = (long long)T * D / 4;
  const int threads = 256;
  const long long blocks = (n4 + threads - 1) / threads;
  return es::launch_pdl(es::ep_combine_kernel, dim3((unsigned)blocks), dim3(threads), 0,
                        static_cast<cudaStream_t>(stream), partials, extra, (int)world, (int)T,
                        (int)D, out, out_dtype == ES_DTYPE_F32 ? 1 : 0) == cudaSuccess
             ? ES_OK
             : ES_ERR_CUDA;
}


// ---- peer-to-peer exchange ------------------------------------------------

static es_status ep_args(const es_ep_plan* p, es::EpArgs* a) {
  if (!p || !p->peers || !p->window || !p->owner || !p->local_id || !p->err)
    return ES_ERR_INVALID_ARG;
  if (p->world < 1 || p->world > 32 || p->rank < 0 || p->rank >= p->world || p->cap < 1 ||
      p->hidden <= 0 || p->hidden % 8 || p->top_k < 1 || p->top_k > 16 || p->num_experts < 1)
    return ES_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(p->window) % 256) return ES_ERR_INVALID_ARG;
  a->world = p->world; a->rank = p->rank; a->cap = p->cap; a->D = p->hidden; a->k = p->top_k;
  a->E = p->num_experts; a->owner = p->owner; a->local_id = p->local_id; a->peers = p->peers;
  a->window = p->window; a->err = p->err;
  return ES_OK;
}

static es_status launch_status(cudaError_t e) { return e == cudaSuccess ? ES_OK : ES_ERR_CUDA; }

es_status es_ep_window_bytes(int32_t world, int32_t cap, int32_t hidden, int32_t top_k,
                             size_t* bytes_out) {
  if (!bytes_out || world < 1 || world > 32 || cap < 1 || hidden <= 0 || hidden % 8 ||
      top_k < 1 || top_k > 16)
    return ES_ERR_INVALID_ARG;
  *bytes_out = es::carve_ep_window(nullptr, world, cap, hidden, top_k).bytes;
  return ES_OK;
}

es_status es_ep_window_alloc(size_t bytes, void** window_out, void* ipc_handle_out) {
  if (!bytes || !window_out || !ipc_handle_out) return ES_ERR_INVALID_ARG;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handle");
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return ES_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return ES_ERR_CUDA;
  }
  memcpy(ipc_handle_out, &h, sizeof(h));
  *window_out = p;
  return ES_OK;
}

es_status es_ep_window_open(const void* ipc_handle, void** window_out) {
  if (!ipc_handle || !window_out) return ES_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return ES_ERR_CUDA;
  *window_out = p;
  return ES_OK;
}

es_status es_ep_window_close(void* peer_window) {
  if (!peer_window) return ES_ERR_INVALID_ARG;
  return launch_status(cudaIpcCloseMemHandle(peer_window));
}

es_status es_ep_window_free(void* window) {
  if (!window) return ES_ERR_INVALID_ARG;
  return launch_status(cudaFree(window));
}

es_status es_ep_dispatch(const es_ep_plan* plan, const void* x_bf16, const int32_t* topk_idx,
                         const float* topk_w, int32_t T, es_stream_t stream) {
  es::EpArgs a{};
  es_status s = ep_args(plan, &a);
  if (s != ES_OK) return s;
  if (T < 0 || T > a.cap) return ES_ERR_INVALID_ARG;
  if (T > 0 && (!x_bf16 || !topk_idx || !topk_w)) return ES_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(x_bf16) % 16) return ES_ERR_INVALID_ARG;
  // every destination gets its flag, also for an empty batch
  const int chunks = T > 0 ? (T + es::kDispatchTok - 1) / es::kDispatchTok : 1;
  es::ep_dispatch_kernel<<<dim3(a.world, chunks), es::kEpThreads, 0,
                           static_cast<cudaStream_t>(stream)>>>(
      a, static_cast<const uint16_t*>(x_bf16), topk_idx, topk_w, T);
  return launch_status(cudaGetLastError());
}

es_status es_ep_receive(const es_ep_plan* plan, int32_t* idx_out, float* w_out,
                        es_stream_t stream) {
  es::EpArgs a{};
  es_status s = ep_args(plan, &a);
  if (s != ES_OK) return s;
  if (!idx_out || !w_out) return ES_ERR_INVALID_ARG;
  const int chunks = (a.cap + es::kRecvRows - 1) / es::kRecvRows;
  es::ep_receive_kernel<<<dim3(a.world, chunks), es::kEpThreads, 0,
                          static_cast<cudaStream_t>(stream)>>>(a, idx_out, w_out);
  return launch_status(cudaGetLastError());
}

es_status es_ep_rows_offset(const es_ep_plan* plan, size_t* offset_out) {
  es::EpArgs a{};
  es_status s = ep_args(plan, &a);
  if (s != ES_OK) return s;
  if (!offset_out) return ES_ERR_INVALID_ARG;
  char* base = reinterpret_cast<char*>(uintptr_t(1) << 20);
  const es::EpWindow w = es::carve_ep_window(base, a.world, a.cap, a.D, a.k);
  *offset_out = reinterpret_cast<char*>(w.rows_in) - base;
  return ES_OK;
}

es_status es_ep_return(const es_ep_plan* plan, const float* y, es_stream_t stream) {
  es::EpArgs a{};
  es_status s = ep_args(plan, &a);
  if (s != ES_OK) return s;
  if (!y || reinterpret_cast<uintptr_t>(y) % 16 || a.D % 4) return ES_ERR_INVALID_ARG;
  const int chunks = (a.cap + es::kReturnRows - 1) / es::kReturnRows;
  es::ep_return_kernel<<<dim3(a.world, chunks), es::kEpThreads, 0,
                         static_cast<cudaStream_t>(stream)>>>(a, y);
  return launch_status(cudaGetLastError());
}

es_status es_ep_combine_p2p(const es_ep_plan* plan, const int32_t* topk_idx, const float* extra,
                            int32_t T, void* out, int32_t out_dtype, es_stream_t stream) {
  es::EpArgs a{};
  es_status s = ep_args(plan, &a);
  if (s != ES_OK) return s;
  if (T < 0 || T > a.cap || a.D % 4) return ES_ERR_INVALID_ARG;
  if (out_dtype != ES_DTYPE_BF16 && out_dtype != ES_DTYPE_F32) return ES_ERR_UNSUPPORTED;
  if (T == 0) return ES_ERR_INVALID_ARG;  // the step counter advances in this kernel
  if (!topk_idx || !out) return ES_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(extra)) % 16)
    return ES_ERR_INVALID_ARG;
  const int cb = (a.D / 4 + es::kEpThreads - 1) / es::kEpThreads;
  es::ep_combine_p2p_kernel<<<dim3(T, cb), es::kEpThreads, 0,
                              static_cast<cudaStream_t>(stream)>>>(
      a, topk_idx, extra, T, out, out_dtype == ES_DTYPE_F32 ? 1 : 0);
  return launch_status(cudaGetLastError());
}

}  // extern "C"
