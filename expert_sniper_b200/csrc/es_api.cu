// C ABI of the MoE block (include/es_moe.h): argument checks, workspace
// carving and kernel launches. No allocation, no host synchronisation except
// in es_moe_read_error.
#include <cuda_runtime.h>

#include "es_kernels.cuh"
#include "es_moe.h"

namespace {

using es::Workspace;

es_status check_cfg(const es_moe_cfg* c) {
  if (!c) return ES_ERR_INVALID_ARG;
  if (c->group_size != 64 || c->bits != 4) return ES_ERR_UNSUPPORTED;
  if (c->hidden <= 0 || c->inter <= 0 || c->num_experts <= 0 || c->top_k <= 0)
    return ES_ERR_INVALID_ARG;
  // gate/up CTAs give each warp 4 groups of D; down warps hold I/64 tiles
  const int nw = c->hidden / 256;
  if (c->hidden % 256 || !(nw == 1 || nw == 2 || nw == 3 || nw == 4 || nw == 6 || nw == 8 ||
                           nw == 12 || nw == 16))
    return ES_ERR_UNSUPPORTED;
  const int kg = c->inter / 64;
  if (c->inter % 64 || !(kg == 4 || kg == 8 || kg == 12 || kg == 16 || kg == 24 || kg == 32))
    return ES_ERR_UNSUPPORTED;
  if (c->num_experts > es::kMaxExperts) return ES_ERR_UNSUPPORTED;
  if (c->top_k > es::kMaxTopK) return ES_ERR_UNSUPPORTED;
  if (c->shared_inter != 0 && c->shared_inter != c->inter) return ES_ERR_UNSUPPORTED;
  if (c->kernel_path < 0 || c->kernel_path > 4) return ES_ERR_INVALID_ARG;
  if (c->x_dtype != ES_DTYPE_BF16 && c->x_dtype != ES_DTYPE_F16) return ES_ERR_UNSUPPORTED;
  // the decode kernels and the fused tiny-batch kernel read bf16 activations only
  if (c->x_dtype == ES_DTYPE_F16 && (c->kernel_path == 1 || c->kernel_path == 4))
    return ES_ERR_UNSUPPORTED;
  return ES_OK;
}

// Which expert-FFN kernels run: 0 = the register-operand decode kernels,
// 1 = tensor-core GEMMs with 128-token tiles (A in shared memory), 2 = tensor-
// core GEMMs with 32-token tiles (A in tensor memory). Automatic, by the
// average (token, expert) pairs per routed expert p = T k / E (and T >= 64):
// decode below p = 4, 32-token tiles up to p = 48, 128-token tiles above --
// the crossovers measured on a B200 for the Qwen3-30B and Qwen3-Next layers.
enum { kFfnDecode = 0, kFfnTensorLarge = 1, kFfnTensorSmall = 2, kFfnFused = 3 };
constexpr long long kFoldScatterSlots = 8192;
int ffn_variant(const es_moe_cfg* c, int T) {
  const bool fused_fits = c->x_dtype == ES_DTYPE_BF16 &&
                          es::small_path_fits(T, c->hidden, c->inter, c->num_experts, c->top_k,
                                              c->shared_inter > 0);
  if (c->kernel_path == 4) return fused_fits ? kFfnFused : kFfnDecode;
  if (c->kernel_path == 3) return kFfnTensorSmall;
  if (c->kernel_path == 2) return kFfnTensorLarge;
  if (c->kernel_path == 1) return kFfnDecode;  // (fp16 x is rejected with path 1)
  const long long pk = (long long)T * c->top_k;
  if (T >= 64 && pk > 48LL * c->num_experts) return kFfnTensorLarge;
  if (T >= 64 && pk >= 4LL * c->num_experts) return kFfnTensorSmall;
  // fp16 activations are read by the tensor-core kernels only
  if (c->x_dtype == ES_DTYPE_F16) return kFfnTensorSmall;
  return fused_fits ? kFfnFused : kFfnDecode;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

es_status cuda_status(cudaError_t e) { return e == cudaSuccess ? ES_OK : ES_ERR_CUDA; }

// Optional per-kernel instrumentation: events[i] is recorded before kernel i
// (router, dispatch, gate/up, down, combine) and events[5] after the last.
struct Marks {
  void* const* ev = nullptr;
  cudaError_t mark(int i, cudaStream_t st) const {
    if (!ev) return cudaSuccess;
    // under stream capture the record must become an event-record node of
    // the graph (cudaEventRecordExternal), so it fires on every replay
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(st, &cs);
    if (e != cudaSuccess) return e;
    cudaEvent_t h = static_cast<cudaEvent_t>(ev[i]);
    return cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(h, st, cudaEventRecordExternal)
                                               : cudaEventRecord(h, st);
  }
};

es::DispatchArgs dispatch_args(const es_moe_cfg* cfg, const Workspace& w, const int32_t* idx,
                               const float* wts, int T) {
  es::DispatchArgs d{};
  d.bitmap = w.bitmap; d.idx = idx; d.w = wts; d.T = T; d.E = cfg->num_experts; d.k = cfg->top_k;
  d.has_shared = cfg->shared_inter > 0; d.W = w.W; d.wpre = w.wpre; d.n_active = w.n_active;
  d.act_e = w.act_e; d.act_off = w.act_off; d.act_n = w.act_n;
  d.pair_tok = w.pair_tok; d.pos_shared = w.pos; d.cs_pos = w.cs_pos; d.cs_w = w.cs_w;
  d.ticket = w.ticket; d.item_ctr = w.item_ctr;
  return d;
}

// Front end: router (or given routing), operand prep and dispatch, one launch.
es_status run_front(const es_moe_cfg* cfg, const Workspace& w, es::RouteArgs r,
                    const int32_t* idx, const float* wts, int T, cudaStream_t st,
                    const Marks& mk) {
  es::DispatchArgs d = dispatch_args(cfg, w, idx, wts, T);
  r.bitmap = w.bitmap;
  if (mk.mark(0, st) != cudaSuccess) return ES_ERR_CUDA;
  if (es::launch_front(r, d, st) != cudaSuccess) return ES_ERR_CUDA;
  return cuda_status(mk.mark(1, st));
}

// Tensor-core path front end: routing with slot counters + scaled fp16
// activations (one launch), then slot -> pair scatter.
es_status run_pf_front(const es_moe_cfg* cfg, const Workspace& w, const es::RouteArgs& r, int T,
                       cudaStream_t st, const Marks& mk) {
  es::PfFrontArgs d{};
  d.cs_pos = w.cs_pos; d.cs_w = w.cs_w; d.rank = w.rank;
  d.cnt = reinterpret_cast<int*>(w.bitmap);  // zero between calls, like the bitmaps
  d.off_e = w.wpre; d.n_active = w.n_active; d.act_e = w.act_e; d.act_off = w.act_off;
  d.act_n = w.act_n; d.ticket = w.ticket; d.item_ctr = w.item_ctr;
  // up to kFoldScatterSlots slots the front end's last CTA scatters them
  // itself; larger batches use the grid-wide scatter kernel
  d.fold_scatter = (long long)T * w.kk <= kFoldScatterSlots;
  d.pair_tok = w.pair_tok; d.pos_shared = w.pos;
  es::PfScatterArgs sc{};
  sc.cs_pos = w.cs_pos; sc.rank = w.rank; sc.off_e = w.wpre; sc.pair_tok = w.pair_tok;
  sc.pos_shared = w.pos; sc.T = T; sc.E = cfg->num_experts; sc.k = cfg->top_k;
  sc.has_shared = cfg->shared_inter > 0;
  if (mk.mark(0, st) != cudaSuccess) return ES_ERR_CUDA;
  if (es::launch_pf_front(r, d, st) != cudaSuccess) return ES_ERR_CUDA;
  if (!d.fold_scatter && es::launch_pf_scatter(sc, st) != cudaSuccess) return ES_ERR_CUDA;
  return cuda_status(mk.mark(1, st));
}

// Tensor-core path: grouped GEMMs (gate/up, down) and the fp16-row combine.
es_status run_pf_ffn(const es_moe_cfg* cfg, const Workspace& w, const void* packed, void* out,
                     int out_f32, int T, bool small, cudaStream_t st, const Marks& mk) {
  const int E1 = cfg->num_experts + (cfg->shared_inter > 0 ? 1 : 0);
  const long long pairs = (long long)T * w.kk;
  const int nt = small ? es::kSmallTile : es::kLargeTile;
  const long long tiles = pairs / nt + (pairs < E1 ? pairs : E1);  // >= sum of ceil(n_e / nt)
  es::PfArgs a{};
  a.packed = static_cast<const uint8_t*>(packed);
  a.expert_bytes = es::expert_bytes(cfg->hidden, cfg->inter);
  a.D = cfg->hidden; a.I = cfg->inter; a.E1 = E1;
  a.n_active = w.n_active; a.act_e = w.act_e; a.act_off = w.act_off; a.act_n = w.act_n;
  a.pair_tok = w.pair_tok; a.x16 = w.x_perm; a.xinv = w.xsum; a.h16 = w.h16;
  a.y16 = reinterpret_cast<uint16_t*>(w.y_pair); a.err = w.err;
  const long long gu_units = tiles * (cfg->inter / 128), dn_units = tiles * (cfg->hidden / 128);
  const int gu_max = gu_units > (1 << 30) ? (1 << 30) : (int)gu_units;
  const int dn_max = dn_units > (1 << 30) ? (1 << 30) : (int)dn_units;
  if (mk.mark(2, st) != cudaSuccess) return ES_ERR_CUDA;
  if (es::launch_pf_gateup(a, T, gu_max, small, st) != cudaSuccess) return ES_ERR_CUDA;
  if (mk.mark(3, st) != cudaSuccess) return ES_ERR_CUDA;
  if (es::launch_pf_down(a, (long long)w.P, dn_max, small, st) != cudaSuccess) return ES_ERR_CUDA;
  if (mk.mark(4, st) != cudaSuccess) return ES_ERR_CUDA;
  es::CombineArgs cb{};
  cb.cs_pos = w.cs_pos; cb.cs_w = w.cs_w; cb.pos_shared = w.pos; cb.sgate = w.sgate;
  cb.y_pair = w.y_pair; cb.y_f16 = 1;
  cb.T = T; cb.D = cfg->hidden; cb.k = cfg->top_k; cb.has_shared = cfg->shared_inter > 0;
  cb.out = out; cb.out_f32 = out_f32;
  if (es::launch_combine(cb, st) != cudaSuccess) return ES_ERR_CUDA;
  return cuda_status(mk.mark(5, st));
}

// Shared tail of es_moe_forward / es_moe_expert_ffn: FFN and combine.
es_status run_ffn(const es_moe_cfg* cfg, const Workspace& w, const void* packed, void* out,
                  int out_f32, int T, cudaStream_t st, const Marks& mk) {
  const int E = cfg->num_experts, k = cfg->top_k;
  const int has_shared = cfg->shared_inter > 0;
  const long long routed_max = (long long)T * k < E ? (long long)T * k : E;
  const int max_active = (int)routed_max + has_shared;
  es::FfnArgs f{};
  f.packed = static_cast<const uint8_t*>(packed);
  f.expert_bytes = es::expert_bytes(cfg->hidden, cfg->inter);
  f.D = cfg->hidden; f.I = cfg->inter;
  f.n_active = w.n_active; f.act_e = w.act_e; f.act_off = w.act_off; f.act_n = w.act_n;
  f.pair_tok = w.pair_tok; f.x_perm = w.x_perm; f.xsum = w.xsum;
  f.h16 = w.h16; f.y_pair = w.y_pair; f.err = w.err;
  f.partials = w.partials; f.counters = w.counters; f.item_ctr = w.item_ctr;
  f.split_k = es::ffn_split_k(T, max_active, cfg->hidden, cfg->inter);
  f.split_k_down = es::ffn_split_k_down(T, max_active, cfg->hidden, cfg->inter);
  if (mk.mark(2, st) != cudaSuccess) return ES_ERR_CUDA;
  if (es::launch_ffn_gateup(f, max_active, st) != cudaSuccess) return ES_ERR_CUDA;
  if (mk.mark(3, st) != cudaSuccess) return ES_ERR_CUDA;
  if (es::launch_ffn_down(f, max_active, st) != cudaSuccess) return ES_ERR_CUDA;
  if (mk.mark(4, st) != cudaSuccess) return ES_ERR_CUDA;
  es::CombineArgs cb{};
  cb.cs_pos = w.cs_pos; cb.cs_w = w.cs_w; cb.pos_shared = w.pos; cb.sgate = w.sgate;
  cb.y_pair = w.y_pair; cb.y_f16 = 0;
  cb.T = T; cb.D = cfg->hidden; cb.k = k; cb.has_shared = has_shared;
  cb.out = out; cb.out_f32 = out_f32;
  if (es::launch_combine(cb, st) != cudaSuccess) return ES_ERR_CUDA;
  return cuda_status(mk.mark(5, st));
}

// The fused tiny-batch block: one cooperative kernel (es_small.cu). The
// instrumentation events all land around that one kernel (the whole block
// shows as the front-end interval).
es_status run_small(const es_moe_cfg* cfg, const Workspace& w, const es::RouteArgs& r,
                    const void* packed, void* out, int out_f32, cudaStream_t st,
                    const Marks& mk) {
  es::SmallArgs a{};
  a.logits = r.logits; a.logits_f32 = r.logits_f32; a.bias = r.bias;
  a.in_idx = r.in_idx; a.in_w = r.in_w; a.x = r.x; a.sg_w = r.sg_w;
  a.packed = static_cast<const uint8_t*>(packed);
  a.expert_bytes = es::expert_bytes(cfg->hidden, cfg->inter);
  a.T = r.T; a.D = cfg->hidden; a.E = cfg->num_experts; a.k = cfg->top_k; a.I = cfg->inter;
  a.renorm = r.renorm; a.has_shared = r.has_shared;
  a.out = out; a.out_f32 = out_f32; a.out_idx = r.out_idx; a.out_w = r.out_w;
  a.part = w.partials; a.part_slots = (long long)w.part_slots; a.h16 = w.h16;
  // the counter region is zero between calls on every path
  a.ctr = w.counters; a.err = w.err;
  if (mk.mark(0, st) != cudaSuccess) return ES_ERR_CUDA;
  if (es::launch_small(a, st) != cudaSuccess) return ES_ERR_CUDA;
  for (int i = 1; i <= 5; ++i)
    if (mk.mark(i, st) != cudaSuccess) return ES_ERR_CUDA;
  return ES_OK;
}

es_status check_common(const es_moe_cfg* cfg, const void* x, const void* packed,
                       void* out, int32_t out_dtype, int32_t T, void* ws,
                       size_t ws_bytes, Workspace* w) {
  es_status s = check_cfg(cfg);
  if (s != ES_OK) return s;
  if (T < 0 || T > 65535) return ES_ERR_UNSUPPORTED;
  if (out_dtype != ES_DTYPE_BF16 && out_dtype != ES_DTYPE_F32) return ES_ERR_UNSUPPORTED;
  if (!ws || !aligned(ws, 256)) return ES_ERR_INVALID_ARG;
  *w = es::carve_workspace(ws, cfg->hidden, cfg->num_experts, cfg->top_k, cfg->inter,
                           cfg->shared_inter > 0, T);
  if (ws_bytes < w->bytes) return ES_ERR_WORKSPACE;
  if (T == 0) return ES_OK;
  if (!x || !packed || !out) return ES_ERR_INVALID_ARG;
  if (!aligned(x, 16) || !aligned(packed, 16) || !aligned(out, 16)) return ES_ERR_INVALID_ARG;
  return ES_OK;
}

// Shared tail of es_moe_prepare / es_moe_prepare_blocks: the shared expert
// (when configured) and the launch.
es_status prepare_common(const es_moe_cfg* cfg, const es_mlx_layer* layer, es::PrepareArgs& a,
                         void* packed, es_stream_t stream) {
  const es_mlx_proj* shared[3] = {&layer->shared_gate_proj, &layer->shared_up_proj,
                                  &layer->shared_down_proj};
  const int has_shared = cfg->shared_inter > 0;
  for (int p = 0; p < 3 && has_shared; ++p) {
    if (!shared[p]->weight || !shared[p]->scales || !shared[p]->biases) return ES_ERR_INVALID_ARG;
    a.sw[p] = shared[p]->weight; a.ss[p] = shared[p]->scales; a.sb[p] = shared[p]->biases;
  }
  a.D = cfg->hidden; a.I = cfg->inter; a.E = cfg->num_experts; a.has_shared = has_shared;
  a.packed = static_cast<uint8_t*>(packed);
  return cuda_status(es::launch_prepare(a, static_cast<cudaStream_t>(stream)));
}

}  // namespace

extern "C" {

const char* es_status_str(es_status status) {
  switch (status) {
    case ES_OK: return "ok";
    case ES_ERR_INVALID_ARG: return "invalid argument";
    case ES_ERR_UNSUPPORTED: return "unsupported shape";
    case ES_ERR_WORKSPACE: return "workspace too small";
    case ES_ERR_CUDA: return "CUDA runtime error";
    case ES_ERR_DEVICE: return "device-side invariant violation";
  }
  return "unknown status";
}

int32_t es_version(void) { return (1 << 16) | 1; }

es_status es_moe_packed_bytes(const es_moe_cfg* cfg, size_t* bytes_out) {
  es_status s = check_cfg(cfg);
  if (s != ES_OK) return s;
  if (!bytes_out) return ES_ERR_INVALID_ARG;
  const int E1 = cfg->num_experts + (cfg->shared_inter > 0 ? 1 : 0);
  *bytes_out = es::expert_bytes(cfg->hidden, cfg->inter) * (size_t)E1;
  return ES_OK;
}

es_status es_moe_prepare(const es_moe_cfg* cfg, const es_mlx_layer* layer,
                         void* packed, size_t packed_bytes, es_stream_t stream) {
  es_status s = check_cfg(cfg);
  if (s != ES_OK) return s;
  if (!layer || !packed || !aligned(packed, 256)) return ES_ERR_INVALID_ARG;
  size_t need = 0;
  es_moe_packed_bytes(cfg, &need);
  if (packed_bytes < need) return ES_ERR_INVALID_ARG;
  es::PrepareArgs a{};
  const es_mlx_proj* routed[3] = {&layer->gate, &layer->up, &layer->down};
  for (int p = 0; p < 3; ++p) {
    if (!routed[p]->weight || !routed[p]->scales || !routed[p]->biases) return ES_ERR_INVALID_ARG;
    // stacked [E, N, K/8] uint32 and [E, N, K/64] fp16
    const size_t N = p < 2 ? cfg->inter : cfg->hidden, K = p < 2 ? cfg->hidden : cfg->inter;
    a.w[p] = reinterpret_cast<const uint8_t*>(routed[p]->weight);
    a.s[p] = reinterpret_cast<const uint8_t*>(routed[p]->scales);
    a.b[p] = reinterpret_cast<const uint8_t*>(routed[p]->biases);
    a.ew[p] = N * (K / 8) * 4;
    a.es[p] = a.eb[p] = N * (K / es::kGroup) * 2;
  }
  return prepare_common(cfg, layer, a, packed, stream);
}

es_status es_moe_prepare_blocks(const es_moe_cfg* cfg, const void* blocks, size_t block_bytes,
                                const int64_t* inner_offsets, const es_mlx_layer* shared_layer,
                                void* packed, size_t packed_bytes, es_stream_t stream) {
  es_status s = check_cfg(cfg);
  if (s != ES_OK) return s;
  if (!blocks || !inner_offsets || !packed || !aligned(packed, 256) || !aligned(blocks, 16))
    return ES_ERR_INVALID_ARG;
  size_t need = 0;
  es_moe_packed_bytes(cfg, &need);
  if (packed_bytes < need) return ES_ERR_INVALID_ARG;
  const size_t D = cfg->hidden, I = cfg->inter;
  // per-expert bytes of the 9 tensors in TENSOR_ORDER
  const size_t nbytes[9] = {I * D / 2, I * (D / 64) * 2, I * (D / 64) * 2,
                            I * D / 2, I * (D / 64) * 2, I * (D / 64) * 2,
                            D * I / 2, D * (I / 64) * 2, D * (I / 64) * 2};
  for (int t = 0; t < 9; ++t) {
    const int64_t o = inner_offsets[t];
    if (o < 0 || (size_t)o + nbytes[t] > block_bytes || (o % 4) != 0) return ES_ERR_INVALID_ARG;
  }
  if (block_bytes % 16) return ES_ERR_INVALID_ARG;
  es::PrepareArgs a{};
  const uint8_t* base = static_cast<const uint8_t*>(blocks);
  for (int p = 0; p < 3; ++p) {
    a.w[p] = base + inner_offsets[3 * p];
    a.s[p] = base + inner_offsets[3 * p + 1];
    a.b[p] = base + inner_offsets[3 * p + 2];
    a.ew[p] = a.es[p] = a.eb[p] = block_bytes;
  }
  es_mlx_layer lay{};
  if (shared_layer) {
    lay.shared_gate_proj = shared_layer->shared_gate_proj;
    lay.shared_up_proj = shared_layer->shared_up_proj;
    lay.shared_down_proj = shared_layer->shared_down_proj;
  }
  return prepare_common(cfg, &lay, a, packed, stream);
}

es_status es_moe_workspace_bytes(const es_moe_cfg* cfg, int32_t max_tokens, size_t* bytes_out) {
  es_status s = check_cfg(cfg);
  if (s != ES_OK) return s;
  if (!bytes_out || max_tokens < 0 || max_tokens > 65535) return ES_ERR_INVALID_ARG;
  *bytes_out = es::carve_workspace(nullptr, cfg->hidden, cfg->num_experts, cfg->top_k,
                                   cfg->inter, cfg->shared_inter > 0, max_tokens).bytes;
  return ES_OK;
}

es_status es_moe_kernel_family(const es_moe_cfg* cfg, int32_t T, int32_t* path_out) {
  es_status s = check_cfg(cfg);
  if (s != ES_OK) return s;
  if (!path_out || T < 1 || T > 65535) return ES_ERR_INVALID_ARG;
  static const int32_t kPath[4] = {1, 2, 3, 4};  // decode, 128-token, 32-token, fused
  *path_out = kPath[ffn_variant(cfg, T)];
  return ES_OK;
}

es_status es_moe_route(const es_moe_cfg* cfg, const void* logits, int32_t logits_dtype,
                       const float* cache_bias, int32_t T, int32_t* topk_idx, float* topk_w,
                       es_stream_t stream) {
  es_status s = check_cfg(cfg);
  if (s != ES_OK) return s;
  if (T < 0) return ES_ERR_INVALID_ARG;
  if (logits_dtype != ES_DTYPE_BF16 && logits_dtype != ES_DTYPE_F32) return ES_ERR_UNSUPPORTED;
  if (cfg->top_k > cfg->num_experts) return ES_ERR_UNSUPPORTED;
  if (T == 0) return ES_OK;
  if (!logits || !topk_idx || !topk_w) return ES_ERR_INVALID_ARG;
  es::RouteArgs r{};
  r.logits = logits; r.logits_f32 = logits_dtype == ES_DTYPE_F32; r.bias = cache_bias;
  r.T = T; r.D = cfg->hidden; r.E = cfg->num_experts; r.k = cfg->top_k;
  r.renorm = cfg->norm_topk_prob != 0; r.W = (T + 31) / 32;
  r.out_idx = topk_idx; r.out_w = topk_w;
  es::DispatchArgs d{};
  return cuda_status(es::launch_front(r, d, static_cast<cudaStream_t>(stream)));
}

es_status es_moe_expert_ffn(const es_moe_cfg* cfg, const void* x, const int32_t* topk_idx,
                            const float* topk_w, const void* shared_gate_w, const void* packed,
                            void* out, int32_t out_dtype, int32_t T, void* workspace,
                            size_t workspace_bytes, es_stream_t stream) {
  Workspace w{};
  es_status s = check_common(cfg, x, packed, out, out_dtype, T, workspace, workspace_bytes, &w);
  if (s != ES_OK || T == 0) return s;
  if (!topk_idx || !topk_w) return ES_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  es::RouteArgs r{};
  r.in_idx = topk_idx; r.in_w = topk_w;
  r.x = static_cast<const uint16_t*>(x);
  r.sg_w = static_cast<const uint16_t*>(shared_gate_w);
  r.T = T; r.D = cfg->hidden; r.E = cfg->num_experts; r.k = cfg->top_k;
  r.renorm = cfg->norm_topk_prob != 0; r.has_shared = cfg->shared_inter > 0; r.W = w.W;
  r.x_f16 = cfg->x_dtype == ES_DTYPE_F16;
  r.sgate = w.sgate; r.x_perm = w.x_perm; r.xsum = w.xsum; r.err = w.err;
  Marks mk;
  const int v = ffn_variant(cfg, T);
  if (v == kFfnFused) {
    r.out_idx = nullptr; r.out_w = nullptr;
    return run_small(cfg, w, r, packed, out, out_dtype == ES_DTYPE_F32, st, mk);
  }
  if (v != kFfnDecode) {
    r.out_idx = nullptr; r.out_w = nullptr;
    es_status s2 = run_pf_front(cfg, w, r, T, st, mk);
    if (s2 != ES_OK) return s2;
    return run_pf_ffn(cfg, w, packed, out, out_dtype == ES_DTYPE_F32, T, v == kFfnTensorSmall,
                      st, mk);
  }
  es_status s2 = run_front(cfg, w, r, topk_idx, topk_w, T, st, mk);
  if (s2 != ES_OK) return s2;
  return run_ffn(cfg, w, packed, out, out_dtype == ES_DTYPE_F32, T, st, mk);
}

es_status es_moe_forward(const es_moe_cfg* cfg, const void* x, const void* logits,
                         int32_t logits_dtype, const float* cache_bias, const void* shared_gate_w,
                         const void* packed, void* out, int32_t out_dtype, int32_t* topk_idx,
                         float* topk_w, int32_t T, void* workspace, size_t workspace_bytes,
                         es_stream_t stream) {
  return es_moe_forward_timed(cfg, x, logits, logits_dtype, cache_bias, shared_gate_w, packed, out,
                              out_dtype, topk_idx, topk_w, T, workspace, workspace_bytes, stream,
                              nullptr, 0);
}

es_status es_moe_forward_timed(const es_moe_cfg* cfg, const void* x, const void* logits,
                               int32_t logits_dtype, const float* cache_bias,
                               const void* shared_gate_w, const void* packed, void* out,
                               int32_t out_dtype, int32_t* topk_idx, float* topk_w, int32_t T,
                               void* workspace, size_t workspace_bytes, es_stream_t stream,
                               void* const* events, int32_t n_events) {
  Workspace w{};
  es_status s = check_common(cfg, x, packed, out, out_dtype, T, workspace, workspace_bytes, &w);
  if (s != ES_OK || T == 0) return s;
  if (!logits) return ES_ERR_INVALID_ARG;
  if (logits_dtype != ES_DTYPE_BF16 && logits_dtype != ES_DTYPE_F32) return ES_ERR_UNSUPPORTED;
  if (cfg->top_k > cfg->num_experts) return ES_ERR_UNSUPPORTED;
  if (events && n_events != 6) return ES_ERR_INVALID_ARG;
  Marks mk;
  mk.ev = events;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* idx = topk_idx ? topk_idx : w.topk_idx;
  float* wts = topk_w ? topk_w : w.topk_w;
  es::RouteArgs r{};
  r.logits = logits; r.logits_f32 = logits_dtype == ES_DTYPE_F32; r.bias = cache_bias;
  r.x = static_cast<const uint16_t*>(x);
  r.sg_w = static_cast<const uint16_t*>(shared_gate_w);
  r.T = T; r.D = cfg->hidden; r.E = cfg->num_experts; r.k = cfg->top_k;
  r.renorm = cfg->norm_topk_prob != 0; r.has_shared = cfg->shared_inter > 0; r.W = w.W;
  r.x_f16 = cfg->x_dtype == ES_DTYPE_F16;
  r.out_idx = idx; r.out_w = wts;
  r.sgate = w.sgate; r.x_perm = w.x_perm; r.xsum = w.xsum; r.err = w.err;
  const int v = ffn_variant(cfg, T);
  if (v == kFfnFused)
    return run_small(cfg, w, r, packed, out, out_dtype == ES_DTYPE_F32, st, mk);
  if (v != kFfnDecode) {
    es_status s2 = run_pf_front(cfg, w, r, T, st, mk);
    if (s2 != ES_OK) return s2;
    return run_pf_ffn(cfg, w, packed, out, out_dtype == ES_DTYPE_F32, T, v == kFfnTensorSmall,
                      st, mk);
  }
  es_status s2 = run_front(cfg, w, r, idx, wts, T, st, mk);
  if (s2 != ES_OK) return s2;
  return run_ffn(cfg, w, packed, out, out_dtype == ES_DTYPE_F32, T, st, mk);
}

es_status es_moe_read_error(const void* workspace, int32_t clear, uint32_t* flags_out,
                            es_stream_t stream) {
  if (!workspace || !flags_out || !aligned(workspace, 256)) return ES_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  if (cudaMemcpyAsync(&v, workspace, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) return ES_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return ES_ERR_CUDA;
  // clearing also drops the recorded site of a timed-out wait (words 1-3)
  if (clear && cudaMemsetAsync(const_cast<void*>(workspace), 0, 16, st) != cudaSuccess)
    return ES_ERR_CUDA;
  *flags_out = v;
  return ES_OK;
}

}  // extern "C"
