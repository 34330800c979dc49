// Launch arguments and host launchers of the MoE block kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "es_layout.h"

namespace es {

struct RouteArgs {
  // routing source: either logits (+ optional bias) or given top-k
  const void* logits;       // [T][E] bf16 or f32
  int logits_f32;
  const float* bias;        // [E] or null
  const int32_t* in_idx;    // [T][k] given routing, or null
  const float* in_w;        // [T][k]
  // activations
  const uint16_t* x;        // [T][D] bf16 or null (route only)
  const uint16_t* sg_w;     // [D] bf16 shared gate weight or null
  int T, D, E, k, renorm, has_shared, W;
  int x_f16;                // x is fp16 (tensor-core path only), else bf16
  // outputs
  int32_t* out_idx;         // [T][k] or null
  float* out_w;             // [T][k] or null
  uint32_t* bitmap;         // [E1][W] or null
  float* sgate;             // [T] or null
  uint16_t* x_perm;         // [T][D] or null
  float* xsum;              // [T][D/64] or null
  uint32_t* err;
};

struct DispatchArgs {
  const uint32_t* bitmap;   // [E1][W]
  const int32_t* idx;       // [T][k]
  const float* w;           // [T][k]
  int T, E, k, has_shared, W;
  int32_t* wpre;            // [E1][W]
  int32_t* n_active;
  int32_t* act_e;
  int32_t* act_off;
  int32_t* act_n;
  int32_t* pair_tok;
  int32_t* pos_shared;      // [T] pair of the shared expert
  int32_t* cs_pos;          // [T][k] sorted pair of the r-th smallest expert id, -1 = none
  float* cs_w;              // [T][k] its routing weight
  int* ticket;              // CTAs done routing (zero between calls)
  int* item_ctr;            // [2] FFN work counters, zeroed here for the FFN kernels
};

struct FfnArgs {
  const uint8_t* packed;
  size_t expert_bytes;
  int D, I;
  const int32_t* n_active;
  const int32_t* act_e;
  const int32_t* act_off;
  const int32_t* act_n;
  const int32_t* pair_tok;
  const uint16_t* x_perm;
  const float* xsum;
  uint16_t* h16;            // [P][I] fp16, fragment order
  float* y_pair;
  uint32_t* err;
  float* partials;          // split-K partial sums (split_k > 1)
  int* counters;            // split-K arrival counters, zero between calls
  int* item_ctr;            // [2] dynamic item counters (gate/up, down)
  int split_k;              // K split of gate/up items
  int split_k_down;         // K split of down items
};

struct CombineArgs {
  const int32_t* cs_pos;    // [T][k]
  const float* cs_w;        // [T][k]
  const int32_t* pos_shared;  // [T]
  const float* sgate;       // [T]
  const void* y_pair;       // [P][D] fp32, or fp16 when y_f16
  int y_f16;
  int T, D, k, has_shared;
  void* out;
  int out_f32;
};

// Tensor-core path (large batches). Front end: routing with per-expert slot
// counters instead of token bitmaps, scaled fp16 activations in nibble order.
struct PfFrontArgs {
  int32_t* cs_pos;          // [T][k] expert id of the r-th smallest id (pair index after scatter)
  float* cs_w;              // [T][k]
  int32_t* rank;            // [T][k] rank of the slot inside its expert's list
  int* cnt;                 // [E] slot counters (zero between calls)
  int32_t* off_e;           // [E1] first pair of each expert
  int32_t* n_active;
  int32_t* act_e;
  int32_t* act_off;
  int32_t* act_n;
  int* ticket;              // CTAs done routing (zero between calls)
  int* item_ctr;            // [2] zeroed for symmetry with the decode front end
  // small batches: the last CTA also turns slots into pair indices (the
  // work of pf_scatter), saving a launch; pair_tok / pos_shared are written
  int fold_scatter;
  int32_t* pair_tok;        // [P]
  int32_t* pos_shared;      // [T]
};

struct PfScatterArgs {
  int32_t* cs_pos;          // [T][k] expert id in, pair index out
  const int32_t* rank;      // [T][k]
  const int32_t* off_e;     // [E1]
  int32_t* pair_tok;        // [P]
  int32_t* pos_shared;      // [T]
  int T, E, k, has_shared;
};

// Grouped GEMM over (active expert, 128-row block, token tile) units.
struct alignas(64) PfArgs {
  CUtensorMap tm_b;         // B rows: x16 (gate/up) or h16 (down); set by the launcher
  CUtensorMap tm_a;         // packed code tiles, one 5-D box per stage; set by the launcher
  const uint8_t* packed;
  size_t expert_bytes;
  int D, I;
  int E1;                   // experts in the packed blob (routed + shared)
  const int32_t* n_active;
  const int32_t* act_e;
  const int32_t* act_off;
  const int32_t* act_n;
  const int32_t* pair_tok;
  const uint16_t* x16;      // [T][D] fp16, nibble order, scaled per token
  const float* xinv;        // [T] inverse scales
  uint16_t* h16;            // [P][I] fp16, nibble order
  uint16_t* y16;            // [P][D] fp16
  uint32_t* err;
};

// The fused tiny-batch block (es_small.cu), T <= kSmallMaxTokens.
struct SmallArgs {
  // routing source: logits (+ optional bias) or given top-k
  const void* logits;
  int logits_f32;
  const float* bias;
  const int32_t* in_idx;    // [T][k] or null
  const float* in_w;        // [T][k]
  const uint16_t* x;        // [T][D] bf16
  const uint16_t* sg_w;     // [D] bf16 shared gate weight or null
  const uint8_t* packed;
  size_t expert_bytes;
  int T, D, E, k, I, renorm, has_shared;
  int ks_gu, ks_dn;         // K shares of the gate/up and down items
  long long part_slots;     // 2 KB slots in `part` (capacity check)
  void* out;
  int out_f32;
  int32_t* out_idx;         // [T][k] or null
  float* out_w;
  float* part;              // split-K partial sums (gate/up, then reused by down)
  uint16_t* h16;            // [P][I] fp16, fragment order
  int* ctr;                 // [2] grid-barrier counters, zero between calls
  uint32_t* err;
};

struct PrepareArgs {
  // routed experts of projection p (gate, up, down): weight / scales / biases
  // of expert e start at w[p] + e * ew[p] bytes (and likewise s, b), so both
  // stacked MLX tensors ([E, N, K/8], stride N*K/2 bytes) and the streaming
  // format's fixed expert blocks (stride = block size) are read in place
  const uint8_t* w[3];
  const uint8_t* s[3];
  const uint8_t* b[3];
  size_t ew[3], es[3], eb[3];
  // shared expert (no expert axis) or nulls
  const uint32_t* sw[3];
  const uint16_t* ss[3];
  const uint16_t* sb[3];
  int D, I, E, has_shared;
  uint8_t* packed;
};

// Launch with programmatic stream serialization (see pdl_wait in es_common.cuh).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// router (+ operand prep + dispatch when r.bitmap is set), one launch
cudaError_t launch_front(const RouteArgs& r, const DispatchArgs& d, cudaStream_t st);
int sm_count();
// K split of gate/up items for a batch of T tokens (1 above kSplitKMaxTokens)
int ffn_split_k(int T, int max_active, int D, int I);
int ffn_split_k_down(int T, int max_active, int D, int I);
cudaError_t launch_ffn_gateup(const FfnArgs& a, int max_active, cudaStream_t st);
cudaError_t launch_ffn_down(const FfnArgs& a, int max_active, cudaStream_t st);
cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st);
// tensor-core path
cudaError_t launch_pf_front(const RouteArgs& r, const PfFrontArgs& d, cudaStream_t st);
cudaError_t launch_pf_scatter(const PfScatterArgs& a, cudaStream_t st);
// token tiles of the tensor-core GEMMs: large batches (A in shared memory)
// and small ones (A in tensor memory)
constexpr int kLargeTile = 128;
constexpr int kSmallTile = 32;
cudaError_t launch_pf_gateup(const PfArgs& a, long long tokens, int max_units, bool small,
                             cudaStream_t st);
cudaError_t launch_pf_down(const PfArgs& a, long long pairs, int max_units, bool small,
                           cudaStream_t st);
cudaError_t launch_prepare(const PrepareArgs& a, cudaStream_t st);
// fused tiny-batch block: whether a call can take it (T <= kSmallMaxTokens,
// also the automatic choice's limit), and the launch
bool small_path_fits(int T, int D, int I, int E, int k, int has_shared);
cudaError_t launch_small(SmallArgs a, cudaStream_t st);

}  // namespace es
