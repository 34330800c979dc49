/*
 * es_moe.h — C ABI of the B200 MoE block (router -> dispatch -> 4-bit expert
 * FFN -> combine) for Expert Sniper's MLX-affine expert format.
 *
 * Conventions
 *   - Every pointer argument except `cfg` and the `*_bytes` / error outputs is
 *     caller-owned DEVICE memory on the current CUDA device.
 *   - Nothing here allocates device memory, and nothing on the forward path
 *     synchronises the host: kernels are queued on `stream` (a cudaStream_t
 *     passed as void*, NULL = legacy default stream).
 *   - Errors are status codes; no exception crosses this boundary. Invariant
 *     violations detected inside a kernel are recorded in an error word that
 *     lives in the workspace and is read with es_moe_read_error().
 *   - Calls that share a workspace must be ordered on one stream.
 *
 * Expert weight format (the reference's on-disk / MLX format, one expert):
 *   gate_proj / up_proj : weight [I, D/8] uint32, scales [I, D/64] fp16,
 *                         biases [I, D/64] fp16
 *   down_proj           : weight [D, I/8] uint32, scales [D, I/64] fp16,
 *                         biases [D, I/64] fp16
 *   code q of column k sits in bits 4*(k%8) of word k/8 of its row, and
 *   w = scale * q + bias per 64-column group.
 * (src/mlx_expert_sniper/download.py:73-77 TENSOR_ORDER, download.py:189-248,
 *  src/mlx_expert_sniper/engine.py:12-13 BITS=4, GROUP_SIZE=64.)
 */
#ifndef ES_MOE_H
#define ES_MOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(ES_BUILD_LIB) && defined(__GNUC__)
#define ES_API __attribute__((visibility("default")))
#else
#define ES_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* es_stream_t; /* cudaStream_t */

typedef enum es_status {
  ES_OK = 0,
  ES_ERR_INVALID_ARG = 1,   /* null pointer, bad size, misaligned buffer     */
  ES_ERR_UNSUPPORTED = 2,   /* shape outside what the kernels implement      */
  ES_ERR_WORKSPACE = 3,     /* workspace smaller than es_moe_workspace_bytes */
  ES_ERR_CUDA = 4,          /* a CUDA runtime call failed                    */
  ES_ERR_DEVICE = 5         /* a kernel flagged an invariant violation       */
} es_status;

typedef enum es_dtype {
  ES_DTYPE_BF16 = 0,
  ES_DTYPE_F16 = 1,
  ES_DTYPE_F32 = 2
} es_dtype;

/* Device error word bits (es_moe_read_error). */
#define ES_DEVERR_BAD_EXPERT_ID 0x1u   /* top-k index outside [-1, E)        */
#define ES_DEVERR_NONFINITE_LOGIT 0x2u /* NaN logit seen by the router        */
#define ES_DEVERR_CAPACITY 0x4u        /* pair list larger than the workspace */
#define ES_DEVERR_TIMEOUT 0x8u         /* a bounded in-kernel wait gave up    */
#define ES_DEVERR_RANGE 0x10u          /* |silu(g)*u| beyond fp16, saturated  */

/* Shape of one MoE block. Mirrors the streaming config.json keys the
 * reference reads (download.py:477-523: num_experts, num_experts_per_tok,
 * moe_intermediate_size, norm_topk_prob, shared_expert_intermediate_size,
 * quantization{bits, group_size}). */
typedef struct es_moe_cfg {
  int32_t hidden;         /* D = 256 * {1,2,3,4,6,8,12,16}                    */
  int32_t num_experts;    /* E routed experts, 1..1024                       */
  int32_t top_k;          /* k, 1..16 (k <= E for the router)                 */
  int32_t inter;          /* I: 256, 512, 768, 1024, 1536 or 2048             */
  int32_t group_size;     /* must be 64                                       */
  int32_t bits;           /* must be 4                                        */
  int32_t norm_topk_prob; /* 1: renormalise the k selected probabilities      */
  int32_t shared_inter;   /* 0: no shared expert; else its I (must == inter)  */
  int32_t kernel_path;    /* which expert-FFN kernels run (no reference
                           * counterpart; results agree within the parity
                           * tolerance either way):
                           *   0 = automatic, by the average (token,
                           *       expert) pairs per routed expert
                           *       p = T * top_k / num_experts: with
                           *       T >= 64, path 2 for p > 48, path 3 for
                           *       4 <= p <= 48; path 4 for T <= 16; the
                           *       decode path otherwise (path 3 for fp16
                           *       x);
                           *   1 = decode path (register-operand GEMV on the
                           *       4-bit codes, fp32 per-pair rows);
                           *   2 = tensor-core path (tcgen05 grouped GEMM,
                           *       fp16 operands dequantised in shared
                           *       memory, fp16 per-pair rows);
                           *   3 = tensor-core path with 32-token tiles and
                           *       the dequantised weights in tensor memory
                           *       (same arithmetic as 2);
                           *   4 = the fused tiny-batch kernel (T <= 16, bf16
                           *       x): the whole block in one cooperative
                           *       launch, decode-path arithmetic; path 0
                           *       takes it for T <= 16 with bf16 x; larger
                           *       batches given path 4 run the decode path */
  int32_t x_dtype;        /* activations x: ES_DTYPE_BF16 (0, the model
                           * dtype) or ES_DTYPE_F16 (the Expert Network's
                           * wire dtype, protocol.py:3-9); fp16 x runs the
                           * tensor-core kernels, which read it without
                           * rounding (kernel_path 1 rejects it)            */
} es_moe_cfg;

/* Per-projection MLX tensors for all experts of one layer, stacked on a
 * leading expert axis ([E, ...]), device pointers. The shared expert, when
 * cfg->shared_inter > 0, is passed separately without the expert axis. */
typedef struct es_mlx_proj {
  const uint32_t* weight; /* [E, N, K/8]  */
  const uint16_t* scales; /* [E, N, K/64] fp16 bits */
  const uint16_t* biases; /* [E, N, K/64] fp16 bits */
} es_mlx_proj;

typedef struct es_mlx_layer {
  es_mlx_proj gate; /* N = I, K = D */
  es_mlx_proj up;   /* N = I, K = D */
  es_mlx_proj down; /* N = D, K = I */
  es_mlx_proj shared_gate_proj; /* shared expert, no expert axis, or NULLs */
  es_mlx_proj shared_up_proj;
  es_mlx_proj shared_down_proj;
} es_mlx_layer;

/* Static string for a status code. */
ES_API const char* es_status_str(es_status status);

/* ABI version, (major << 16) | minor. */
ES_API int32_t es_version(void);

/* Bytes of the packed (device-resident) weights of one layer: exactly the
 * reference's per-expert bytes 3*D*I*0.5625 times (E + has_shared).
 * Replaces the per-call re-stacking of `stack_proj`
 * (src/mlx_expert_sniper/engine.py:22-30): the layout is built once. */
ES_API es_status es_moe_packed_bytes(const es_moe_cfg* cfg, size_t* bytes_out);

/* One-time repack of a layer's MLX tensors into the tiled device layout the
 * kernels stream. `packed` must be 256-byte aligned and hold
 * es_moe_packed_bytes() bytes. Counterpart of reader.get_experts + stack_proj
 * (src/mlx_expert_sniper/expert_io.py:420-436, engine.py:22-30). */
ES_API es_status es_moe_prepare(const es_moe_cfg* cfg, const es_mlx_layer* layer,
                         void* packed, size_t packed_bytes, es_stream_t stream);

/* The same repack from a streaming-format layer image already in device
 * memory: the reference's layer_XX.bin minus its 16 KB JSON header, i.e.
 * E fixed-size expert blocks of `block_bytes` each (a multiple of 16384),
 * holding the nine tensors of TENSOR_ORDER (gate, up, down x weight,
 * scales, biases) at `inner_offsets[0..8]` from the start of a block, fp16
 * scales and biases. The shared expert, which the streaming files do not
 * carry, comes from `shared_layer` (its shared_*_proj members) or NULL.
 * Counterpart of the reader's pread + parse of one expert block
 * (src/mlx_expert_sniper/expert_io.py:280-284, 338-362) and the writer's
 * layout (src/mlx_expert_sniper/download.py:73-77, 197-212). */
ES_API es_status es_moe_prepare_blocks(const es_moe_cfg* cfg, const void* blocks,
                                       size_t block_bytes, const int64_t* inner_offsets,
                                       const es_mlx_layer* shared_layer, void* packed,
                                       size_t packed_bytes, es_stream_t stream);

/* Workspace bytes needed by es_moe_forward / es_moe_expert_ffn for up to
 * `max_tokens` tokens per call (non-decreasing in max_tokens). The workspace
 * must be zero-filled once before its first use (it holds counters that the
 * kernels return to zero after every call). */
ES_API es_status es_moe_workspace_bytes(const es_moe_cfg* cfg, int32_t max_tokens,
                                 size_t* bytes_out);

/* The expert-FFN kernel family a call with T tokens runs under `cfg`, as
 * an es_moe_cfg.kernel_path value (1 decode, 2 128-token tensor-core
 * tiles, 3 32-token tiles, 4 fused one-launch): the automatic rule applied,
 * or the path cfg names. Host-only; needs no GPU. */
ES_API es_status es_moe_kernel_family(const es_moe_cfg* cfg, int32_t T, int32_t* path_out);

/* Router: logits (+ optional additive cache bias, promoted to fp32) ->
 * softmax (fp32) -> top-k -> optional renormalisation.
 *   logits     [T, E] bf16 or f32 (logits_dtype)
 *   cache_bias [E] f32 or NULL (NULL = no bias, as for bias == 0)
 *   topk_idx   [T, k] int32 out, in descending probability order
 *   topk_w     [T, k] f32 out
 * Ties in the selection key go to the lower expert id.
 * Counterpart of src/mlx_expert_sniper/generate.py:122-136 (and
 * engine_30b.py:158-165, models/qwen4_exp.py:463-472). */
ES_API es_status es_moe_route(const es_moe_cfg* cfg, const void* logits,
                       int32_t logits_dtype, const float* cache_bias,
                       int32_t T, int32_t* topk_idx, float* topk_w,
                       es_stream_t stream);

/* Expert FFN + combine for given routing:
 *   out[t] = sum_j w[t,j] * down(silu(gate(x_t)) * up(x_t))[idx[t,j]]
 *            (+ sigmoid(x_t . shared_gate_w) * shared(x_t) if shared)
 * An index of -1 skips that slot (the partition mask of the expert-parallel
 * partial). The k terms of a token are summed in ascending expert id order,
 * in fp32; the shared term is added last.
 *   x              [T, D] bf16
 *   topk_idx       [T, k] int32 in [-1, E)
 *   topk_w         [T, k] f32
 *   shared_gate_w  [D] bf16 or NULL (NULL with a shared expert = gate 1.0)
 *   out            [T, D] bf16 or f32 (out_dtype)
 * Counterpart of run_expert_ffn (src/mlx_expert_sniper/engine.py:15-42,
 * engine_30b.py:15-42, engine_next.py:15-42), the shared expert of
 * generate.py:173-178, and compute_partial's masking
 * (src/expert_network/node.py:142-172). */
ES_API es_status es_moe_expert_ffn(const es_moe_cfg* cfg, const void* x,
                            const int32_t* topk_idx, const float* topk_w,
                            const void* shared_gate_w, const void* packed,
                            void* out, int32_t out_dtype, int32_t T,
                            void* workspace, size_t workspace_bytes,
                            es_stream_t stream);

/* The whole block: es_moe_route followed by es_moe_expert_ffn, sharing the
 * workspace. topk_idx / topk_w may be NULL (kept in the workspace).
 * Counterpart of the MoE part of make_forward's layer loop
 * (src/mlx_expert_sniper/generate.py:122-181). */
ES_API es_status es_moe_forward(const es_moe_cfg* cfg, const void* x,
                         const void* logits, int32_t logits_dtype,
                         const float* cache_bias, const void* shared_gate_w,
                         const void* packed, void* out, int32_t out_dtype,
                         int32_t* topk_idx, float* topk_w, int32_t T,
                         void* workspace, size_t workspace_bytes,
                         es_stream_t stream);

/* es_moe_forward with instrumentation: `events` holds 6 cudaEvent_t that are
 * recorded on `stream` before the router, dispatch, gate/up, down and combine
 * kernels and after the combine, so the caller can read each kernel's device
 * time with cudaEventElapsedTime. n_events must be 6 (or events NULL). */
ES_API es_status es_moe_forward_timed(const es_moe_cfg* cfg, const void* x,
                                      const void* logits, int32_t logits_dtype,
                                      const float* cache_bias,
                                      const void* shared_gate_w, const void* packed,
                                      void* out, int32_t out_dtype,
                                      int32_t* topk_idx, float* topk_w, int32_t T,
                                      void* workspace, size_t workspace_bytes,
                                      es_stream_t stream, void* const* events,
                                      int32_t n_events);

/* ---------------------------------------------------------------------------
 * Expert parallelism (experts sharded over the GPUs of one box)
 * ------------------------------------------------------------------------- */

/* Routing masks for every destination rank: for d in [0, world), token t,
 * slot j:  send_idx[d][t][j] = local_id[e] if owner[e] == d else -1 (e =
 * topk_idx[t][j]), send_w[d][t][j] = topk_w[t][j]. owner / local_id map a
 * global expert id to its rank and to its index in that rank's shard.
 * `workspace` (optional, may be NULL) receives ES_DEVERR_BAD_EXPERT_ID.
 * Counterpart of the partition mask of compute_partial
 * (src/expert_network/node.py:158-163), computed once on the home rank. */
ES_API es_status es_ep_mask(const int32_t* topk_idx, const float* topk_w,
                            const int32_t* owner, const int32_t* local_id,
                            int32_t num_experts, int32_t top_k, int32_t T,
                            int32_t world, int32_t* send_idx, float* send_w,
                            void* workspace, es_stream_t stream);

/* out[t] = sum over r = 0..world-1, in that order, of partials[r][t] (fp32),
 * plus extra[t] when extra != NULL (e.g. the shared expert), cast to
 * out_dtype. partials [world][T][D] f32; 16-byte aligned buffers.
 * Counterpart of the fixed node-order sum of compute_distributed
 * (src/expert_network/reader.py:278-286). */
ES_API es_status es_ep_combine(const float* partials, const float* extra,
                               int32_t world, int32_t T, int32_t D, void* out,
                               int32_t out_dtype, es_stream_t stream);

/* ---- peer-to-peer exchange over NVLink (no collective library on the data
 * path). Each rank owns an exchange window (es_ep_window_*) that every other
 * rank of the box maps through CUDA IPC. Per layer step, in stream order:
 *   es_moe_route        home rank: top-k of its own tokens
 *   es_ep_dispatch      home rank: for every destination rank, the tokens
 *                       with at least one slot owned there, packed in token
 *                       order (bf16 row, token id, local expert ids or -1,
 *                       weights), written into that rank's window; then a
 *                       step flag
 *   es_ep_receive       owner rank: waits for every source's flag and lists
 *                       the received rows' routing for es_moe_expert_ffn
 *   es_moe_expert_ffn   owner rank: its experts on the received rows
 *   es_ep_return        owner rank: each row's fp32 partial written back
 *                       into its home rank's window, then a step flag
 *   es_ep_combine_p2p   home rank: waits for every owner's flag, sums the
 *                       partials of the owners each token used in rank
 *                       order (+ extra), advances the step counter
 * The step counter lives in the window, so a captured CUDA graph of the
 * whole step replays correctly. Every wait is bounded (about a second):
 * on timeout the kernel sets ES_DEVERR_TIMEOUT in `err` and returns.
 * Counterpart of the Expert Network's per-layer HTTP exchange:
 * src/expert_network/reader.py:237-292 (driver) and node.py:142-198 (node). */
typedef struct es_ep_plan {
  int32_t world, rank;
  int32_t cap;              /* most home tokens per rank and step            */
  int32_t hidden, top_k, num_experts;
  const int32_t* owner;     /* [E] device: rank that owns each global expert */
  const int32_t* local_id;  /* [E] device: index of the expert on its owner  */
  void* const* peers;       /* [world] device array: every rank's window base
                             * as mapped in this process (own one at [rank]) */
  void* window;             /* this rank's window                             */
  uint32_t* err;            /* device error word (e.g. a workspace's)         */
} es_ep_plan;

/* Bytes of one rank's exchange window for `world` ranks, `cap` home tokens
 * per step, hidden size and top-k. */
ES_API es_status es_ep_window_bytes(int32_t world, int32_t cap, int32_t hidden, int32_t top_k,
                                    size_t* bytes_out);
/* Allocate (cudaMalloc) and zero a window of `bytes` on the current device
 * and export it: *ipc_handle_out receives a 64-byte cudaIpcMemHandle_t. */
ES_API es_status es_ep_window_alloc(size_t bytes, void** window_out, void* ipc_handle_out);
/* Map a peer's window from its 64-byte handle (cudaIpcOpenMemHandle). */
ES_API es_status es_ep_window_open(const void* ipc_handle, void** window_out);
/* Unmap a peer's window / free this rank's own. */
ES_API es_status es_ep_window_close(void* peer_window);
ES_API es_status es_ep_window_free(void* window);

ES_API es_status es_ep_dispatch(const es_ep_plan* plan, const void* x_bf16,
                                const int32_t* topk_idx, const float* topk_w, int32_t T,
                                es_stream_t stream);
/* idx_out / w_out: [world * cap][k] routing of the window's received rows
 * (rows beyond a source's count: -1 / 0). The rows themselves are
 * window + es_ep_rows_offset(): [world * cap][hidden] bf16. */
ES_API es_status es_ep_receive(const es_ep_plan* plan, int32_t* idx_out, float* w_out,
                               es_stream_t stream);
ES_API es_status es_ep_rows_offset(const es_ep_plan* plan, size_t* offset_out);
/* y: [world * cap][hidden] fp32 partials of the received rows. */
ES_API es_status es_ep_return(const es_ep_plan* plan, const float* y, es_stream_t stream);
/* out[t] = sum over owners d (rank order) used by token t of the returned
 * partial (+ extra[t] if extra != NULL), as out_dtype; topk_idx is the home
 * routing passed to es_ep_dispatch. */
ES_API es_status es_ep_combine_p2p(const es_ep_plan* plan, const int32_t* topk_idx,
                                   const float* extra, int32_t T, void* out, int32_t out_dtype,
                                   es_stream_t stream);

/* es_moe_forward for callers that cannot allocate device memory (a runtime
 * that owns the whole GPU arena, a plugin whose host forbids outside
 * allocations, a loop where cudaMalloc's implicit synchronisation is not
 * allowed). Same arguments minus the workspace: the scratch is a 64 MiB
 * array built into the library, resident on every device that loads it
 * until the process exits. A batch whose es_moe_workspace_bytes exceeds
 * 64 MiB returns ES_ERR_WORKSPACE. The first call on a device resolves the
 * array's address (make it before any stream capture on that device). All
 * calls on a device share the array: order them on one stream, since calls
 * that overlap on the GPU race. Device error flags: es_moe_noalloc_read_error.
 * No counterpart in the reference (an addition of this library). */
ES_API es_status es_moe_forward_noalloc(const es_moe_cfg* cfg, const void* x,
                                        const void* logits, int32_t logits_dtype,
                                        const float* cache_bias,
                                        const void* shared_gate_w,
                                        const void* packed, void* out,
                                        int32_t out_dtype, int32_t* topk_idx,
                                        float* topk_w, int32_t T,
                                        es_stream_t stream);

/* The device error word (ES_DEVERR_* bits) of the last
 * es_moe_forward_noalloc call on the current device: each call clears it
 * first. Blocks the host on `stream`; clears it when `clear` != 0. */
ES_API es_status es_moe_noalloc_read_error(int32_t clear, uint32_t* flags_out,
                                           es_stream_t stream);

/* Synchronously read (and clear when `clear` != 0) the device error word of
 * a workspace. Blocks the host on `stream`. When ES_DEVERR_TIMEOUT is set by
 * the tensor-core kernels, the next three 32-bit words of the workspace hold
 * the first timed-out wait since they were last cleared (site id, CTA, stage
 * or unit); clearing resets them too. No reference counterpart. */
ES_API es_status es_moe_read_error(const void* workspace, int32_t clear,
                            uint32_t* flags_out, es_stream_t stream);

/* ---- decoder helpers: the caller's per-layer loop around the block ------
 * bf16 tensors, fp32 arithmetic. Counterparts of the MLX ops of the layer
 * loop in src/mlx_expert_sniper/generate.py:114-122 (input_layernorm,
 * residual adds, post_attention_layernorm) and of Qwen3 attention's q/k
 * norm + rotary + cache update (mlx_lm qwen3_moe Attention, called at
 * generate.py:118). */

/* For each of `rows` rows of `cols`: if delta != NULL, h += delta (rounded
 * to bf16 in place); then out = h * rsqrt(mean(h^2) + eps) * weight. */
ES_API es_status es_dec_add_rmsnorm(void* h, const void* delta, const void* weight,
                                    void* out, int32_t rows, int32_t cols, float eps,
                                    es_stream_t stream);

/* qkv [batch][(heads + 2*kv_heads) * head_dim] is one fused projection
 * (q heads, then k heads, then v heads). q and k heads get an RMS norm over
 * head_dim (weights q_norm / k_norm, result rounded to bf16) and the rotary
 * embedding of position *pos (device int64) on their two halves, from
 * cos_table / sin_table [max_ctx][head_dim/2] f32. q goes to q_out
 * [batch][heads][head_dim]; k and v are written to k_cache / v_cache
 * [batch][kv_heads][max_ctx][head_dim] at *pos. Requires *pos < max_ctx. */
ES_API es_status es_dec_qk_norm_rope_kv(const void* qkv, const void* q_norm,
                                        const void* k_norm, const float* cos_table,
                                        const float* sin_table, const int64_t* pos,
                                        void* q_out, void* k_cache, void* v_cache,
                                        int32_t batch, int32_t heads, int32_t kv_heads,
                                        int32_t head_dim, int32_t max_ctx, float eps,
                                        es_stream_t stream);

/* y[b][n] = sum_k weight[n][k] * x[b][k] for b < batch (1..4), bf16 in and
 * out, fp32 accumulation: the projections of a decode step at small batch
 * (x @ W^T with W [n][k] row-major). k % 8 == 0, 16-byte aligned weight and
 * x, batch * k * 2 <= 200 KB. */
ES_API es_status es_dec_gemv(const void* weight, const void* x, void* y, int32_t batch,
                             int32_t n, int32_t k, es_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ES_MOE_H */
