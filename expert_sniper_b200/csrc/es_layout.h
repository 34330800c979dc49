// Packed weight layout and workspace layout of the MoE block. Shared by host
// and device code.
//
// Packed layout (one layer, built once by es_moe_prepare):
//   experts 0..E-1 (then the shared expert, if any), each exactly
//   3*D*I*9/16 bytes -- the reference's per-expert bytes, no padding.
//   Inside an expert (rb = 16-row block):
//     gate/up region: for each pair of row blocks, G in [0, D/64), the two
//                     blocks, proj in {gate, up}: one 576-byte tile
//     down region:    for each quad of row blocks, G in [0, I/64), the four
//                     blocks: one 576-byte tile
//   so a warp streaming one (pair or quad, group) run gets all tiles that
//   share one activation fragment.
//   A tile covers 16 rows x 64 columns (one quantisation group):
//     bytes [0, 512)  codes. Lane l = 4*g + c of a warp owns bytes
//                     [16l, 16l + 16): words 2c and 2c+1 of the group for
//                     row g, then the same two words for row g + 8 -- the
//                     exact A fragment of four m16n8k16 steps.
//     bytes [512, 576) for g in 0..7: (scale, bias) of row g then of row
//                     g + 8, fp16 each -- 8 bytes per g.
//   Column k of a tile row is nibble k % 8 of word k / 8, as in MLX.
//
// Activation operand layout ("fragment order"), used for x and h: a row of
// K values is stored as K/16 chunks of 16; chunk q holds, for s in 0..3 and
// slot in 0..3, element 16q + s + 4*slot at position 4s + slot. A lane that
// reads chunk q of a group gets its two B-fragment registers for each of the
// four k-steps as consecutive words.
//
// Nibble order (tensor-core path, x16 and h rows): each run of 8 values
// 8q..8q+7 is stored as 8q + {0, 4, 1, 5, 2, 6, 3, 7} -- the order in which
// one packed code word converts to four fp16 pairs (nibbles s and s + 4 per
// pair) -- so weights and activations share one K permutation.
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifndef __CUDACC__
#define __host__
#define __device__
#endif

namespace es {

constexpr int kGroup = 64;
constexpr int kTileBytes = 576;
constexpr int kTileCodeBytes = 512;
constexpr int kMaxTopK = 16;
constexpr int kMaxExperts = 1024;
constexpr int kMaxSplitK = 8;         // K split of gate/up items for tiny batches
constexpr int kSplitKMaxTokens = 8;   // ... used only up to this many tokens
// the fused one-launch kernel: most tokens, and most pairs of one expert
// entry (an expert with more pairs takes several entries of this many)
constexpr int kSmallMaxTokens = 16;
constexpr int kSmallEntryPairs = 8;
// its K split: kMaxSplitK shares up to kSplitKMaxTokens tokens, this many
// above (twice the entries, half the shares: the same partials)
constexpr int kSmallSplitKLarge = 4;

__host__ __device__ inline size_t expert_bytes(int D, int I) {
  return (size_t)3 * D * I * 9 / 16;
}
__host__ __device__ inline size_t gateup_region_bytes(int D, int I) {
  return (size_t)2 * D * I * 9 / 16;
}
// gate/up tiles: pairs of 16-row blocks, then group, then block of the pair,
// then (gate, up): the 4 tiles of one (pair, group) are contiguous.
__host__ __device__ inline size_t gateup_tile_off(int GD, int rb, int G, int proj) {
  return ((((size_t)(rb >> 1) * GD + G) * 2 + (rb & 1)) * 2 + proj) * kTileBytes;
}
// down tiles: quads of 16-row blocks, then group, then block of the quad:
// the 4 tiles of one (quad, group) are contiguous.
__host__ __device__ inline size_t down_tile_off(int D, int I, int rb, int G) {
  return gateup_region_bytes(D, I) +
         (((size_t)(rb >> 2) * (I / kGroup) + G) * 4 + (rb & 3)) * kTileBytes;
}
// position of element d (0..K-1) of a row in fragment order
__host__ __device__ inline int frag_pos(int d) {
  const int q = d >> 4, r = d & 15;
  return (q << 4) + 4 * (r & 3) + (r >> 2);
}

// position of element i of a row in nibble order
__host__ __device__ inline int nib_pos(int i) {
  return (i & ~7) | (((i & 3) << 1) | ((i >> 2) & 1));
}

__host__ __device__ inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Device pointers carved from the caller's workspace for a call with T tokens.
struct Workspace {
  uint32_t* err;       // [64] error word + reserved
  uint32_t* bitmap;    // [E1][W]   token bitmap per expert
  int32_t* wpre;       // [E1][W]   exclusive popcount prefix per word
  int32_t* n_active;   // [1]
  int32_t* act_e;      // [E1]      active expert ids, ascending
  int32_t* act_off;    // [E1]      first sorted pair of each active expert
  int32_t* act_n;      // [E1]      pairs of each active expert
  int32_t* pair_tok;   // [P]       token of each sorted pair
  int32_t* pos;        // [T]       pair of the shared expert
  int32_t* cs_pos;     // [T][k]    pairs of a token in expert id order
  float* cs_w;         // [T][k]    their weights
  int32_t* rank;       // [T][k]    tensor-core path: slot's rank inside its expert
  int32_t* topk_idx;   // [T][k]
  float* topk_w;       // [T][k]
  float* sgate;        // [T]       shared-expert gate
  uint16_t* x_perm;    // [T][D]    bf16, fragment order (decode kernels);
                       //           tensor-core path: scaled fp16, nibble order
  float* xsum;         // [T][D/64] (decode kernels); tensor-core path: [T]
                       //           inverse power-of-two scale of each x16 row
  uint16_t* h16;       // [P][I]    fp16 h, fragment order (decode) or nibble
                       //           order (tensor-core path)
  float* y_pair;       // [P][D]    fp32 (decode); fp16 [P][D] (tensor-core path)
  float* partials;     // split-K partials (T <= 8): [slot][KS][512]
  int* counters;       // split-K arrivals per slot; zero between calls
  int* ticket;         // front-end CTAs done; zero between calls
  int* item_ctr;       // [2] FFN work counters
  int W, P, kk, E1;
  size_t bytes;
  // regions the kernels expect at zero when a call starts (they leave them
  // at zero when a call completes): the error block and control words from
  // `err`, the token bitmaps (tensor-core path: slot counters) from
  // `bitmap`, the split-K arrival counters from `counters`
  size_t zero_ctl_bytes, zero_bitmap_bytes, zero_counter_bytes;
  size_t part_slots;   // 2 KB split-K slots in `partials`
};

// Carve (or, with base == nullptr, just size) the workspace for T tokens.
inline Workspace carve_workspace(void* base, int D, int E, int k, int I,
                                 int has_shared, int T) {
  Workspace w{};
  const int E1 = E + (has_shared ? 1 : 0);
  const int W = (T + 31) / 32 > 0 ? (T + 31) / 32 : 1;
  const int kk = k + (has_shared ? 1 : 0);
  const int P = (T > 0 ? T : 1) * kk;
  const int Tm = T > 0 ? T : 1;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  size_t o_err = take(256);
  size_t o_ctl = take(256);
  // The regions that must be zero when a call starts sit first, at offsets
  // that do not depend on T, so that calls with different T on one
  // workspace find them zero: the counters (the split-K arrivals of the
  // decode kernels, used up to kSplitKMaxTokens tokens, and the fused
  // tiny-batch kernel's two barrier words), sized for kSplitKMaxTokens
  // tokens whatever T is; then the token bitmaps, whose size grows with T
  // (a smaller T uses a prefix of the region).
  const size_t As8 = (size_t)(((long long)kSplitKMaxTokens * k < E ? kSplitKMaxTokens * k : E) +
                              (has_shared ? 1 : 0));
  const size_t cnt_all = As8 * (I / 32) > As8 * (D / 64) ? As8 * (I / 32) : As8 * (D / 64);
  size_t o_cnt = take(cnt_all * 4);
  size_t o_bitmap = take((size_t)E1 * W * 4);
  size_t o_wpre = take((size_t)E1 * W * 4);
  size_t o_nact = take(4);
  size_t o_acte = take((size_t)E1 * 4);
  size_t o_actoff = take((size_t)E1 * 4);
  size_t o_actn = take((size_t)E1 * 4);
  size_t o_ptok = take((size_t)P * 4);
  size_t o_pos = take((size_t)Tm * kk * 4);
  size_t o_cspos = take((size_t)Tm * k * 4);
  size_t o_csw = take((size_t)Tm * k * 4);
  size_t o_rank = take((size_t)Tm * k * 4);
  size_t o_tidx = take((size_t)Tm * k * 4);
  size_t o_tw = take((size_t)Tm * k * 4);
  size_t o_sg = take((size_t)Tm * 4);
  size_t o_xp = take((size_t)Tm * D * 2);
  size_t o_xs = take((size_t)Tm * (D / kGroup) * 4);
  size_t o_hh = take((size_t)P * I * 2);
  size_t o_y = take((size_t)P * D * 4);
  // split-K partials: the decode kernels use them up to kSplitKMaxTokens
  // tokens (one entry per active expert, kMaxSplitK shares); the fused kernel
  // the same way, and from there up to kSmallMaxTokens with entries of at
  // most kSmallEntryPairs pairs and kSmallSplitKLarge shares. Larger T keeps
  // the largest amount, so the size never shrinks as T grows.
  const long long Ts = Tm < kSplitKMaxTokens ? Tm : kSplitKMaxTokens;
  const size_t As = (size_t)((Ts * k < E ? Ts * k : E) + (has_shared ? 1 : 0));
  size_t shares = As * kMaxSplitK;   // entries x shares, per row pair / quad
  if (Tm > kSplitKMaxTokens) {
    const long long Tf = Tm < kSmallMaxTokens ? Tm : kSmallMaxTokens;
    const long long per_e = (Tf + kSmallEntryPairs - 1) / kSmallEntryPairs;
    const long long routed = Tf * k < (long long)E * per_e ? Tf * k : (long long)E * per_e;
    const size_t Af = (size_t)(routed + (has_shared ? per_e : 0));
    if (Af * kSmallSplitKLarge > shares) shares = Af * kSmallSplitKLarge;
  }
  // split-K slots of gate/up (row pairs) and down (row quads), 2 KB each
  const size_t gu_slots = shares * (I / 32);
  const size_t dn_slots = shares * (D / 64);
  const size_t part_items = gu_slots > dn_slots ? gu_slots : dn_slots;
  size_t o_part = take(part_items * 512 * 4);
  w.part_slots = part_items;
  w.bytes = off;
  w.zero_ctl_bytes = o_cnt - o_err;
  w.zero_bitmap_bytes = (size_t)E1 * W * 4;
  w.zero_counter_bytes = cnt_all * 4;
  w.W = W;
  w.P = P;
  w.kk = kk;
  w.E1 = E1;
  if (base) {
    char* b = static_cast<char*>(base);
    w.err = reinterpret_cast<uint32_t*>(b + o_err);
    w.ticket = reinterpret_cast<int*>(b + o_ctl);
    w.item_ctr = reinterpret_cast<int*>(b + o_ctl) + 1;
    w.bitmap = reinterpret_cast<uint32_t*>(b + o_bitmap);
    w.wpre = reinterpret_cast<int32_t*>(b + o_wpre);
    w.n_active = reinterpret_cast<int32_t*>(b + o_nact);
    w.act_e = reinterpret_cast<int32_t*>(b + o_acte);
    w.act_off = reinterpret_cast<int32_t*>(b + o_actoff);
    w.act_n = reinterpret_cast<int32_t*>(b + o_actn);
    w.pair_tok = reinterpret_cast<int32_t*>(b + o_ptok);
    w.pos = reinterpret_cast<int32_t*>(b + o_pos);
    w.cs_pos = reinterpret_cast<int32_t*>(b + o_cspos);
    w.cs_w = reinterpret_cast<float*>(b + o_csw);
    w.rank = reinterpret_cast<int32_t*>(b + o_rank);
    w.topk_idx = reinterpret_cast<int32_t*>(b + o_tidx);
    w.topk_w = reinterpret_cast<float*>(b + o_tw);
    w.sgate = reinterpret_cast<float*>(b + o_sg);
    w.x_perm = reinterpret_cast<uint16_t*>(b + o_xp);
    w.xsum = reinterpret_cast<float*>(b + o_xs);
    w.h16 = reinterpret_cast<uint16_t*>(b + o_hh);
    w.y_pair = reinterpret_cast<float*>(b + o_y);
    w.partials = reinterpret_cast<float*>(b + o_part);
    w.counters = reinterpret_cast<int*>(b + o_cnt);
  }
  return w;
}

// Expert-parallel exchange window of one rank (es_ep_*): device memory
// that the other ranks of the box map (CUDA IPC) and write into directly
// over NVLink. Every rank carves the same layout, so a rank finds a peer's
// fields from the peer's base pointer. Written by peers: flags_in, cnt_in,
// rows_in, tok_in, idx_in, w_in (one region per source rank) and flags_ret,
// ret_in (one region per owner rank). Local only: epoch and tickets.
struct EpWindow {
  uint32_t* epoch;     // [1]   steps completed by this rank
  int* tickets;        // [3 * world] CTA tickets of dispatch / return / combine
  uint32_t* flags_in;  // [world] step whose rows source s has delivered
  uint32_t* flags_ret; // [world] step whose partials owner d has delivered
  int32_t* cnt_in;     // [world] rows source s sent in its last step
  uint16_t* rows_in;   // [world][cap][D] bf16 activation rows, by source
  int32_t* tok_in;     // [world][cap] home token of each row
  int32_t* idx_in;     // [world][cap][k] local expert ids (-1: not ours)
  float* w_in;         // [world][cap][k] routing weights
  float* ret_in;       // [world][cap][D] fp32 partials of my tokens, by owner
  size_t bytes;
};

__host__ __device__ inline EpWindow carve_ep_window(void* base, int world, int cap, int D, int k) {
  EpWindow w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t rows = (size_t)world * cap;
  size_t o_epoch = take(4);
  size_t o_tk = take((size_t)3 * world * 4);
  size_t o_fin = take((size_t)world * 4);
  size_t o_fret = take((size_t)world * 4);
  size_t o_cnt = take((size_t)world * 4);
  size_t o_rows = take(rows * D * 2);
  size_t o_tok = take(rows * 4);
  size_t o_idx = take(rows * k * 4);
  size_t o_w = take(rows * k * 4);
  size_t o_ret = take(rows * D * 4);
  w.bytes = off;
  if (base) {
    char* b = static_cast<char*>(base);
    w.epoch = reinterpret_cast<uint32_t*>(b + o_epoch);
    w.tickets = reinterpret_cast<int*>(b + o_tk);
    w.flags_in = reinterpret_cast<uint32_t*>(b + o_fin);
    w.flags_ret = reinterpret_cast<uint32_t*>(b + o_fret);
    w.cnt_in = reinterpret_cast<int32_t*>(b + o_cnt);
    w.rows_in = reinterpret_cast<uint16_t*>(b + o_rows);
    w.tok_in = reinterpret_cast<int32_t*>(b + o_tok);
    w.idx_in = reinterpret_cast<int32_t*>(b + o_idx);
    w.w_in = reinterpret_cast<float*>(b + o_w);
    w.ret_in = reinterpret_cast<float*>(b + o_ret);
  }
  return w;
}

}  // namespace es
