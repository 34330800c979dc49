// Device helpers shared by the MoE block kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "es_layout.h"

#define ES_DEV __device__ __forceinline__

namespace es {

// ---------------------------------------------------------------------------
// 4-bit codes -> bf16 operands.
//
// A bf16 with bits 0x4300 | q (q < 128) is exactly 128 + q, so OR-ing a
// nibble into the mantissa of 128.0 converts it with one LOP3 and no
// rounding. For a packed word w (code n at bits 4n), pair s (0..3) gives
// the bf16x2 (128 + n_s, 128 + n_{s+4}): the low half holds nibble s, the
// high half nibble s + 4.
// ---------------------------------------------------------------------------
ES_DEV uint32_t code_pair(uint32_t w, int s) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n"
      : "=r"(r)
      : "r"(w >> (4 * s)), "r"(0x000F000Fu), "r"(0x43004300u));
  return r;
}

// Makes `v` opaque at this point of the program: values computed from it
// below cannot be hoisted above (used to keep code conversions inside the
// token loop instead of holding all of them in registers).
ES_DEV void opaque(uint32_t& v) { asm volatile("" : "+r"(v)); }

// Same for fp16 operands: 0x6400 | q is exactly 1024 + q.
ES_DEV uint32_t code_pair_f16(uint32_t w, int s) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n"
      : "=r"(r)
      : "r"(w >> (4 * s)), "r"(0x000F000Fu), "r"(0x64006400u));
  return r;
}

ES_DEV void mma_f16(float (&d)[4], const uint32_t a0, const uint32_t a1, const uint32_t a2,
                    const uint32_t a3, const uint32_t b0, const uint32_t b1, const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]),
        "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// D = A * B + C, m16n8k16, bf16 inputs, fp32 accumulate (register operands:
// the decode GEMV converts codes in registers and never stages them in
// shared memory).
ES_DEV void mma_bf16(float (&d)[4], const uint32_t a0, const uint32_t a1,
                     const uint32_t a2, const uint32_t a3, const uint32_t b0,
                     const uint32_t b1, const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]),
        "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// Streaming 16-byte load of packed weights: read once, keep out of L1.
ES_DEV uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// The same 16-byte streaming load with an L2 cache policy (createpolicy),
// e.g. evict-first for data read once per call, so that it is the first
// to leave L2 and the small data and code around it stay.
ES_DEV uint4 ld_stream16_pol(const void* p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}
ES_DEV uint2 ld_nc8_pol(const void* p, uint64_t pol) {
  uint2 r;
  asm volatile("ld.global.nc.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;\n"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p), "l"(pol));
  return r;
}

ES_DEV uint2 ld_stream8(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

ES_DEV float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

ES_DEV float half_bits_to_float(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

ES_DEV float lo_half_f(uint32_t v) { return half_bits_to_float(v & 0xFFFFu); }
ES_DEV float hi_half_f(uint32_t v) { return half_bits_to_float(v >> 16); }

// Round-to-nearest-even fp32 -> bf16 bits.
ES_DEV uint16_t float_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Orderable key of a float: larger float -> larger unsigned key. NaN maps to
// 0 (below -inf) so it is never selected.
ES_DEV uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (f != f) return 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

ES_DEV float silu_f(float g) { return g / (1.0f + __expf(-g)); }

ES_DEV void set_error(uint32_t* err, uint32_t bit) {
  if (err) atomicOr(err, bit);
}

// ---------------------------------------------------------------------------
// Bulk async copies (TMA engine, non-tensor form) into shared memory,
// completed through an mbarrier transaction count. No cluster multicast.
// ---------------------------------------------------------------------------
ES_DEV uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

ES_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count));
}

ES_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

ES_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// global -> shared bulk copy; dst, src 16-byte aligned, bytes % 16 == 0
ES_DEV void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;\n" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// L2 policy for data read exactly once (streamed expert weights)
ES_DEV uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}

// The waiting thread is suspended (issuing nothing) until the phase completes
// or about a millisecond passes, so waiting warps leave the issue slots to
// the warps that work.
ES_DEV bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(phase), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Non-blocking test of the same condition.
ES_DEV bool mbar_test_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after ~2^31 SM cycles (about a second) and reports it.
ES_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
  if (mbar_test_wait(bar, phase)) return true;  // fast path: no clock read
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, phase)) {
    if (clock64() - t0 > (1LL << 31)) return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while the previous kernel of the stream is still
// running; pdl_wait() blocks until that kernel has completed and its writes
// are visible, pdl_trigger() lets the next kernel start launching. Both are
// no-ops for a normal launch.
// ---------------------------------------------------------------------------
ES_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
ES_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// Shared-memory loads as plain C++ so the compiler orders them after the
// mbarrier waits (asm volatile with a memory clobber) that publish the data.
ES_DEV uint4 ld_shared16(const void* p) { return *reinterpret_cast<const uint4*>(p); }
ES_DEV uint2 ld_shared8(const void* p) { return *reinterpret_cast<const uint2*>(p); }

}  // namespace es
