// Device helpers shared by the MM kernels: streaming loads, programmatic dependent launch,
// the integer MMA, and the in-register decoders of openTPU's packed 4-bit elements (reference
// opentpu/quant.py:264-266 DEC_INT4 / DEC_FP4, 275-278 unpack4).
#pragma once
#include <cstdint>

namespace otq {

// Weight bytes are read once: bypass L1, and ask L2 to fetch the whole 256-byte segment.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ld_stream4(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Bring [p, p + bytes) into L2 (bytes a multiple of 16, p 16-byte aligned).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// D = A (16x32 s8, row) * B (32x8 s8, col), exact int32 (the C input is zero).
__device__ __forceinline__ void imma(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                     uint32_t b0, uint32_t b1, int (&d)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// d += A * B (exact while the sums stay below 2^31).
__device__ __forceinline__ void imma_acc(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, int (&d)[4]) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// E2M1 codes (stored doubled: {0,1,2,3,4,6,8,12}, sign in bit 3) of one 8-nibble word ->
// exact signed bytes: elements 0..3 in lo, 4..7 in hi.
__device__ __forceinline__ void fp4_bytes(uint32_t w, uint32_t& lo, uint32_t& hi) {
  constexpr uint32_t kPosLo = 0x03020100u, kPosHi = 0x0C080604u;   // +0 +1 +2 +3 | +4 +6 +8 +12
  constexpr uint32_t kNegLo = 0xFDFEFF00u, kNegHi = 0xF4F8FAFCu;   // -0 -1 -2 -3 | -4 -6 -8 -12
  const uint32_t sel_lo = w & 0x7777u, sel_hi = (w >> 16) & 0x7777u;
  const uint32_t w4 = w << 4;
  const uint32_t s_lo = prmt(w4, w, 0xD9C8u);   // nibble k's sign bit replicated over byte k
  const uint32_t s_hi = prmt(w4, w, 0xFBEAu);
  lo = (prmt(kPosLo, kPosHi, sel_lo) & ~s_lo) | (prmt(kNegLo, kNegHi, sel_lo) & s_lo);
  hi = (prmt(kPosLo, kPosHi, sel_hi) & ~s_hi) | (prmt(kNegLo, kNegHi, sel_hi) & s_hi);
}

// int4 two's-complement nibbles of one word -> value + 8 (0..15) as bytes: the even elements
// (low nibbles) in lo, the odd ones in hi.
__device__ __forceinline__ void int4_bytes(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x8 = w ^ 0x88888888u;
  lo = x8 & 0x0F0F0F0Fu;
  hi = (x8 >> 4) & 0x0F0F0F0Fu;
}

// m << (shA - dw), or 0 where the shift is negative (the group is below the window).
__device__ __forceinline__ int shifted(int m, int shA, int dw) {
  const int sh = shA - dw;
  return sh >= 0 ? (m << sh) : 0;
}

// An nvfp4 sub-block scale byte (E4M3, positive) -> multiplier m and offset dw (reference
// opentpu/quant.py:370-401 _nv; docs/isa.md MX scale rows): m = E ? 8 + M : M,
// dw = 15 - max(E, 1).
__device__ __forceinline__ void e4m3_term(uint32_t e, int& m, int& dw) {
  const int E = static_cast<int>((e >> 3) & 15u);
  m = E ? 8 + static_cast<int>(e & 7u) : static_cast<int>(e & 7u);
  dw = 15 - max(E, 1);
}

}  // namespace otq

namespace otq {

// ---------------------------------------------------------------- mbarriers and bulk copies
// Every wait is bounded: after kSpinLimit polls (about half a second with the back-off) it
// records kStatusTimeout in the library's status word and returns false.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// Make barrier initializations visible to the async proxy (bulk copies) and the other threads.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* status) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i >= 16) __nanosleep(64);
  }
  if (status != nullptr) atomicOr(status, 1);   // kStatusTimeout
  return false;
}
// [src, src + bytes) -> shared dst (this CTA only), completing `bytes` of transaction on bar.
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst), "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

}  // namespace otq
