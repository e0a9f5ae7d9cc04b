// QACT / QST row quantization as a CTA-wide device routine (reference docs/isa.md
// "Quantization"; opentpu/fp32.py:321-343 quantize_mx; opentpu/isasim.py:913-959 QACT).
//
// One row x[0..n) of fp32 is quantized by the whole CTA:
//   amax = the largest |x| by bit pattern (after the flush), S = amax * f32(1/127),
//   inv = 127 * recip(amax) (S = inv = 0 for an all-zero row);
//   per group of g elements (g a multiple of 32): d = the group offset (0 in ROW mode),
//   q = q8(x * (inv * 2^d)).
// The row is first staged into shared memory with cp.async (every load in flight at once,
// so the latency is paid once, not once per segment); pass 1 reduces each 32-element
// segment's magnitude maximum with one warp reduction, the row maximum and the group maxima
// come from those, and pass 2 emits the bytes through a caller functor.
#pragma once
#include "otq_fp32.cuh"

namespace otq {

// The threads that run a row quantization together: the whole CTA (BAR = 0, a CTA barrier), or
// NT threads that meet on named barrier BAR. tid is the thread's index within the group.
template <int NT, int BAR = 0>
struct ThreadGroup {
  int tid;
  __device__ __forceinline__ void sync() const {
    if constexpr (BAR == 0) {
      __syncthreads();
    } else {
      asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
    }
  }
};

struct QactRowResult {
  float S;      // the row's scale
  float inv;    // 127 * recip(amax), or 0
  uint32_t amax_bits;
};

// Copy x[0..n) (global) into xs (shared) with cp.async, 16 bytes a copy when x is 16-byte
// aligned, else 4. The global side is read through L2 only (.cg / .ca on the first touch): x
// may have been written by the kernel launched just before this one. Ends with every copy
// complete and a barrier of the group.
template <int NT, int BAR>
__device__ __forceinline__ void stage_row(const ThreadGroup<NT, BAR>& grp,
                                          const float* __restrict__ x, float* xs, int n) {
  const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(xs));
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    for (int i = grp.tid * 4; i < n; i += NT * 4)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(base + 4u * i), "l"(x + i)
                   : "memory");
  } else {
    for (int i = grp.tid; i < n; i += NT)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(base + 4u * i), "l"(x + i)
                   : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  grp.sync();
}

// xs: the row in shared memory (stage_row); seg: shared scratch of n/32 words; red: shared
// scratch of 40 words. All threads of the group call it; emit(i, q, d_group) is called once per
// element i with the quantized byte and the offset of element i's group. The 32 lanes of a
// warp call emit together for the 32 elements of one segment, so emit may use warp
// collectives.
template <int NT, int BAR, class Emit>
__device__ __forceinline__ QactRowResult qact_row(const ThreadGroup<NT, BAR>& grp, const float* xs,
                                                  int n, int g, bool row_mode, uint32_t* seg,
                                                  uint32_t* red, Emit emit) {
  const int lane = grp.tid & 31;
  const int warp = grp.tid >> 5;
  constexpr int NW = NT / 32;
  const int nseg = n >> 5;
  // pass 1: segment maxima
  uint32_t tmax = 0u;
  for (int s = warp; s < nseg; s += NW) {
    const float v = otq_flush(xs[(s << 5) + lane]);
    const uint32_t mb = __float_as_uint(v) & 0x7FFFFFFFu;
    const uint32_t sm = __reduce_max_sync(0xFFFFFFFFu, mb);
    if (lane == 0) seg[s] = sm;
    tmax = sm > tmax ? sm : tmax;   // identical on every lane
  }
  if (lane == 0) red[warp] = tmax;
  grp.sync();
  if (warp == 0) {
    uint32_t m = lane < NW ? red[lane] : 0u;
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if (lane == 0) {
      float S = 0.0f, inv = 0.0f;
      if (m != 0u) {
        const float amax = __uint_as_float(m);
        S = fmul(amax, __uint_as_float(kInv127Bits));
        inv = fmul(127.0f, recip(amax));
      }
      red[NW] = __float_as_uint(S);
      red[NW + 1] = __float_as_uint(inv);
      red[NW + 2] = m;
    }
  }
  grp.sync();
  QactRowResult r;
  r.S = __uint_as_float(red[NW]);
  r.inv = __uint_as_float(red[NW + 1]);
  r.amax_bits = red[NW + 2];
  // pass 2: offsets and bytes
  const int spg = g >> 5;   // segments per group
  for (int s = warp; s < nseg; s += NW) {
    int d = 0;
    if (!row_mode) {
      const int s0 = (s / spg) * spg;
      uint32_t gm = 0u;
      for (int t = 0; t < spg; ++t) gm = max(gm, seg[s0 + t]);
      d = group_offset(gm, r.amax_bits);
    }
    const float scale = fmul(r.inv, pow2i(d));
    const int i = (s << 5) + lane;
    const int qv = q8(fmul(xs[i], scale));
    emit(i, qv, d);
  }
  grp.sync();   // seg / red / xs are reused by the next row
  return r;
}

}  // namespace otq

namespace otq {

__device__ __forceinline__ float4 ld_cg4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t mag_bits(float v) {
  return __float_as_uint(otq_flush(v)) & 0x7FFFFFFFu;
}

// The same QACT as qact_row for 32-element groups, four elements a thread at a time: one pass
// reads x (straight from global memory through L2: x may be the output of the kernel launched
// just before, read after griddepcontrol.wait; or, with x and xt null, from xs itself) into xs, with each 32-element segment's maximum
// from an 8-lane shuffle reduction; one more pass quantizes. n % 128 == 0; all NT threads of
// the CTA call it. x4: x is 16-byte aligned (else four scalar loads). segm: shared scratch of
// n/32 words; red: of NT/32 + 3 words. emit(i, q0, q1, q2, q3, d) gets elements 4i..4i+3 and
// their group's offset; the 8 threads of a group call it together (lanes 8k..8k+7 of a warp).
// Ends with a barrier.
// Two (value, tag) words of a tagged row: each 8-byte element is read single-copy atomically,
// bypassing L1 (the row is written by other GPUs while this kernel runs).
__device__ __forceinline__ void ld_tagged2(const unsigned long long* p, unsigned long long& a,
                                           unsigned long long& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// The word's tag is behind `expect` (serial-number order: tags may wrap around 2^32).
__device__ __forceinline__ bool behind(unsigned long long w, uint32_t expect) {
  return static_cast<int>(static_cast<uint32_t>(w >> 32) - expect) < 0;
}

// BAR: 0 -- the whole CTA meets on __syncthreads (NT = the CTA's threads); else the NT threads
// 0 .. NT - 1 meet on named barrier BAR (the CTA's other threads do something else).
// ASYNC: every thread's cp.async copies are completed before the last barrier (the caller's
// copies issued before the call are then visible to the whole group).
template <int NT, int BAR = 0, bool ASYNC = false, class Emit4>
__device__ __forceinline__ QactRowResult qact_row4(const float* __restrict__ x, bool x4, float* xs,
                                                   int n, bool row_mode, uint32_t* segm,
                                                   uint32_t* red, Emit4 emit,
                                                   const unsigned long long* xt = nullptr,
                                                   uint32_t expect = 0, int* status = nullptr,
                                                   float* S_out = nullptr,
                                                   uint32_t limit = 1u << 22) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = NT / 32;
  const int n4 = n >> 2;   // a multiple of 32: every lane of a warp runs the same iterations
  uint32_t tmax = 0u;
  // x comes from L2 (the previous kernel wrote it): all of a thread's loads of a batch are in
  // flight together, so the prologue pays one memory latency a batch, not one a chunk
  constexpr int kB = 4;
  for (int i0 = tid; i0 < n4; i0 += NT * kB) {
    float4 v[kB];
    unsigned long long w[kB][4];
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const int i = i0 + b * NT;   // warp-uniform bound: n4 is a multiple of 32
      if (i >= n4) continue;
      if (xt != nullptr) {
        ld_tagged2(xt + 4 * i, w[b][0], w[b][1]);
        ld_tagged2(xt + 4 * i + 2, w[b][2], w[b][3]);
      } else if (x == nullptr) {
        v[b] = *reinterpret_cast<const float4*>(xs + 4 * i);   // the row is in xs already
      } else if (x4) {
        v[b] = ld_cg4(x + 4 * i);
      } else {
        v[b].x = __ldcg(x + 4 * i);
        v[b].y = __ldcg(x + 4 * i + 1);
        v[b].z = __ldcg(x + 4 * i + 2);
        v[b].w = __ldcg(x + 4 * i + 3);
      }
    }
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const int i = i0 + b * NT;
      if (i >= n4) continue;
      if (xt != nullptr) {
        // a tagged row (value in the low word, the writer's tag in the high word): wait,
        // bounded (`limit` polls), until the four elements carry at least the expected tag
        for (uint32_t spin = 0;
             behind(w[b][0], expect) || behind(w[b][1], expect) || behind(w[b][2], expect) ||
             behind(w[b][3], expect);
             ++spin) {
          if (spin >= limit) {
            if (status != nullptr) atomicOr(status, 1);   // a writer never arrived: not valid
            break;
          }
          if (spin >= 16) __nanosleep(32);
          ld_tagged2(xt + 4 * i, w[b][0], w[b][1]);
          ld_tagged2(xt + 4 * i + 2, w[b][2], w[b][3]);
        }
        v[b] = make_float4(__uint_as_float(static_cast<uint32_t>(w[b][0])),
                           __uint_as_float(static_cast<uint32_t>(w[b][1])),
                           __uint_as_float(static_cast<uint32_t>(w[b][2])),
                           __uint_as_float(static_cast<uint32_t>(w[b][3])));
      }
      *reinterpret_cast<float4*>(xs + 4 * i) = v[b];
      uint32_t m = max(max(mag_bits(v[b].x), mag_bits(v[b].y)), max(mag_bits(v[b].z), mag_bits(v[b].w)));
      m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
      m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
      m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, 4));
      if ((lane & 7) == 0) segm[i >> 3] = m;
      tmax = max(tmax, m);
    }
  }
  tmax = __reduce_max_sync(0xFFFFFFFFu, tmax);
  if (lane == 0) red[warp] = tmax;
  if constexpr (BAR == 0) { __syncthreads(); } else { asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory"); }
  // every warp reduces the warp maxima and derives the scales itself: one barrier, not two
  uint32_t m = lane < NW ? red[lane] : 0u;
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  QactRowResult r;
  r.S = 0.0f;
  r.inv = 0.0f;
  r.amax_bits = m;
  if (m != 0u) {
    const float amax = __uint_as_float(m);
    r.S = fmul(amax, __uint_as_float(kInv127Bits));
    r.inv = fmul(127.0f, recip(amax));
  }
  if (S_out != nullptr && tid == 0) *S_out = r.S;   // ordered before its readers by the barrier below
  for (int i = tid; i < n4; i += NT) {
    const float4 v = *reinterpret_cast<const float4*>(xs + 4 * i);
    const int d = row_mode ? 0 : group_offset(segm[i >> 3], r.amax_bits);
    const float scale = fmul(r.inv, pow2i(d));
    emit(i, q8(fmul(v.x, scale)), q8(fmul(v.y, scale)), q8(fmul(v.z, scale)), q8(fmul(v.w, scale)), d);
  }
  if constexpr (ASYNC) asm volatile("cp.async.wait_all;" ::: "memory");
  if constexpr (BAR == 0) { __syncthreads(); } else { asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory"); }
  return r;
}

}  // namespace otq
