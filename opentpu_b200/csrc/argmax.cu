// Greedy token selection on the device: the index of the first maximum of a logit row, the
// reference's greedy sink (llm/generate.py:252-280 over qwen3._lm_head, qwen3.py:2052-2087:
// numpy argmax, ties to the lowest id), so the decode loop reads back one id instead of the row.
//
// Each element becomes a 64-bit key, ord(value) << 32 | ~index, where ord maps fp32 to an
// unsigned integer of the same order (negative values complemented, non-negative ones with the
// sign bit set): the largest key is the largest value and, among equal values, the lowest index.
// Threads reduce their elements, warps and CTAs reduce by shuffles and shared memory, and each
// CTA folds its key into the accumulator word with one 64-bit atomicMax; the CTA that finishes
// last (a count in the second word) turns the key into the index. Both words are zeroed by a
// memset on the same stream before the launch.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "otq_internal.h"

namespace otq {
namespace {

constexpr int kArgThreads = 512;

// numpy's comparison: -0 equals +0, and a NaN is larger than everything (argmax stops at the
// first NaN), so both zeros map to one key and every NaN to the largest.
__device__ __forceinline__ unsigned long long key_of(float v, uint32_t i) {
  uint32_t b = __float_as_uint(v);
  if ((b & 0x7FFFFFFFu) == 0u) b = 0u;
  const uint32_t o = (b & 0x7FFFFFFFu) > 0x7F800000u ? 0xFFFFFFFFu
                     : (b & 0x80000000u)             ? ~b
                                                     : (b | 0x80000000u);
  return (static_cast<unsigned long long>(o) << 32) | (0xFFFFFFFFu - i);
}

// acc: [key accumulator, finished-CTA count], both zero at launch. The last CTA writes the
// index to *index (which may be acc itself) and leaves the count at zero.
__global__ void __launch_bounds__(kArgThreads) argmax_kernel(const float* __restrict__ x, int64_t n,
                                                            int64_t stride, int64_t* acc,
                                                            int64_t* index) {
  unsigned long long best = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kArgThreads + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kArgThreads) {
    const unsigned long long k = key_of(__ldg(x + i * stride), static_cast<uint32_t>(i));
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    best = v > best ? v : best;
  }
  __shared__ unsigned long long part[kArgThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgThreads / 32; ++w) best = part[w] > best ? part[w] : best;
    atomicMax(reinterpret_cast<unsigned long long*>(acc), best);
    __threadfence();
    if (atomicAdd(reinterpret_cast<unsigned long long*>(acc + 1), 1ull) == gridDim.x - 1) {
      const unsigned long long k = atomicMax(reinterpret_cast<unsigned long long*>(acc), 0ull);
      acc[1] = 0;
      *index = static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
    }
  }
}

}  // namespace

int argmax_launch(const float* x, int64_t n, int64_t stride, int64_t* acc, int64_t* index,
                  cudaStream_t stream) {
  if (cudaMemsetAsync(acc, 0, 2 * sizeof(int64_t), stream) != cudaSuccess) return kErrCuda;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  const int64_t want = (n + kArgThreads * 8 - 1) / (kArgThreads * 8);   // 8 elements a thread
  const int grid = static_cast<int>(want < 1 ? 1 : (want > sm_count(dev) ? sm_count(dev) : want));
  argmax_kernel<<<grid, kArgThreads, 0, stream>>>(x, n, stride, acc, index);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace otq

// ---------------------------------------------------------------- the allocation-free variant
// The same kernel with its two scratch words (key accumulator, CTA count) in this library's own
// device memory instead of the caller's: for callers that can only write into buffers they are
// handed. The array below is a module variable, present on every GPU that loads the library
// until the process exits; its device address comes from cudaGetSymbolAddress, once per device
// (host code only sees a host-side stand-in under the array's name). Every call shares it: the
// launch zeroes both words first (cudaMemsetAsync on the caller's stream), and calls that
// overlap on the GPU race on them.
namespace otq {
namespace {

// A call uses words 0 and 1 only (every call the same two); the array is 256 bytes so that it
// starts and ends on its own 256-byte boundary, not to give calls separate slots.
constexpr int kNoAllocScratchWords = 32;
static __device__ __align__(256) int64_t g_argmax_scratch[kNoAllocScratchWords];

std::mutex g_scratch_mu;
int64_t* g_scratch_dev[kMaxDevices] = {nullptr};

// This device's address of g_argmax_scratch, looked up on the device's first call (with the
// device current) and kept for the life of the process. A cudaDeviceReset unloads the module and
// invalidates the kept address: this entry point must not be called on a device after a reset.
int64_t* scratch_address(int dev) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_dev[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_argmax_scratch) != cudaSuccess || p == nullptr) return nullptr;
    g_scratch_dev[dev] = static_cast<int64_t*>(p);
  }
  return g_scratch_dev[dev];
}

}  // namespace

int argmax_noalloc_launch(const float* x, int64_t n, int64_t stride, int64_t* index,
                          cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kErrCuda;
  int64_t* scratch = scratch_address(dev);
  if (scratch == nullptr) return kErrCuda;
  return argmax_launch(x, n, stride, scratch, index, stream);
}

}  // namespace otq
