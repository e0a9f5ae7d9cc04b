// Device and host helpers of the tcgen05 tensor-core kernels (prefill.cu, w8a8.cu): 2-D tensor
// copies into shared memory, the shared-memory matrix descriptor of the 128-byte swizzle
// layout, MMA commits, the tensor-memory fences, and tensor-map encoding through the driver
// entry point.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>

namespace otq {

// A 2-D box of `map` at (x, y) into shared dst, completing its bytes on mbarrier bar. The
// box's bytes are always written (elements outside the tensor as zeros).
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// UMMA shared-memory descriptor of a K-major tile in the 128-byte swizzle layout: rows 128 bytes
// apart, 8-row groups 1024 bytes apart (leading offset 16 bytes, unused by this layout; stride
// offset 1024 bytes; version 1; layout type 2 = 128-byte swizzle). A K step of 32 bytes (16
// bf16, 32 int8) advances the start address by 32 bytes inside the swizzle atom.
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1u) << 16) |
         (static_cast<uint64_t>(1024u >> 4) << 32) | (static_cast<uint64_t>(1u) << 46) |
         (static_cast<uint64_t>(2u) << 61);
}

// The barrier's next phase completes when every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

inline EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// A row-major [outer][inner] tensor (stride_bytes between rows) with a box_inner x box_outer box.
inline bool encode_2d(EncodeFn enc, CUtensorMap* map, CUtensorMapDataType type, const void* base,
                      int64_t inner, int64_t outer, int64_t stride_bytes, CUtensorMapSwizzle swizzle,
                      int box_inner, int box_outer) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace otq
