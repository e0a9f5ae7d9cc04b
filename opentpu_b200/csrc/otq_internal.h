// Internal declarations shared by the CUDA translation units of libotq.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/otq.h"

namespace otq {

constexpr int kOk = OTQ_OK;
constexpr int kErrArg = OTQ_ERR_ARG;
constexpr int kErrAlign = OTQ_ERR_ALIGN;
constexpr int kErrFormat = OTQ_ERR_FORMAT;
constexpr int kErrCuda = OTQ_ERR_CUDA;
constexpr int kErrDevice = OTQ_ERR_DEVICE;

constexpr int kFmtInt8 = OTQ_FMT_INT8;
constexpr int kFmtInt4 = OTQ_FMT_INT4;
constexpr int kFmtFp4 = OTQ_FMT_FP4;
constexpr int kFmtNvfp4 = OTQ_FMT_NVFP4;

constexpr int kMmUnit = OTQ_MM_UNIT;
constexpr int kMmAcc = OTQ_MM_ACC;
constexpr int kMmAscale = OTQ_MM_ASCALE;
constexpr int kMmRsc = OTQ_MM_RSC;

constexpr int kMaxDevices = 64;

// Bits of the library's device status word (otq_status_word): a bounded wait ran out.
constexpr int kStatusTimeout = 1;

struct MMParams {
  int fmt;
  int flags;
  const uint8_t* rows;
  int64_t rs;
  const uint8_t* srows;
  int64_t srs;
  int k0;
  int64_t N;
  int K;
  // activations: x (fp32, quantized by the kernel's QACT prologue) or q / Sa / da
  const float* x;
  int64_t ldx;
  int row_mode;
  const int8_t* q;
  int64_t ldq;
  const float* Sa;
  const uint8_t* da;
  int64_t ldd;
  int M;
  const float* alpha;
  float* y;
  int64_t ldy;
  int split;    // otq_qmm_ex's k_split (0 picks)
  int* status;   // device status word (may be null): kStatusTimeout bits
  const otq_peer* peer;   // otq_qmm_peer's output fan-out over NVLink, or null
};

// One projection of the prefill GEMM (prefill.cu), checked by the caller: x bf16 [M, K] (ldx
// elements, 16-byte aligned rows), rows int8 [N, K] (rs bytes), Sw the first fp32 word of each
// scale row (srs bytes; srows unused with OTQ_MM_UNIT), y fp32 [M, N] (ldy floats).
struct W8A16Proj {
  int flags;
  const uint8_t* rows;
  int64_t rs;
  const uint8_t* srows;
  int64_t srs;
  int64_t N, K;
  const uint16_t* x;
  int64_t ldx, M;
  float* y;
  int64_t ldy;
};
constexpr int kW8A16MaxGroup = 8;

// One projection of the exact W8A8 tensor-core MM (w8a8.cu), checked by the caller: rows int8
// [N, K] (rs bytes, 16-byte aligned), Sw the first fp32 word of each scale row (srows unused
// with OTQ_MM_UNIT), planes the buffer qact_planes_launch wrote for M rows of K, y fp32 [M, N]
// (ldy floats).
struct W8A8Proj {
  int flags;
  const uint8_t* rows;
  int64_t rs;
  const uint8_t* srows;
  int64_t srs;
  int64_t N, K;
  const void* planes;
  int64_t M;
  float* y;
  int64_t ldy;
};
constexpr int kW8A8MaxGroup = 8;

int sm_count(int dev);
// argmax.cu: acc = two words (key accumulator, CTA count) zeroed on the stream here; the index
// goes to *index (acc itself for otq_argmax)
int argmax_launch(const float* x, int64_t n, int64_t stride, int64_t* acc, int64_t* index,
                  cudaStream_t stream);
// the same with the scratch words in argmax.cu's own device array (otq_argmax_noalloc)
int argmax_noalloc_launch(const float* x, int64_t n, int64_t stride, int64_t* index,
                          cudaStream_t stream);
int w8a16_launch(const W8A16Proj* projs, int count, cudaStream_t stream);   // prefill.cu
// w8a8.cu: the planes buffer (bytes for M rows of K; QACT into it) and the tensor-core MM
int64_t qact_planes_bytes(int64_t M, int64_t K);
int qact_planes_launch(const float* x, int64_t ldx, int64_t M, int64_t K, int row_mode,
                       void* planes, cudaStream_t stream);
int w8a8_launch(const W8A8Proj* projs, int count, cudaStream_t stream);
int mm_launch(const MMParams& p, cudaStream_t stream, bool pdl);    // gemv.cu
int chain_launch(const otq_proj* projs, int count, cudaStream_t stream);
int chain_reset();   // the grid barrier's count back to zero
int set_tag_wait_limit(uint32_t polls);   // gemv.cu: otq_set_wait_limit
int set_step_wait_limit(uint32_t polls);  // step.cu: otq_set_wait_limit
// step.cu: the persistent decode step
int step_layout(const otq_step_proj* projs, int count, int world, int64_t* offsets, int64_t* total);
int64_t step_table_bytes();
int step_prepare(const otq_step* step, void* table);
int step_launch(const otq_step* step, const void* table, cudaStream_t stream);
int* status_word();   // this device's status word (device address), or null

// Launch with an optional programmatic-dependent-launch attribute (the kernel then may start
// while the previous kernel in the stream finishes; it waits with griddepcontrol.wait before
// reading anything that kernel wrote).
template <class P>
int launch_kernel(const void* fn, int grid, int block, size_t smem, cudaStream_t stream, bool pdl,
                  const P& params) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(block, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* args[] = {const_cast<P*>(&params)};
  const cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
  return e == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace otq
