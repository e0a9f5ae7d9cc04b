// Row quantization kernels: QACT / QST bytes into plain arrays (otq_quantize_rows) and the
// int8 weight formats MM streams (otq_pack_int8: int8x rows + scale rows, or RSC).
// One CTA quantizes one row with the shared routine of qact.cuh.
#include <cuda_runtime.h>

#include <cstdint>

#include "otq_fp32.cuh"
#include "otq_internal.h"
#include "qact.cuh"

namespace otq {
namespace {

constexpr int kThreads = 256;

struct QuantParams {
  const float* x;
  int64_t rows;
  int n;
  int64_t ldx;
  int group;
  int row_mode;
  // plain outputs
  int8_t* q;
  int64_t ldq;
  float* S;
  uint8_t* d;
  int64_t ldd;
  // packed outputs (pack != 0): q into rows, Sw and offsets into scale rows
  int pack;
  int rsc;
  uint8_t* prow;
  int64_t rs;
  uint8_t* srow;
  int64_t srs;
};

__global__ void __launch_bounds__(kThreads) quantize_rows_kernel(const QuantParams p) {
  extern __shared__ __align__(16) uint32_t qsm[];
  float* xs = reinterpret_cast<float*>(qsm);
  uint32_t* seg = qsm + p.n;
  uint32_t* red = seg + (p.n >> 5);
  const int64_t row = blockIdx.x;
  const ThreadGroup<kThreads> grp{static_cast<int>(threadIdx.x)};
  stage_row(grp, p.x + row * p.ldx, xs, p.n);
  const float* x = xs;
  const int g = p.group;
  if (!p.pack) {
    int8_t* q = p.q + row * p.ldq;
    uint8_t* d = p.d ? p.d + row * p.ldd : nullptr;
    QactRowResult r = qact_row(grp, x, p.n, g, p.row_mode != 0, seg, red,
                                         [&](int i, int qv, int dg) {
                                           q[i] = static_cast<int8_t>(qv);
                                           if (d != nullptr && (i % g) == 0) d[i / g] =
                                               static_cast<uint8_t>(dg);
                                         });
    if (threadIdx.x == 0) p.S[row] = r.S;
  } else {
    uint8_t* q = p.prow + row * p.rs;
    uint8_t* s = p.srow + row * p.srs;
    const int nb = p.n / g;
    QactRowResult r = qact_row(grp, x, p.n, g, p.row_mode != 0, seg, red,
                                         [&](int i, int qv, int dg) {
                                           q[i] = static_cast<uint8_t>(static_cast<int8_t>(qv));
                                           if (!p.rsc && (i % g) == 0) s[4 + i / g] =
                                               static_cast<uint8_t>(dg);
                                         });
    if (threadIdx.x == 0) *reinterpret_cast<float*>(s) = r.S;
    // the scale row's padding bytes are written as zeros (quant.py pack_scales)
    const int used = p.rsc ? 4 : 4 + nb;
    for (int64_t b = used + threadIdx.x; b < p.srs; b += kThreads) s[b] = 0;
    for (int64_t b = p.n + threadIdx.x; b < p.rs; b += kThreads) q[b] = 0;
  }
}

}  // namespace

int quantize_rows_launch(const float* x, int64_t rows, int n, int64_t ldx, int group,
                         int row_mode, int8_t* q, int64_t ldq, float* S, uint8_t* d, int64_t ldd,
                         int pack, int rsc, uint8_t* prow, int64_t rs, uint8_t* srow, int64_t srs,
                         cudaStream_t stream) {
  if (rows == 0) return kOk;
  QuantParams p{x, rows, n, ldx, group, row_mode, q, ldq, S, d, ldd, pack, rsc, prow, rs, srow,
                srs};
  const size_t smem = static_cast<size_t>(n + n / 32 + 40) * 4;
  if (rows > 0x7FFFFFFF || smem > 227 * 1024) return kErrArg;
  static size_t configured[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return kErrCuda;
  if (smem > 48 * 1024 && configured[dev] < smem) {
    if (cudaFuncSetAttribute(quantize_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = smem;
  }
  return launch_kernel(reinterpret_cast<const void*>(quantize_rows_kernel),
                       static_cast<int>(rows), kThreads, smem, stream, false, p);
}

}  // namespace otq
