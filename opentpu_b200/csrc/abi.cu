// The extern "C" entry points of libotq (declared in include/otq.h): host-side validation of
// every shape, stride, alignment and flag, then the launch. No exception crosses the ABI and
// nothing is allocated.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <cstring>

#include "otq_internal.h"

namespace otq {

int quantize_rows_launch(const float* x, int64_t rows, int n, int64_t ldx, int group,
                         int row_mode, int8_t* q, int64_t ldq, float* S, uint8_t* d, int64_t ldd,
                         int pack, int rsc, uint8_t* prow, int64_t rs, uint8_t* srow, int64_t srs,
                         cudaStream_t stream);
int pack_mx4_launch(int fmt, const float* W, int64_t N, int K, int64_t ldw, uint8_t* rows,
                    int64_t rs, uint8_t* srows, int64_t srs, cudaStream_t stream);
int pack_g32_launch(const float* W, int64_t N, int64_t K, int64_t ldw, uint8_t* codes,
                    uint16_t* scales, cudaStream_t stream);
int linear_g32_launch(const uint8_t* codes, const uint16_t* scales, int64_t N, int K,
                      const float* x, int64_t ldx, int M, int accumulate, float* y, int64_t ldy,
                      cudaStream_t stream);

// The library's device status word (one per device that loads the library): kernels record
// a bounded wait that ran out here; otq_status_word reads and clears it.
__device__ int g_status_word = 0;

namespace {

thread_local char g_last_cuda[256] = "";

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return kOk;
  std::strncpy(g_last_cuda, cudaGetErrorString(e), sizeof(g_last_cuda) - 1);
  return kErrCuda;
}

int finish(int st) {
  if (st == kErrCuda) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) cuda_status(e);
  }
  return st;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int device_ok() {
  static int checked[kMaxDevices] = {0};   // 0 unknown, 1 ok, -1 refused
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return kErrDevice;
  if (checked[dev] == 0) {
    int major = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_status(e);
    checked[dev] = major == 10 ? 1 : -1;
  }
  return checked[dev] == 1 ? kOk : kErrDevice;
}

int fmt_window(int fmt) {
  switch (fmt) {
    case kFmtInt8: return 16;
    case kFmtInt4:
    case kFmtFp4: return 11;
    case kFmtNvfp4: return 13;
    default: return -1;
  }
}

// Scale-row alignment MM requires (docs/isa.md "MM": ssa/srs multiples of 4, 8 or 16).
int64_t scale_align(int fmt, bool rsc) {
  if (rsc || fmt == kFmtInt8) return 4;
  return fmt == kFmtNvfp4 ? 16 : 8;
}

// Bytes of scale row that MM reads for blocks [k0, k0 + KB).
int64_t scale_need(int fmt, bool rsc, int k0, int64_t KB) {
  if (rsc) return 4;
  switch (fmt) {
    case kFmtInt8: return 4 + k0 + KB;
    case kFmtInt4:
    case kFmtFp4: return 8 + 4 * (k0 + KB);
    default: return 16 + 8 * (k0 + KB);
  }
}

constexpr int64_t kStrideLimit = int64_t(1) << 31;   // strides are 32-bit in the kernels

int check_weights(int fmt, int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
                  int64_t srs, int k0, int64_t N, int64_t K) {
  if (fmt_window(fmt) < 0) return kErrFormat;
  if (flags & ~(kMmUnit | kMmAcc | kMmAscale | kMmRsc)) return kErrArg;
  const bool unit = flags & kMmUnit, rsc = flags & kMmRsc;
  if (rsc && fmt == kFmtNvfp4) return kErrFormat;            // isa.py:527
  if ((flags & kMmAscale) && !(unit && (flags & kMmAcc))) {  // isa.py ASCALE needs UNIT and ACC
    return kErrArg;
  }
  if (N <= 0 || K <= 0 || K % OTQ_D != 0 || K > 255 * OTQ_D) return kErrArg;
  if (k0 < 0 || k0 > 255) return kErrArg;
  if (rows == nullptr) return kErrArg;
  const int64_t used = fmt == kFmtInt8 ? K : K / 2;
  if (rs < used) return kErrArg;
  if (!aligned(rows, 16) || rs % 16) return kErrAlign;
  if (rs >= kStrideLimit || srs >= kStrideLimit) return kErrArg;
  if (!unit) {
    if (srows == nullptr) return kErrArg;
    const int64_t a = scale_align(fmt, rsc);
    if (!aligned(srows, a) || srs % a) return kErrAlign;
    if (srs < scale_need(fmt, rsc, k0, K / OTQ_D)) return kErrArg;
  }
  return kOk;
}


int check_out(int64_t M, int64_t N, const float* y, int64_t ldy, int flags, const float* alpha) {
  if (M <= 0 || M > 0x7FFFFFFF || y == nullptr || ldy < N || ldy >= kStrideLimit) return kErrArg;
  if ((flags & kMmAscale) && alpha == nullptr) return kErrArg;
  return kOk;
}

}  // namespace

// The address is looked up once per device (under a lock: two host threads may make their first
// calls together) and kept; a cudaDeviceReset invalidates it.
int* status_word() {
  static int* addr[kMaxDevices] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<int*>(p);
  }
  return addr[dev];
}

int sm_count(int dev) {
  static int cache[kMaxDevices] = {0};
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace otq

using namespace otq;

extern "C" {

const char* otq_version(void) { return "libotq 0.1 (sm_100a)"; }

const char* otq_status_string(int status) {
  switch (status) {
    case OTQ_OK: return "ok";
    case OTQ_ERR_ARG: return "invalid argument (size, stride, flag or null pointer)";
    case OTQ_ERR_ALIGN: return "misaligned pointer or stride";
    case OTQ_ERR_FORMAT: return "unknown weight format or unsupported format/flag combination";
    case OTQ_ERR_CUDA: return "CUDA error";
    case OTQ_ERR_DEVICE: return "the current device is not compute capability 10.x";
    default: return "unknown status";
  }
}

const char* otq_last_cuda_error(void) { return g_last_cuda; }

int otq_device_check(void) { return device_ok(); }

int otq_quantize_rows(const float* x, int64_t rows, int64_t n, int64_t ldx, int group,
                      int row_mode, int8_t* q, int64_t ldq, float* S, uint8_t* d, int64_t ldd,
                      void* stream) {
  int st = device_ok();
  if (st) return st;
  if (rows < 0 || n <= 0 || n > 32768 || group <= 0 || group % 32 || n % group) return kErrArg;
  if (x == nullptr || q == nullptr || S == nullptr || ldx < n || ldq < n) return kErrArg;
  if (!row_mode && (d == nullptr || ldd < n / group)) return kErrArg;
  if (!aligned(x, 4)) return kErrAlign;
  return finish(quantize_rows_launch(x, rows, static_cast<int>(n), ldx, group, row_mode, q, ldq, S,
                                     d, ldd, 0, 0, nullptr, 0, nullptr, 0,
                                     static_cast<cudaStream_t>(stream)));
}

int otq_pack_int8(const float* W, int64_t N, int64_t K, int64_t ldw, int rsc, uint8_t* rows,
                  int64_t rs, uint8_t* srows, int64_t srs, void* stream) {
  int st = device_ok();
  if (st) return st;
  if (N < 0 || K <= 0 || K % OTQ_D || K > 32768 || ldw < K) return kErrArg;
  if (W == nullptr || rows == nullptr || srows == nullptr || rs < K) return kErrArg;
  const int64_t need = rsc ? 4 : 4 + 4 * ((K / OTQ_D + 3) / 4);
  if (srs < need) return kErrArg;
  if (!aligned(srows, 4) || srs % 4) return kErrAlign;
  return finish(quantize_rows_launch(W, N, static_cast<int>(K), ldw, OTQ_D, rsc ? 1 : 0, nullptr,
                                     0, nullptr, nullptr, 0, 1, rsc ? 1 : 0, rows, rs, srows, srs,
                                     static_cast<cudaStream_t>(stream)));
}

int otq_quantize_mxu(int fmt, const float* W, int64_t N, int64_t K, int64_t ldw, uint8_t* rows,
                     int64_t rs, uint8_t* srows, int64_t srs, void* stream) {
  int st = device_ok();
  if (st) return st;
  if (fmt_window(fmt) < 0) return kErrFormat;
  if (N < 0 || K <= 0 || K % OTQ_D || K > 32768 || ldw < K) return kErrArg;
  if (W == nullptr || rows == nullptr || srows == nullptr) return kErrArg;
  const int64_t KB = K / OTQ_D;
  const int64_t need_rs = fmt == kFmtInt8 ? K : 128 * ((K + 255) / 256);
  const int64_t need_srs = fmt == kFmtInt8 ? 4 + 4 * ((KB + 3) / 4)
                           : fmt == kFmtNvfp4 ? 16 + 16 * ((KB + 1) / 2)
                                              : 8 + 8 * ((KB + 1) / 2);
  if (rs < need_rs || srs < need_srs) return kErrArg;
  if (!aligned(srows, scale_align(fmt, false)) || srs % scale_align(fmt, false)) return kErrAlign;
  if (!aligned(W, 4)) return kErrAlign;
  if (fmt == kFmtInt8)
    return finish(quantize_rows_launch(W, N, static_cast<int>(K), ldw, OTQ_D, 0, nullptr, 0,
                                       nullptr, nullptr, 0, 1, 0, rows, rs, srows, srs,
                                       static_cast<cudaStream_t>(stream)));
  return finish(pack_mx4_launch(fmt, W, N, static_cast<int>(K), ldw, rows, rs, srows, srs,
                                static_cast<cudaStream_t>(stream)));
}

int otq_mm(int fmt, int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows, int64_t srs,
           int k0, int64_t N, int64_t K, const int8_t* q, int64_t ldq, const float* Sa,
           const uint8_t* da, int64_t ldd, int64_t M, const float* alpha, float* y, int64_t ldy,
           void* stream) {
  int st = device_ok();
  if (st) return st;
  if ((st = check_weights(fmt, flags, rows, rs, srows, srs, k0, N, K))) return st;
  if ((st = check_out(M, N, y, ldy, flags, alpha))) return st;
  if (q == nullptr || Sa == nullptr || da == nullptr || ldq < K || ldd < K / 32 ||
      ldq >= kStrideLimit || ldd >= kStrideLimit)
    return kErrArg;
  MMParams p{};
  p.fmt = fmt;
  p.flags = flags;
  p.rows = rows;
  p.rs = rs;
  p.srows = srows;
  p.srs = srs;
  p.k0 = k0;
  p.N = N;
  p.K = static_cast<int>(K);
  p.q = q;
  p.ldq = ldq;
  p.Sa = Sa;
  p.da = da;
  p.ldd = ldd;
  p.M = static_cast<int>(M);
  p.alpha = alpha;
  p.y = y;
  p.ldy = ldy;
  return finish(mm_launch(p, static_cast<cudaStream_t>(stream), false));
}

int otq_qmm_ex(int fmt, int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
               int64_t srs, int k0, int64_t N, int64_t K, const float* x, int64_t ldx,
               int row_mode, int64_t M, const float* alpha, float* y, int64_t ldy,
               int k_split, int pdl, void* stream) {
  int st = device_ok();
  if (st) return st;
  if ((st = check_weights(fmt, flags, rows, rs, srows, srs, k0, N, K))) return st;
  if ((st = check_out(M, N, y, ldy, flags, alpha))) return st;
  if (x == nullptr || ldx < K || ldx >= kStrideLimit) return kErrArg;
  if (!aligned(x, 4)) return kErrAlign;
  if (k_split != 0 && k_split != 1 && k_split != 2 && k_split != 4 && k_split != 8 && k_split != 32)
    return kErrArg;
  MMParams p{};
  p.fmt = fmt;
  p.flags = flags;
  p.rows = rows;
  p.rs = rs;
  p.srows = srows;
  p.srs = srs;
  p.k0 = k0;
  p.N = N;
  p.K = static_cast<int>(K);
  p.x = x;
  p.ldx = ldx;
  p.row_mode = row_mode ? 1 : 0;
  p.M = static_cast<int>(M);
  p.alpha = alpha;
  p.y = y;
  p.ldy = ldy;
  p.split = k_split;
  return finish(mm_launch(p, static_cast<cudaStream_t>(stream), pdl != 0));
}

int otq_qmm_peer(int fmt, int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
                 int64_t srs, int k0, int64_t N, int64_t K, const float* x, int64_t ldx,
                 int row_mode, float* y, const otq_peer* peer, int pdl, void* stream) {
  int st = device_ok();
  if (st) return st;
  if ((st = check_weights(fmt, flags, rows, rs, srows, srs, k0, N, K))) return st;
  if ((st = check_out(1, N, y, N, flags, nullptr))) return st;
  if (flags & (kMmAscale | kMmAcc)) return kErrArg;
  if (x == nullptr || ldx < K || ldx >= kStrideLimit) return kErrArg;
  if (peer == nullptr || peer->world < 1 || peer->world > 8 || peer->rank < 0 ||
      peer->rank >= peer->world || peer->seq == nullptr || peer->done == nullptr)
    return kErrArg;
  if (peer->tags != OTQ_TAGS_COUNTED && peer->tags != OTQ_TAGS_STEPPED) return kErrArg;
  if (peer->tags == OTQ_TAGS_STEPPED && (peer->step_pos < 0 || peer->step_pos >= 1023))
    return kErrArg;
  if (!aligned(y, 16) || !aligned(x, peer->wait ? 16 : 4)) return kErrAlign;
  if (!aligned(peer->seq, 4) || !aligned(peer->done, 4)) return kErrAlign;
  for (int r = 0; r < peer->world; ++r)
    if (peer->delta[r] % 16) return kErrAlign;
  MMParams p{};
  p.fmt = fmt;
  p.flags = flags;
  p.rows = rows;
  p.rs = rs;
  p.srows = srows;
  p.srs = srs;
  p.k0 = k0;
  p.N = N;
  p.K = static_cast<int>(K);
  p.x = x;
  p.ldx = ldx;
  p.row_mode = row_mode ? 1 : 0;
  p.M = 1;
  p.y = y;
  p.ldy = N;
  p.peer = peer;
  return finish(mm_launch(p, static_cast<cudaStream_t>(stream), pdl != 0));
}

int otq_qmm(int fmt, int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
            int64_t srs, int k0, int64_t N, int64_t K, const float* x, int64_t ldx, int row_mode,
            int64_t M, const float* alpha, float* y, int64_t ldy, void* stream) {
  return otq_qmm_ex(fmt, flags, rows, rs, srows, srs, k0, N, K, x, ldx, row_mode, M, alpha, y,
                    ldy, 0, 0, stream);
}

int otq_qmm_chain(const otq_proj* projs, int count, void* stream) {
  int st = device_ok();
  if (st) return st;
  if (projs == nullptr || count < 0) return kErrArg;
  for (int i = 0; i < count; ++i) {
    const otq_proj& p = projs[i];
    if ((st = check_weights(p.fmt, p.flags, p.rows, p.rs, p.srows, p.srs, p.k0, p.N, p.K))) return st;
    if (p.flags & kMmAscale) return kErrArg;
    if (p.x == nullptr || p.y == nullptr) return kErrArg;
    if (!aligned(p.x, 4) || !aligned(p.y, 4)) return kErrAlign;
  }
  if (count == 0) return kOk;
  return finish(chain_launch(projs, count, static_cast<cudaStream_t>(stream)));
}

int otq_gemm_w8a16_group(const otq_gemm_proj* projs, int count, void* stream) {
  int st = device_ok();
  if (st) return st;
  if (projs == nullptr || count < 0 || count > kW8A16MaxGroup) return kErrArg;
  W8A16Proj w[kW8A16MaxGroup];
  for (int i = 0; i < count; ++i) {
    const otq_gemm_proj& p = projs[i];
    if (p.flags & ~(kMmUnit | kMmRsc | kMmAcc)) return kErrArg;
    if (!(p.flags & (kMmUnit | kMmRsc))) return kErrFormat;   // int8x block offsets: otq_qmm
    if (p.N <= 0 || p.K <= 0 || p.M <= 0 || p.K % 8 || p.K > 0x7FFFFFFF || p.N > 0x7FFFFFFF ||
        p.M > 0x7FFFFFFF)
      return kErrArg;
    if (p.rows == nullptr || p.x == nullptr || p.y == nullptr) return kErrArg;
    if (!(p.flags & kMmUnit) && p.srows == nullptr) return kErrArg;
    if (p.rs < p.K || p.ldx < p.K || p.ldy < p.N || p.rs >= kStrideLimit ||
        p.ldx >= kStrideLimit || p.ldy >= kStrideLimit)
      return kErrArg;
    if (!aligned(p.rows, 16) || p.rs % 16 || !aligned(p.x, 16) || p.ldx % 8 || !aligned(p.y, 4))
      return kErrAlign;
    if (!(p.flags & kMmUnit) && (!aligned(p.srows, 4) || p.srs % 4 || p.srs < 4)) return kErrAlign;
    w[i] = W8A16Proj{p.flags, p.rows, p.rs, p.srows, p.srs, p.N, p.K, p.x, p.ldx, p.M, p.y, p.ldy};
  }
  if (count == 0) return kOk;
  return finish(w8a16_launch(w, count, static_cast<cudaStream_t>(stream)));
}

int otq_gemm_w8a16(int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
                   int64_t srs, int64_t N, int64_t K, const uint16_t* x, int64_t ldx, int64_t M,
                   float* y, int64_t ldy, void* stream) {
  const otq_gemm_proj p{flags, rows, rs, srows, srs, N, K, x, ldx, M, y, ldy};
  return otq_gemm_w8a16_group(&p, 1, stream);
}

int64_t otq_qact_planes_bytes(int64_t M, int64_t K) {
  if (M < 0 || K <= 0 || K % 32 || K > 65536 || M > (int64_t{1} << 30)) return kErrArg;
  return qact_planes_bytes(M, K);
}

int otq_qact_planes(const float* x, int64_t ldx, int64_t M, int64_t K, int row_mode,
                    void* planes, int64_t bytes, void* stream) {
  int st = device_ok();
  if (st) return st;
  const int64_t need = otq_qact_planes_bytes(M, K);
  if (need < 0) return static_cast<int>(need);
  if (x == nullptr || planes == nullptr || ldx < K || ldx >= kStrideLimit || bytes < need ||
      (row_mode != 0 && row_mode != 1))
    return kErrArg;
  if (!aligned(x, 4) || !aligned(planes, 16)) return kErrAlign;
  return finish(qact_planes_launch(x, ldx, M, K, row_mode, planes, static_cast<cudaStream_t>(stream)));
}

int otq_gemm_w8a8_group(const otq_gemm8_proj* projs, int count, void* stream) {
  int st = device_ok();
  if (st) return st;
  if (projs == nullptr || count < 0 || count > kW8A8MaxGroup) return kErrArg;
  W8A8Proj w[kW8A8MaxGroup];
  int n = 0;
  for (int i = 0; i < count; ++i) {
    const otq_gemm8_proj& p = projs[i];
    if (p.flags & ~(kMmUnit | kMmRsc | kMmAcc)) return kErrArg;
    if (!(p.flags & (kMmUnit | kMmRsc))) return kErrFormat;   // int8x block offsets: otq_qmm
    if (p.N <= 0 || p.M < 0 || p.M > 32768 || p.N > 0x7FFFFFFF || otq_qact_planes_bytes(p.M, p.K) < 0)
      return kErrArg;
    if (p.rows == nullptr || p.planes == nullptr || p.y == nullptr) return kErrArg;
    if (!(p.flags & kMmUnit) && p.srows == nullptr) return kErrArg;
    if (p.rs < p.K || p.ldy < p.N || p.rs >= kStrideLimit || p.ldy >= kStrideLimit) return kErrArg;
    if (!aligned(p.rows, 16) || p.rs % 16 || !aligned(p.planes, 16) || !aligned(p.y, 4))
      return kErrAlign;
    if (!(p.flags & kMmUnit) && (!aligned(p.srows, 4) || p.srs % 4 || p.srs < 4)) return kErrAlign;
    if (p.M == 0) continue;
    w[n++] = W8A8Proj{p.flags, p.rows, p.rs, p.srows, p.srs, p.N, p.K, p.planes, p.M, p.y, p.ldy};
  }
  if (n == 0) return kOk;
  return finish(w8a8_launch(w, n, static_cast<cudaStream_t>(stream)));
}

int otq_qmm_tc(int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows, int64_t srs,
               int64_t N, int64_t K, const float* x, int64_t ldx, int row_mode, int64_t M,
               void* planes, int64_t planes_bytes, float* y, int64_t ldy, void* stream) {
  const otq_gemm8_proj p{flags, rows, rs, srows, srs, N, K, planes, M, y, ldy};
  // the projection's checks first: nothing is launched for a call that would fail
  if (flags & ~(kMmUnit | kMmRsc | kMmAcc)) return kErrArg;
  if (!(flags & (kMmUnit | kMmRsc))) return kErrFormat;
  if (rows == nullptr || y == nullptr || N <= 0 || M > 32768 || rs < K || ldy < N) return kErrArg;
  int st = otq_qact_planes(x, ldx, M, K, row_mode, planes, planes_bytes, stream);
  if (st) return st;
  return otq_gemm_w8a8_group(&p, 1, stream);
}

int otq_argmax(const float* x, int64_t n, int64_t stride, int64_t* out, void* stream) {
  int st = device_ok();
  if (st) return st;
  if (x == nullptr || out == nullptr || n < 1 || n >= (int64_t{1} << 32) || stride < 1 ||
      stride > (int64_t{1} << 20))
    return kErrArg;
  if (!aligned(x, 4) || !aligned(out, 16)) return kErrAlign;
  return finish(argmax_launch(x, n, stride, out, out, static_cast<cudaStream_t>(stream)));
}

int otq_argmax_noalloc(const float* x, int64_t n, int64_t stride, int64_t* index, void* stream) {
  int st = device_ok();
  if (st) return st;
  if (x == nullptr || index == nullptr || n < 1 || n >= (int64_t{1} << 32) || stride < 1 ||
      stride > (int64_t{1} << 20))
    return kErrArg;   // n past 2^32 - 1: the row's index no longer fits the scratch key
  if (!aligned(x, 4) || !aligned(index, 8)) return kErrAlign;
  return finish(argmax_noalloc_launch(x, n, stride, index, static_cast<cudaStream_t>(stream)));
}

int otq_status_word(int* value, int reset) {
  int st = device_ok();
  if (st) return st;
  if (value == nullptr) return kErrArg;
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_status_word, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e);
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_status_word, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e);
    if (v != 0 && (st = chain_reset())) return st;   // a barrier may have been left mid-way
  }
  *value = v;
  return kOk;
}

int otq_set_wait_limit(uint32_t polls) {
  int st = device_ok();
  if (st) return st;
  if ((st = set_tag_wait_limit(polls))) return finish(st);
  return finish(set_step_wait_limit(polls));
}

int otq_step_layout(const otq_step_proj* projs, int count, int world, int64_t* offsets,
                    int64_t* total_words) {
  if (projs == nullptr || total_words == nullptr || count < 1 || count > OTQ_STEP_MAX ||
      world < 1 || world > 8)
    return kErrArg;
  for (int i = 0; i < count; ++i)
    if (projs[i].N <= 0) return kErrArg;
  return step_layout(projs, count, world, offsets, total_words);
}

namespace {
int check_step(const otq_step* s) {
  if (s == nullptr || s->projs == nullptr || s->count < 1 || s->count > OTQ_STEP_MAX) return kErrArg;
  if (s->world < 1 || s->world > 8 || s->rank < 0 || s->rank >= s->world) return kErrArg;
  if (s->out == nullptr || s->counters == nullptr) return kErrArg;
  if (!aligned(s->out, 16) || !aligned(s->counters, 16)) return kErrAlign;
  for (int r = 0; r < s->world; ++r)
    if (s->delta[r] % 16 || (r == s->rank && s->delta[r] != 0)) return kErrAlign;
  if (s->token != nullptr && !aligned(s->token, 8)) return kErrAlign;
  if (s->embed != nullptr && (s->token_in == nullptr || s->vocab <= 0 || !aligned(s->embed, 16)))
    return kErrArg;
  bool plain_in = false, attn = false;
  auto full = [&](int i) {   // a projection's output row
    const otq_step_proj& q = s->projs[i];
    return (q.epilogue == OTQ_EPI_SWIGLU ? q.N / 2 : q.N) * (q.replicated ? 1 : s->world);
  };
  auto is_proj = [&](int j, int i) {
    return j >= 0 && j < i && s->projs[j].fmt != OTQ_STEP_ATTN;
  };
  for (int i = 0; i < s->count; ++i) {
    const otq_step_proj& p = s->projs[i];
    if (p.fmt == OTQ_STEP_ATTN) {
      attn = true;
      if (!is_proj(p.in, i) || p.head_dim != 128 || p.n_kv <= 0 || p.n_q <= 0 || p.n_q % p.n_kv ||
          p.n_q / p.n_kv > 4 || p.kcache == nullptr || p.vcache == nullptr)
        return kErrArg;
      if (full(p.in) < static_cast<int64_t>(p.n_q + 2 * p.n_kv) * 128) return kErrArg;
      // the combined row and the partial results
      if (p.N < static_cast<int64_t>(p.n_q) * 128 + static_cast<int64_t>(p.n_q) * ((s->max_pos + 31) / 32) * 130)
        return kErrArg;
      if (!aligned(p.kcache, 16) || !aligned(p.vcache, 16)) return kErrAlign;
      if ((p.q_gain && !aligned(p.q_gain, 16)) || (p.k_gain && !aligned(p.k_gain, 16))) return kErrAlign;
      continue;
    }
    const bool g32 = p.fmt == OTQ_STEP_G32;
    if (p.fmt != OTQ_STEP_RSC && !g32) return kErrFormat;
    if (p.replicated != 0 && p.replicated != 1) return kErrArg;
    if (p.epilogue != OTQ_EPI_NONE &&
        (p.epilogue != OTQ_EPI_SWIGLU || p.N % 16 || i == s->count - 1))
      return kErrArg;
    if (p.N <= 0 || p.K <= 0 || p.K % (g32 ? 256 : OTQ_D) || p.K > 255 * OTQ_D) return kErrArg;
    if (p.N * s->world >= (int64_t{1} << 30)) return kErrArg;
    if (p.rows == nullptr || p.rs < (g32 ? p.K / 2 : p.K) || p.rs >= kStrideLimit) return kErrArg;
    if (!aligned(p.rows, 16) || p.rs % 16) return kErrAlign;
    if (g32) {
      if (p.srows == nullptr || p.srs < p.K / 16 || p.srs >= kStrideLimit) return kErrArg;
      if (!aligned(p.srows, 16) || p.srs % 16) return kErrAlign;
    } else if (p.srows != nullptr && (!aligned(p.srows, 4) || p.srs % 4 || p.srs < 4 ||
                                      p.srs >= kStrideLimit)) {
      return kErrAlign;
    }
    switch (p.input) {
      case OTQ_IN_DEFAULT:
        if (p.in == -1) plain_in = true;
        else if (!is_proj(p.in, i) || full(p.in) < p.K) return kErrArg;
        break;
      case OTQ_IN_NORM:
        if (p.gamma == nullptr) return kErrArg;
        if (!aligned(p.gamma, 16)) return kErrAlign;
        if (p.res == -2) plain_in = plain_in || s->embed == nullptr;
        else if (!is_proj(p.res, i) || full(p.res) < p.K) return kErrArg;
        break;
      case OTQ_IN_SWIGLU:
        if (!is_proj(p.in, i) || full(p.in) < 2 * p.K) return kErrArg;
        break;
      case OTQ_IN_ATTN:
        if (p.in < 0 || p.in >= i || s->projs[p.in].fmt != OTQ_STEP_ATTN ||
            p.K != static_cast<int64_t>(s->projs[p.in].n_q) * 128)
          return kErrArg;
        break;
      default:
        return kErrArg;
    }
  }
  if (plain_in && s->x0 == nullptr) return kErrArg;
  if (plain_in && !aligned(s->x0, 16)) return kErrAlign;
  if (attn) {
    if (s->pos == nullptr || s->rope_cos == nullptr || s->rope_sin == nullptr || s->max_pos < 1 ||
        s->max_pos > 65536)
      return kErrArg;
    if (!aligned(s->pos, 4) || !aligned(s->rope_cos, 16) || !aligned(s->rope_sin, 16)) return kErrAlign;
  }
  return kOk;
}
}  // namespace

int otq_step_table_bytes(int64_t* bytes) {
  if (bytes == nullptr) return kErrArg;
  *bytes = step_table_bytes();
  return kOk;
}

int otq_step_prepare(const otq_step* s, void* table) {
  int st = device_ok();
  if (st) return st;
  if ((st = check_step(s))) return st;
  if (table == nullptr) return kErrArg;
  if (!aligned(table, 128)) return kErrAlign;
  return finish(step_prepare(s, table));
}

int otq_decode_step(const otq_step* s, const void* table, void* stream) {
  int st = device_ok();
  if (st) return st;
  if ((st = check_step(s))) return st;
  if (table == nullptr) return kErrArg;
  if (!aligned(table, 128)) return kErrAlign;
  return finish(step_launch(s, table, static_cast<cudaStream_t>(stream)));
}

int otq_pack_g32(const float* W, int64_t N, int64_t K, int64_t ldw, uint8_t* codes,
                 uint16_t* scales, void* stream) {
  int st = device_ok();
  if (st) return st;
  if (N < 0 || K <= 0 || K % 32 || ldw < K || W == nullptr || codes == nullptr ||
      scales == nullptr)
    return kErrArg;
  if (!aligned(scales, 2)) return kErrAlign;
  return finish(pack_g32_launch(W, N, K, ldw, codes, scales, static_cast<cudaStream_t>(stream)));
}

int otq_linear_g32(const uint8_t* codes, const uint16_t* scales, int64_t N, int64_t K,
                   const float* x, int64_t ldx, int64_t M, int accumulate, float* y, int64_t ldy,
                   void* stream) {
  int st = device_ok();
  if (st) return st;
  if (N <= 0 || K <= 0 || K % 128 || K > 65536 || M <= 0 || M > 0x7FFFFFFF) return kErrArg;
  if (codes == nullptr || scales == nullptr || x == nullptr || y == nullptr) return kErrArg;
  if (ldx < K || ldy < N) return kErrArg;
  if (!aligned(codes, 16) || (K / 2) % 16 || !aligned(scales, 2) || !aligned(x, 16) ||
      ldx % 4)
    return kErrAlign;
  if (static_cast<int64_t>(K) * 4 * 2 > 227 * 1024) return kErrArg;
  return finish(linear_g32_launch(codes, scales, N, static_cast<int>(K), x, ldx,
                                  static_cast<int>(M), accumulate, y, ldy,
                                  static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
