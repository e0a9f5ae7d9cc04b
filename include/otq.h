/*
 * libotq -- openTPU's quantized linear layer on NVIDIA B200 (sm_100a): the C ABI.
 *
 * The reference (FeSens/openTPU) is a Python package; this ABI is what its numpy call sites for
 * the quantized linear layer would bind through ctypes. Each entry point names the reference
 * function (path:line inside the reference project) whose results it reproduces.
 *
 * Conventions
 *  - Every pointer is a CUDA device pointer (or managed memory) owned by the caller; no entry
 *    point allocates device memory and none keeps a pointer after it returns.
 *  - `stream` is a cudaStream_t (NULL: the legacy default stream). Calls are asynchronous on
 *    that stream and may be captured into CUDA graphs.
 *  - Return 0 (OTQ_OK) or a negative status; nothing is thrown, nothing is printed, no device
 *    assert is used. Shapes, strides and alignments are checked on the host before a launch.
 *  - Row-major matrices with explicit leading dimensions in ELEMENTS; packed weight rows and
 *    scale rows with strides in BYTES, exactly the reference's byte layouts.
 */
#ifndef OTQ_H_
#define OTQ_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define OTQ_API __attribute__((visibility("default")))
#else
#define OTQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status codes */
#define OTQ_OK 0
#define OTQ_ERR_ARG (-1)    /* a size, stride, flag or null pointer out of range */
#define OTQ_ERR_ALIGN (-2)  /* a pointer or stride not aligned as the entry point requires */
#define OTQ_ERR_FORMAT (-3) /* unknown weight format, or a format/flag combination MM refuses */
#define OTQ_ERR_CUDA (-4)   /* a CUDA runtime error (otq_last_cuda_error names it) */
#define OTQ_ERR_DEVICE (-5) /* the current device is not a compute-capability 10.x GPU */

/* ------------------------------------------------------------------ weight formats
 * The MM instruction's WF codes (opentpu/isa.py:26-27; docs/isa.md "Weight formats"):
 * int8 = int8x (one dw byte a 128-block), int4 = int4x and fp4 = fp4x6 (a word a block: dw and
 * four 6-bit multipliers), nvfp4 (eight E4M3 bytes a block), each under a per-row fp32 Sw. */
#define OTQ_FMT_INT8 0
#define OTQ_FMT_INT4 1
#define OTQ_FMT_FP4 2
#define OTQ_FMT_NVFP4 3

/* MM flag bits, the reference's own values (opentpu/isa.py:21 F_UNIT/F_ACC/F_ASCALE, :30 F_RSC) */
#define OTQ_MM_UNIT 0x1   /* no scale rows: Sw = 1, dw = 0, m = 1 */
#define OTQ_MM_ACC 0x2    /* y = y_old + MM */
#define OTQ_MM_ASCALE 0x8 /* y = y_old * alpha[j] + MM (needs UNIT) */
#define OTQ_MM_RSC 0x80   /* scale rows are Sw alone (4 bytes a row): dw = 0, m = 1 */

/* The quantization block D of every MX entry point (the MXU's D on the reference's targets). */
#define OTQ_D 128

OTQ_API const char* otq_version(void);
OTQ_API const char* otq_status_string(int status);
/* The message of the last CUDA error an entry point met on this thread ("" if none). */
OTQ_API const char* otq_last_cuda_error(void);
/* OTQ_OK if the current device is compute capability 10.x (the library is built for sm_100a). */
OTQ_API int otq_device_check(void);

/* ------------------------------------------------------------------ quantizers */

/* QACT / QST row quantization: fp32.quantize_mx (opentpu/fp32.py:321-343), QACT
 * (opentpu/isasim.py:913-959). Rows of x [rows, n] (ldx floats apart) -> q int8 [rows, n]
 * (ldq bytes apart), S fp32 [rows], d uint8 [rows, n/group] (ldd bytes apart; may be NULL in
 * row mode). group: a multiple of 32 dividing n (QACT: 32 = D/4; QST and int8x weights: 128).
 * row_mode != 0: every d = 0 (QACT/QST flag ROW). n <= 32768. */
OTQ_API int otq_quantize_rows(const float* x, int64_t rows, int64_t n, int64_t ldx, int group,
                      int row_mode, int8_t* q, int64_t ldq, float* S, uint8_t* d, int64_t ldd,
                      void* stream);

/* int8 weight rows as MM streams them. rsc == 0: quant.quantize_mxu(W, "int8") -- int8x
 * (opentpu/quant.py:316-323, scale rows by pack_scales :403-426): rows [N, K] int8 and scale
 * rows [N, srs] = Sw, one dw byte a 128-block, zero padding (srs >= 4 + 4*ceil(K/512)).
 * rsc != 0: runtime.quantize_rows(W, D, row=True) (opentpu/runtime.py:66-76), the
 * "int8 per output row with an fp32 scale" of quant.quantize(W, "int8", g=K)
 * (opentpu/quant.py:218-224): scale rows are Sw alone (srs >= 4). K % 128 == 0, K <= 32768. */
OTQ_API int otq_pack_int8(const float* W, int64_t N, int64_t K, int64_t ldw, int rsc, uint8_t* rows,
                  int64_t rs, uint8_t* srows, int64_t srs, void* stream);

/* Every MX weight format: quant.quantize_mxu(W, fmt) (opentpu/quant.py:510-524 -> quantize_mx
 * :484-503): int8 (_int8x :316-323), int4 / fp4 (_x4 :325-367: int4x / fp4x6, the 13-point
 * squared-error search of the 6-bit multipliers, in float64), nvfp4 (_nv :370-401, per-row
 * fp32 scale, E4M3 per 16 by the same search). rows [N, rs bytes] (rs >= row_bytes: K for
 * int8, 128*ceil(K/256) for 4-bit; padding written 0), scale rows [N, srs bytes]
 * (srs >= quant.scale_bytes; padding written 0). K % 128 == 0, K <= 32768. */
OTQ_API int otq_quantize_mxu(int fmt, const float* W, int64_t N, int64_t K, int64_t ldw,
                             uint8_t* rows, int64_t rs, uint8_t* srows, int64_t srs,
                             void* stream);

/* ------------------------------------------------------------------ MM */

/* MM over one QACT range: Slice._mm (opentpu/isasim.py:749-910; docs/isa.md "MM").
 * Weights: rows [N, rs bytes] (int8: K bytes used; 4-bit: K/2, element 2i in the low nibble),
 * scale rows [N, srs bytes] read at block k0 + k (NULL with OTQ_MM_UNIT).
 * Activations as otq_quantize_rows(group 32) leaves them: q [M, K] (ldq), Sa [M],
 * da [M, K/32] (ldd). Output y [M, N] (ldy floats apart); alpha [M] for OTQ_MM_ASCALE.
 * Bit-exact: one exact integer per output, then the reference's three-product fp32 epilogue.
 * K % 128 == 0, K <= 32640 (KB < 256, the MM field), rows/rs 16-byte aligned, scale rows aligned
 * to 4 (int8, RSC), 8 (int4, fp4) or 16 (nvfp4) bytes; nvfp4 takes no RSC. */
OTQ_API int otq_mm(int fmt, int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows, int64_t srs,
           int k0, int64_t N, int64_t K, const int8_t* q, int64_t ldq, const float* Sa,
           const uint8_t* da, int64_t ldd, int64_t M, const float* alpha, float* y, int64_t ldy,
           void* stream);

/* QACT then MM on fp32 rows, fused in one kernel: what the reference's ol.dot does to a TMEM
 * tile (opentpu/language.py:150-162; compiler.py:2622-2726 emits one QACT for the whole row
 * and one MM; isasim.py:913-959 then 749-910). x [M, K] (ldx floats apart); row_mode != 0 is
 * QACT ROW. Same weight arguments, flags and output as otq_mm. The QACT bytes are recomputed
 * by every CTA in shared memory: nothing is written to global memory but y. */
OTQ_API int otq_qmm(int fmt, int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
            int64_t srs, int k0, int64_t N, int64_t K, const float* x, int64_t ldx, int row_mode,
            int64_t M, const float* alpha, float* y, int64_t ldy, void* stream);

/* Launch-tuning variant of otq_qmm for benchmarks and tests: k_split 32 selects 32-row blocks a
 * warp, 1 8-row blocks, 2 / 4 / 8 8-row blocks whose K range that many warps share; 0 picks. pdl != 0
 * launches with programmatic dependent launch (the kernel streams its first weight chunks, then
 * waits on griddepcontrol before reading x). Same results as otq_qmm for every setting. No
 * counterpart in the reference (its MM has one implementation). */
OTQ_API int otq_qmm_ex(int fmt, int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
               int64_t srs, int k0, int64_t N, int64_t K, const float* x, int64_t ldx,
               int row_mode, int64_t M, const float* alpha, float* y, int64_t ldy,
               int k_split, int pdl, void* stream);

/* The NVLink fan-out of a row-sharded decode projection (otq_qmm_peer). The ranks' output rows
 * live in symmetric buffers (one allocation a rank, mapped into every rank's address space);
 * delta[r] is the byte distance from this rank's buffer to rank r's as mapped here (delta[rank]
 * = 0). world 1 is one GPU: tagged outputs in its own memory, no fan-out. seq, done: two words
 * of this GPU's memory, both zero before this rank's first otq_qmm_peer launch.
 *
 * Counted tags (tags = OTQ_TAGS_COUNTED): the launches keep done at zero between launches and
 * seq equal to the number of otq_qmm_peer launches this rank has run; a launch's outputs carry
 * tag seq + 1, read after the launch before it has finished.
 *
 * Stepped tags (tags = OTQ_TAGS_STEPPED): the launches form steps, a fixed sequence of
 * launches run again and again (a decode step), each with its position step_pos (0 .. 1022) in
 * the step, and seq counts completed steps: position p of step s tags its outputs s * 1024 + p
 * + 1, and with wait != 0 reads x until its tags reach s * 1024 + p (the output of position p -
 * 1 of the same step). Such a launch does not wait for the launch before it to finish (its
 * input's tags order it; launched with pdl != 0 it overlaps that launch's tail); launches with
 * wait == 0 wait for it as usual. The launch with step_last != 0 ends the step: when all its
 * CTAs are done, seq advances. Every launch of a step must follow the one before it on one
 * stream, and only the launch at position p - 1 writes the words a position-p launch waits on. */
#define OTQ_TAGS_COUNTED 0
#define OTQ_TAGS_STEPPED 1
typedef struct otq_peer {
  int rank;
  int world;             /* 1 .. 8 */
  int wait;              /* != 0: x is the previous projection's tagged output row */
  int tags;              /* OTQ_TAGS_COUNTED or OTQ_TAGS_STEPPED */
  int64_t delta[8];
  int* seq;
  int* done;
  int step_pos;          /* stepped tags: this launch's position in its step */
  int step_last;         /* stepped tags: != 0 for the step's last launch */
} otq_peer;

/* QACT + MM of one activation row against this rank's rows of a row-sharded projection
 * (runtime.Weight(shard=0), opentpu/runtime.py:138-142), with the all-gather of the output
 * (the reference's GATHER, opentpu/isasim.py:1413-1438) fused into the kernel. Output rows are
 * tagged: element i is one 8-byte word, the fp32 value in the low 4 bytes and a tag in the high
 * 4, and y is this rank's N words (16-byte aligned) of its symmetric copy of the output row.
 * Each word is also stored at the same place in every other rank's copy over NVLink, with tag =
 * seq + 1. With wait != 0, x is such a tagged row (K words, 16-byte aligned) and the kernel
 * reads each element until its tag reaches seq: every rank's previous output has arrived. With
 * wait == 0, x is plain fp32. Every rank must run the same sequence of launches. The values are
 * otq_qmm's bit for bit; a read that waits too long sets the status word (the launch's outputs
 * are then not valid). No ACC or ASCALE. No counterpart in the reference (its GATHER is a
 * separate instruction). */
OTQ_API int otq_qmm_peer(int fmt, int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
                         int64_t srs, int k0, int64_t N, int64_t K, const float* x, int64_t ldx,
                         int row_mode, float* y, const otq_peer* peer, int pdl, void* stream);

/* One projection of a chain (otq_qmm_chain): the operands of otq_qmm for one activation row. */
typedef struct otq_proj {
  int fmt;               /* OTQ_FMT_* */
  int flags;             /* OTQ_MM_UNIT / OTQ_MM_RSC / OTQ_MM_ACC (ASCALE needs otq_qmm) */
  const uint8_t* rows;   /* weight rows [N][rs] (16-byte aligned, rs a multiple of 16) */
  int64_t rs;
  const uint8_t* srows;  /* scale rows [N][srs], or NULL with OTQ_MM_UNIT */
  int64_t srs;
  int k0;                /* first 128-element block of the scale rows (column part) */
  int64_t N;
  int64_t K;
  const float* x;        /* the activation row [K]; may be an earlier projection's y */
  int row_mode;          /* QACT ROW */
  float* y;              /* [N] */
} otq_proj;

/* QACT + MM of `count` projections in order, one activation row each, in one persistent
 * launch per run of projections of the same format and kind (RSC / UNIT or MX): a projection
 * may read (x) what an earlier one wrote (y) -- a decode step's chain of linear layers. The
 * results are those of otq_qmm called once per projection in order. The CTAs of a launch are
 * co-resident (cooperative launch) and meet at a grid barrier between projections, whose two
 * counter words are static device memory of this library: launches of chains on one device
 * must not overlap (they serialise on a stream or on the device's SMs). A barrier wait is
 * bounded: if it runs out, the status word records it (otq_status_word) and the results are
 * not valid. No counterpart in the reference (its projections are separate programs). */
OTQ_API int otq_qmm_chain(const otq_proj* projs, int count, void* stream);

/* The device status word of the current device (synchronous): bit 0 set means a kernel's
 * bounded wait (on a shared-memory barrier, or a chain's grid barrier) ran out; that launch's
 * outputs are not valid. reset != 0 clears it (and, if it was set, re-arms the grid barrier). No counterpart in the reference (a simulator has no
 * such failure). */
OTQ_API int otq_status_word(int* value, int reset);

/* How long a kernel waits for tagged input words (otq_qmm_peer with wait != 0, otq_decode_step) on the current
 * device: `polls` reads of a word that has not arrived, with a short back-off between them,
 * before the wait gives up, sets bit 0 of the status word and lets the launch finish (its
 * outputs are then not valid). 0 restores the default of 2^22 polls (about a quarter of a
 * second). A failure detector sets a short limit so that a rank that never writes its words
 * turns into a status the host reads instead of a long stall. Applies to launches made after
 * the call. No counterpart in the reference. */
OTQ_API int otq_set_wait_limit(uint32_t polls);

/* ------------------------------------------------------------------ the decode step, one launch */

/* Stage kinds of otq_decode_step: a projection in a weight format, or the attention. */
#define OTQ_STEP_RSC 0   /* int8 rows with a per-row fp32 scale (MM RSC) or UNIT: QACT + MM */
#define OTQ_STEP_G32 1   /* 4-bit group-32 fp16-scale rows (otq_pack_g32): weight-only */
#define OTQ_STEP_ATTN 2  /* no weights: causal softmax attention of one query row over a KV cache */

/* What a projection's input row is. */
#define OTQ_IN_DEFAULT 0 /* x0 when in == -1, else the first K outputs of projection `in` */
#define OTQ_IN_NORM 1    /* the residual row (x0 when res == -2, else the residual so far plus
                            the output of projection `res`), RMSNorm'ed and times gamma */
#define OTQ_IN_SWIGLU 2  /* silu(y[0:K]) * y[K:2K], y the output of projection `in` */
#define OTQ_IN_ATTN 3    /* the output of attention stage `in` */

/* What a projection writes. */
#define OTQ_EPI_NONE 0   /* its N output rows */
#define OTQ_EPI_SWIGLU 1 /* rows are gate and up rows interleaved in blocks of 8 (rows 16j .. 16j + 7
                            gate rows 8j .. 8j + 7, rows 16j + 8 .. 16j + 15 the up rows 8j ..
                            8j + 7; N a multiple of 16, at most 112 rows an SM); it writes
                            silu(gate) * up, N / 2 words */

/* One projection of otq_decode_step. */
typedef struct otq_step_proj {
  const uint8_t* rows;   /* RSC: int8 rows [N][rs]; G32: codes [N][rs] (K/2 bytes used).
                            16-byte aligned, rs a multiple of 16 */
  int64_t rs;
  const uint8_t* srows;  /* RSC: scale rows [N][srs], Sw their first fp32 word, or NULL (UNIT);
                            G32: fp16 scales [N][srs] (K/16 bytes used, 16-byte aligned, srs a
                            multiple of 16) */
  int64_t srs;
  int64_t N;             /* this rank's rows (with world > 1: its contiguous row shard) */
  int64_t K;             /* RSC: a multiple of 128; G32: of 256; at most 8192 (OTQ_IN_NORM: 4096) */
  int in;                /* -1: the input is x0; else the index of an earlier stage (see input) */
  int fmt;               /* OTQ_STEP_RSC, OTQ_STEP_G32 or OTQ_STEP_ATTN */
  int input;             /* OTQ_IN_* */
  int res;               /* OTQ_IN_NORM: -2, or the projection added to the residual first */
  const float* gamma;    /* OTQ_IN_NORM: the norm's gains [K] (16-byte aligned) */
  /* OTQ_STEP_ATTN: `in` is the QKV projection (q [n_q * hd], k [n_kv * hd], v [n_kv * hd]);
   * N = n_q * hd + n_q * ceil(max_pos / 32) * (hd + 2) words: the attention's output row (query
   * head major: the input of an OTQ_IN_ATTN projection) and the partial results of its chunks of
   * 32 positions; K unused. q and k of the new token:
   * per-head RMSNorm times q_gain / k_gain (NULL: none), then rotate-half RoPE at *pos; k and v
   * go into the caches at *pos. At most 2 * (n_q / n_kv) * ceil(max_pos / 32) <= 2048. */
  const float* q_gain;
  const float* k_gain;
  float* kcache;         /* [max_pos][n_kv][hd] fp32 (16-byte aligned) */
  float* vcache;
  int n_q, n_kv, head_dim;   /* head_dim 128, n_q / n_kv at most 4 */
  int epilogue;          /* OTQ_EPI_* (projections; not the last stage) */
  int replicated;        /* world > 1: 0, the rows are this rank's contiguous shard of the
                            projection (its output words go to every rank); 1, every rank holds
                            all N rows and computes the projection alone (its output stays on
                            this GPU: no NVLink traffic) */
} otq_step_proj;

#define OTQ_STEP_MAX 160

typedef struct otq_step {
  const otq_step_proj* projs;
  int count;             /* 1 .. OTQ_STEP_MAX */
  int rank, world;       /* world 1 .. 8: the projections' rows are split over the ranks */
  int64_t delta[8];      /* byte distance from this rank's `out` to rank r's, as mapped here */
  const float* x0;       /* the plain input row (16-byte aligned) */
  float* out;            /* every projection's output row as tagged 8-byte words (fp32 value,
                            32-bit tag), at the word offsets otq_step_layout gives: this rank's
                            copy of a symmetric buffer (16-byte aligned), all zero before the
                            first step */
  int* counters;         /* 4 ints of this GPU's memory (16-byte aligned), zero before the first
                            step: steps completed, CTAs done, the greedy token's accumulator */
  int64_t* token;        /* the index of the first maximum of the last projection's full output
                            row (the greedy token), or NULL */
  /* decoder steps (OTQ_IN_NORM, OTQ_STEP_ATTN): */
  float eps;             /* RMSNorm epsilon */
  const float* rope_cos; /* [max_pos][hd / 2] */
  const float* rope_sin;
  int max_pos;
  int* pos;              /* this step's position (device int), advanced at the end of the step */
  const float* embed;    /* [vocab][K0]: if not NULL, x0 is embed[*token_in] */
  const int64_t* token_in;
  int64_t vocab;
} otq_step;

/* Word offsets of every projection's output row (offsets[count], may be NULL) and the words
 * the buffer needs (total_words): each row N * world words, 16-byte aligned. */
OTQ_API int otq_step_layout(const otq_step_proj* projs, int count, int world, int64_t* offsets,
                            int64_t* total_words);

/* Bytes of the device table otq_step_prepare writes (the projections' tensor maps and
 * operands, read by the kernel; 128-byte aligned device memory of the caller). */
OTQ_API int otq_step_table_bytes(int64_t* bytes);

/* Checks a step and writes its table into `table` (synchronous: call it before any stream
 * capture, and again when a pointer of the step changes). */
OTQ_API int otq_step_prepare(const otq_step* step, void* table);

/* One decode step -- every projection of one activation row in order, each reading an earlier
 * one's output -- as ONE persistent launch (the reference's qwen3_step, opentpu/llm/qwen3.py:
 * 1793, runs them as a sequence of QACT + MM programs, opentpu/isasim.py:749-959, with GATHER,
 * :1413-1438, between row-sharded slices). Projections are ordered by their data: each output
 * element is stored as a tagged word (with world > 1 also into every other rank's copy over
 * NVLink: the all-gather fused in), and a projection reads its input words until their tags
 * show the current step. RSC projections are bit-identical to otq_qmm; G32 ones are otq_linear_g32's
 * arithmetic in another fp32 summation order. `table`: written by otq_step_prepare for this
 * step. Steps must follow one another on one stream (a launch reads the step count the launch
 * before advanced); with world > 1 every rank runs the same steps. A wait that runs out
 * (otq_set_wait_limit) sets the status word. All CTAs must be resident at once (a cooperative
 * launch of one CTA an SM). No counterpart in the reference (its projections are separate
 * programs). */
OTQ_API int otq_decode_step(const otq_step* step, const void* table, void* stream);

/* ------------------------------------------------------------------ prefill GEMM */

/* One projection of otq_gemm_w8a16_group. */
typedef struct otq_gemm_proj {
  int flags;             /* OTQ_MM_RSC (Sw = the first fp32 word of each scale row) or
                            OTQ_MM_UNIT (Sw = 1), either one | OTQ_MM_ACC */
  const uint8_t* rows;   /* int8 weight rows [N][rs] (16-byte aligned, rs a multiple of 16) */
  int64_t rs;
  const uint8_t* srows;  /* scale rows [N][srs] (4-byte aligned), or NULL with OTQ_MM_UNIT */
  int64_t srs;
  int64_t N;
  int64_t K;
  const uint16_t* x;     /* bf16 activations [M][ldx] (16-byte aligned, ldx a multiple of 8) */
  int64_t ldx;
  int64_t M;
  float* y;              /* fp32 output [M][ldy] (4-byte aligned) */
  int64_t ldy;
} otq_gemm_proj;

/* The int8 weight-only linear layer on bf16 activations, as a tensor-core GEMM (prefill):
 * y [M, N] = x [M, K] @ (q * Sw)^T, q the int8-row bytes of otq_pack_int8(rsc = 1) --
 * quant.quantize(W, "int8", g=K) (opentpu/quant.py:218-224) used as `deq @ x`
 * (opentpu/reference.py:14-17). int8 and bf16 are exact in the products; sums are fp32 in
 * tensor-core order, so results agree with a float64 evaluation to a relative tolerance
 * (not bit-exact; otq_qmm is the bit-exact MM). ACC: y += . K % 8 == 0. The reference's own
 * prefill quantizes activations first (QACT); a bf16 path has no single counterpart there. */
OTQ_API int otq_gemm_w8a16(int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
                           int64_t srs, int64_t N, int64_t K, const uint16_t* x, int64_t ldx,
                           int64_t M, float* y, int64_t ldy, void* stream);

/* Up to 8 independent projections of otq_gemm_w8a16 in one launch (their tiles share the
 * GPU's SMs: a layer's projections at prefill). The outputs must not overlap the inputs or
 * each other. No counterpart in the reference (its projections are separate programs). */
OTQ_API int otq_gemm_w8a16_group(const otq_gemm_proj* projs, int count, void* stream);

/* ------------------------------------------------------------------ exact W8A8 MM on tcgen05 */

/* Bytes of the activation planes buffer for M rows of K (M >= 0, K > 0 and K % 32 == 0), or a
 * negative OTQ_ERR_*: about 3 M K. */
OTQ_API int64_t otq_qact_planes_bytes(int64_t M, int64_t K);

/* QACT of x [M, K] fp32 (ldx elements a row; the reference's quantize_mx with an offset per 32
 * elements, opentpu/fp32.py:321-343; row_mode = QACT ROW) into `planes` (device memory, 16-byte
 * aligned, at least otq_qact_planes_bytes(M, K) bytes), the form otq_gemm_w8a8_group reads: a
 * row's QACT scale, its largest kept offset D, and its bytes times 2^(D - d) split into up to
 * three signed base-256 int8 planes. K % 32 == 0, K <= 65536. No counterpart in the reference
 * (its QACT writes bytes and offsets; this is the same quantization laid out for the tensor
 * cores). */
OTQ_API int otq_qact_planes(const float* x, int64_t ldx, int64_t M, int64_t K, int row_mode,
                            void* planes, int64_t bytes, void* stream);

/* One projection of otq_gemm_w8a8_group. */
typedef struct otq_gemm8_proj {
  int flags;             /* OTQ_MM_RSC (Sw = the first fp32 word of each scale row) or
                            OTQ_MM_UNIT (Sw = 1), either one | OTQ_MM_ACC */
  const uint8_t* rows;   /* int8 weight rows [N][rs] (16-byte aligned, rs a multiple of 16) */
  int64_t rs;
  const uint8_t* srows;  /* scale rows [N][srs] (4-byte aligned), or NULL with OTQ_MM_UNIT */
  int64_t srs;
  int64_t N;
  int64_t K;             /* K % 32 == 0, K <= 65536 */
  const void* planes;    /* otq_qact_planes of the activations [M][K] */
  int64_t M;
  float* y;              /* fp32 output [M][ldy] (4-byte aligned) */
  int64_t ldy;
} otq_gemm8_proj;

/* MM of int8-row weights (RSC or UNIT) and QACT activations on the tcgen05 tensor cores
 * (kind::i8), up to 8 independent projections in one launch: y = MM(QACT(x), rows), the same
 * bits as otq_qmm(OTQ_FMT_INT8, flags) -- the reference's exact integer accumulation
 * (opentpu/isasim.py:749-910) and fp32 epilogue, for any M (prefill; batched decode). ACC:
 * y = fadd(y, MM). Outputs must not overlap the inputs or each other. M is at most
 * 32768 tokens a projection. */
OTQ_API int otq_gemm_w8a8_group(const otq_gemm8_proj* projs, int count, void* stream);

/* otq_qact_planes then otq_gemm_w8a8_group of one projection: otq_qmm(OTQ_FMT_INT8, flags, ...,
 * k0 = 0, alpha = NULL) on the tensor cores, with the caller's planes buffer as scratch. */
OTQ_API int otq_qmm_tc(int flags, const uint8_t* rows, int64_t rs, const uint8_t* srows,
                       int64_t srs, int64_t N, int64_t K, const float* x, int64_t ldx,
                       int row_mode, int64_t M, void* planes, int64_t planes_bytes, float* y,
                       int64_t ldy, void* stream);

/* ------------------------------------------------------------------ greedy token */

/* The index of the first maximum of x[0], x[stride], ..., x[(n - 1) * stride] (stride 2 reads
 * the values of a tagged row of otq_qmm_peer): the reference's greedy sink on the LM head's
 * logits (llm/generate.py:252-280, numpy argmax, ties to the lowest index). out: two int64
 * words of device memory (16-byte aligned), used as the reduction's accumulator and CTA count;
 * the call zeroes them on `stream`, and after the launch out[0] holds the index and out[1]
 * zero. 1 <= n < 2^32. */
OTQ_API int otq_argmax(const float* x, int64_t n, int64_t stride, int64_t* out, void* stream);

/* otq_argmax for callers that cannot allocate device memory: a plugin or custom operator inside
 * a host framework that owns every device buffer and hands it only its inputs and outputs, or a
 * latency-critical loop where a cudaMalloc (which may synchronize the device) is not allowed.
 * Such a caller has nowhere to put otq_argmax's 16 bytes of scratch; this call keeps them in a
 * 256-byte array of the library's own device memory (present on every GPU that loads the
 * library, until the process exits) and writes only the result: *index (one int64 of device
 * memory, 8-byte aligned) = the index of the first maximum of x[0], x[stride], ...,
 * x[(n - 1) * stride]. Nothing is allocated. Limits: 1 <= n < 2^32 (the largest row whose
 * index fits the scratch key); a longer row returns OTQ_ERR_ARG. The first call on each device
 * looks up the array's device address (a synchronous runtime call, made with that device
 * current), so make it before any stream capture. Every call uses the same array and zeroes it
 * first: calls that overlap on the GPU (on different streams) race and may return a wrong
 * index. No counterpart in the reference (its argmax is numpy on the host). */
OTQ_API int otq_argmax_noalloc(const float* x, int64_t n, int64_t stride, int64_t* index,
                               void* stream);

/* ------------------------------------------------------------------ 4-bit group-32 fp16 */

/* quant.quantize(W, "int4", g=32, scale="fp16") (opentpu/quant.py:225-227 -> quant_block
 * :132-142 -> _quant_rows :144-170): per 32 elements s = fp16(min(amax/7, 65504)) (1 if amax or
 * s is 0) and w = clip(rint(x/s), -7, 7), computed in float64 as the reference does. Output:
 * codes [N, K/2] bytes (two's-complement nibbles, element 2i low), scales [N, K/32] fp16 bits.
 * K % 32 == 0. */
OTQ_API int otq_pack_g32(const float* W, int64_t N, int64_t K, int64_t ldw, uint8_t* codes,
                 uint16_t* scales, void* stream);

/* Weight-only linear over that format: y [M, N] = x [M, K] @ deq^T with deq = w * s, fp32
 * accumulation (the reference's `quant.quantize(...).deq @ x` pattern,
 * tests/test_quant.py:276-287, reference.py:14-17). Tolerance, not bit-exact. ACC: y += . */
OTQ_API int otq_linear_g32(const uint8_t* codes, const uint16_t* scales, int64_t N, int64_t K,
                   const float* x, int64_t ldx, int64_t M, int accumulate, float* y, int64_t ldy,
                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OTQ_H_ */
