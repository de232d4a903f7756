/* sfb200.h - C ABI of the B200 (sm_100a) sf hot-path library, libsfb200.so.
 *
 * Codes: every sfN value (N = 4..16) is held in device memory as a signed
 * 16-bit integer code k in [-M, M], M = 2^(N-1) - 1, value k / 2^(N-1)
 * (the reference keeps the same signed codes as int64 NumPy arrays,
 * src/sf/_format.py:1-11).  All buffers are caller-owned DEVICE pointers
 * on the current CUDA device; every call is asynchronous on `stream`
 * (a cudaStream_t, NULL = the legacy default stream).  No call allocates
 * device memory.
 *
 * Status: each call adds its event counts into `counts` (device memory,
 * one sfb_counts; the caller zeroes it) and, when `flags` is not NULL,
 * writes one event byte per output (SFB_F_* bits).  An event count is the
 * number of OUTPUTS whose computation raised that event, which is what the
 * reference's runtime counts from its per-output masks
 * (src/sf/_array.py:555-569).
 *
 * Errors: every entry point returns 0 on success or a negative SFB_E* code;
 * sfb_last_error() then gives a message (per thread).  No exception and no
 * process exit crosses this boundary.
 */
#ifndef SFB200_H
#define SFB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SFB_ABI_VERSION 1

#if defined(__GNUC__)
#define SFB_API __attribute__((visibility("default")))
#else
#define SFB_API
#endif

/* return codes */
#define SFB_OK 0
#define SFB_EINVAL (-1)   /* bad argument: width, op, shape, null pointer */
#define SFB_ECUDA (-2)    /* a CUDA runtime error (launch, device) */
#define SFB_ERANGE (-3)   /* a size beyond what the kernels index */
#define SFB_ENODEV (-4)   /* no sm_100 device */

/* per-output event bits written to `flags` */
#define SFB_F_OVERFLOW 1u
#define SFB_F_UNDERFLOW 2u
#define SFB_F_DIVIDE 4u
#define SFB_F_INVALID 8u
#define SFB_F_ACC_CLIPPED 16u /* wide only: the MX accumulator reached its limit */

/* elementwise ops (the reference's device op table, src/sf/_device.py:181-185) */
#define SFB_OP_ADD 0
#define SFB_OP_SUB 1
#define SFB_OP_MUL 2
#define SFB_OP_DIV 3
#define SFB_OP_FMA 4
#define SFB_OP_NEG 5
#define SFB_OP_ABS 6
#define SFB_OP_SQRT 7
#define SFB_OP_POW 8

/* MX engine versions (src/sf/_linalg.py:144-147) */
#define SFB_MX_V492 0
#define SFB_MX_V481 1

typedef struct sfb_counts {
    unsigned long long overflow;    /* outputs that saturated (any step) */
    unsigned long long underflow;   /* outputs where a nonzero result became 0 */
    unsigned long long divide;      /* div outputs with a zero divisor */
    unsigned long long invalid;     /* sqrt outputs of a negative input */
    unsigned long long acc_clipped; /* wide outputs whose accumulator clipped */
    unsigned long long reserved[3];
} sfb_counts;

typedef void *sfb_stream; /* a cudaStream_t */

/* float element types of sfb_scan / sfb_quantize */
#define SFB_F32 0
#define SFB_F64 1

/* Statistics of a float tensor and of its quantization (device memory; the
 * caller zeroes it): scan -> nan_count, inf_count, absmax (largest finite |x|);
 * quantize -> overflow / underflow / invalid counts of the cast, the largest
 * row L1 norm of the codes and the largest |code|. */
typedef struct sfb_qstats {
    unsigned long long nan_count, inf_count;
    double absmax;
    unsigned long long overflow, underflow, invalid;
    long long max_row_l1, max_abs_code;
} sfb_qstats;

/* Library and device. */
SFB_API int sfb_abi_version(void);
SFB_API const char *sfb_last_error(void);
/* Makes `device` current for the calling thread and checks it is an sm_100
 * part.  Replaces the device attributes a reference target declares
 * (src/sf/_device.py:38-50). */
SFB_API int sfb_device_init(int device);

/* Elementwise op over n codes: out[i] = op(a[i], b[i], c[i]).
 * Replaces Device.run(op, fmt, a[, b[, c]]) for op in add, sub, mul, div, fma,
 * neg, abs, sqrt, pow (src/sf/_device.py:96-106, :138-148; semantics of
 * src/sf/_vectorized.py:94-156).  b is read by binary ops and fma, c by fma
 * only; pow_n is pow's exponent (>= 1).  Operands have n elements each (the
 * caller broadcasts).  Events: overflow (add, sub, div, fma), underflow (mul,
 * fma, pow), divide (div), invalid (sqrt). */
SFB_API int sfb_elementwise(int op, int bits, const int16_t *a, const int16_t *b, const int16_t *c,
                    int16_t *out, uint8_t *flags, int64_t n, int pow_n, sfb_counts *counts,
                    sfb_stream stream);

/* Chain matmul: per output a chain of fma in increasing k,
 * acc = clip(acc + trunc(a_k b_k / 2^(N-1))), then (bias != NULL) one
 * saturating add of bias[n].  Replaces Device.run("matmul", fmt, A, B)
 * (src/sf/_device.py:166-168 -> src/sf/_linalg.py:61-81) and, fused, the
 * add that follows it in the linear layer (src/sf/torch/_core.py:376-378).
 * A: batch x M x K, B: batch x K x N, out: batch x M x N, all row-major;
 * stride_a / stride_b / stride_out are the element strides between batch
 * entries (0 broadcasts one matrix over the batch); lda, ldb are the row
 * strides of A and B.  Overflow counts outputs where a chain step or the
 * bias add saturated; underflow outputs where a nonzero product truncated
 * to 0 on a step that did not saturate. */
SFB_API int sfb_matmul_chain(int bits, const int16_t *A, const int16_t *B, const int16_t *bias, int16_t *out,
                     uint8_t *flags, int64_t batch, int64_t M, int64_t N, int64_t K, int64_t lda,
                     int64_t ldb, int64_t stride_a, int64_t stride_b, int64_t stride_out,
                     sfb_counts *counts, sfb_stream stream);

/* The chain matmul of a converted linear layer, fused with its bias add and
 * its float64 dequantization: acc = X (R x K codes) @ WT (K x N codes) as in
 * sfb_matmul_chain, one saturating add of bias[n] (NULL: none), then
 * y = acc / 2^(N-1) * a * s_col[n] in float64, written as float32 (y32) and/or
 * float64 (y64); codes / flags optional.  Replaces the matmul, the add and the
 * dequantization of the reference's chain linear (src/sf/torch/_core.py:374-382).
 * proven_no_saturation: the caller has shown (the reference's L1 bound,
 * src/sf/_linalg.py:84-106) that no partial sum can reach +-max; the chain is
 * then summed without per-step clips.  If that proof is wrong the outputs are
 * not the reference's and counts->reserved[1] counts the outputs found out of
 * range. */
SFB_API int sfb_linear_chain(int bits, const int16_t *X, const int16_t *WT, const int16_t *bias, double a,
                             const double *s_col, int proven_no_saturation, float *y32, double *y64, int16_t *codes,
                             uint8_t *flags, int64_t R, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                             sfb_counts *counts, sfb_stream stream);

/* One pass over n floats (dtype SFB_F32 / SFB_F64): NaN and +-inf counts and
 * the largest finite magnitude, the inputs of the reference's sanitize /
 * finite_absmax (src/sf/torch/_core.py:200-236). */
SFB_API int sfb_scan(const void *x, int dtype, int64_t n, sfb_qstats *stats, sfb_stream stream);

/* codes[r, c] = cast(x[r, c] / s_r) for a rows x cols matrix (row stride ld,
 * codes row stride ldc), s_r = row_scale[r] or the scalar `scale` when
 * row_scale is NULL: the reference's cast of float64 values
 * (src/sf/_vectorized.py:32-71; float32 inputs widen exactly) with its
 * event counts, plus the largest row L1 norm and |code| of the result. */
SFB_API int sfb_quantize(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, double scale,
                         const double *row_scale, int bits, int16_t *codes, int64_t ldc, sfb_qstats *stats,
                         sfb_stream stream);

/* The converted layer's activation scale search with headroom="bound" on the
 * device, one cooperative launch (src/sf/torch/_core.py:200-236, :306-331):
 * scan, a0 = max finite |x| / m, casts of x / a (NaN read as 0, +-inf as +-max
 * finite |x|, the reference's sanitize), the bias step and the L1-bound loop,
 * leaving the final codes (R x K, row stride K) and the result struct on the
 * device.  w_max_abs / w_max_col_l1: max |W code| and max sum_k |W code| of the
 * prepared weight; has_bias, need_max = max |b| / s_w (inf allowed) and a_bias
 * the scale its largest finite ratio needs.  scratch: device bytes of
 * sfb_linear_scale_scratch().  err = 1: the search did not converge in 32
 * steps (the reference raises).  No counterpart entry in the reference, which
 * runs the search on the host. */
typedef struct {
    double a, a0;
    int64_t proven, iterations, nan_count, inf_count, underflow, err;
} sfb_scale_result;
SFB_API int64_t sfb_linear_scale_scratch(void);
SFB_API int sfb_linear_scale(const void *x, int dtype, int64_t R, int64_t K, int64_t ld, int bits,
                             int64_t w_max_abs, int64_t w_max_col_l1, int has_bias, double need_max, double a_bias,
                             int16_t *codes, sfb_scale_result *result, void *scratch, sfb_stream stream);

/* sfb_matmul_chain with a workspace: when the output has few tiles
 * (batch 1), each output's K is split into pieces summarised in parallel and
 * composed in order (the clamp-add maps of the chain compose exactly), the
 * same bits as the sequential chain.  workspace: sfb_matmul_chain_workspace()
 * bytes (0: no split); a smaller or null workspace runs the unsplit kernel. */
SFB_API int64_t sfb_matmul_chain_workspace(int64_t batch, int64_t M, int64_t N, int64_t K);
SFB_API int sfb_matmul_chain_ws(int bits, const int16_t *A, const int16_t *B, const int16_t *bias, int16_t *out,
                                uint8_t *flags, int64_t batch, int64_t M, int64_t N, int64_t K, int64_t lda,
                                int64_t ldb, int64_t stride_a, int64_t stride_b, int64_t stride_out, void *workspace,
                                int64_t workspace_bytes, sfb_counts *counts, sfb_stream stream);

/* sfb_linear_chain in proven mode with the activation scale read from
 * device memory (a_dev: the a of a finished sfb_linear_scale), so the
 * layer's kernels queue without a host round trip. */
SFB_API int sfb_linear_chain_dev(int bits, const int16_t *X, const int16_t *WT, const int16_t *bias,
                                 const double *a_dev, const double *s_col, float *y32, double *y64, int16_t *codes,
                                 uint8_t *flags, int64_t R, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                                 sfb_counts *counts, sfb_stream stream);

/* The bias codes of a converted layer at its scale: cast(b[n] / (a_dev[0] *
 * s_col[n])) with the cast rule of src/sf/_vectorized.py:59-71
 * (src/sf/torch/_core.py:376-378); *n_over += the codes that saturated. */
SFB_API int sfb_bias_codes(int bits, const double *b, const double *a_dev, const double *s_col, int64_t n,
                           int16_t *codes, int64_t *n_over, sfb_stream stream);

/* sfb_quantize with the scale a0 = absmax / m taken on the device from a
 * finished sfb_scan's statistics (1 when absmax is 0): the first pass of the
 * activation scale search (src/sf/torch/_core.py:306-331) without a host
 * round trip between the scan and the quantize. */
SFB_API int sfb_quantize_auto(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                              const sfb_qstats *scan, double m, int bits, int16_t *codes, int64_t ldc,
                              sfb_qstats *stats, sfb_stream stream);

/* Bytes of device workspace sfb_matmul_wide needs for this problem (0 when
 * it needs none); negative on a bad argument. */
SFB_API int64_t sfb_matmul_wide_workspace(int bits, int mx, int64_t batch, int64_t M, int64_t N, int64_t K);

/* Wide (MX engine) matmul: accumulators of the MX version `mx`
 * (src/sf/_linalg.py:261-308), then POP at the per-output shift
 * (src/sf/_linalg.py:201-220): shift_arr (int8, batch x M x N with strides
 * shift_sb / shift_sm / shift_sn, 0 to broadcast) or, when shift_arr is
 * NULL, the scalar `shift` (-32..31).  Replaces Device.run("matmul_wide",
 * fmt, A, B, shift=, mx=) (src/sf/_device.py:171-173).  Overflow counts
 * outputs whose accumulator clipped or whose POP saturated; underflow
 * nonzero totals that rounded to 0; acc_clipped the clipped accumulators.
 * `workspace` is caller-owned device memory of at least
 * sfb_matmul_wide_workspace() bytes (NULL when that is 0). */
SFB_API int sfb_matmul_wide(int bits, int mx, const int16_t *A, const int16_t *B, const int8_t *shift_arr,
                    int shift, int16_t *out, uint8_t *flags, int64_t batch, int64_t M, int64_t N,
                    int64_t K, int64_t lda, int64_t ldb, int64_t stride_a, int64_t stride_b,
                    int64_t stride_out, int64_t shift_sb, int64_t shift_sm, int64_t shift_sn,
                    void *workspace, int64_t workspace_bytes, sfb_counts *counts, sfb_stream stream);

/* Bytes of the prepared form of a wide B operand (N columns, K rows), 0 when
 * this width / MX version has none (the calls then read B's codes).  The
 * prepared form is the reference's prepared weight of its compiled MX loop
 * (_fastmx.prep_b, src/sf/_fastmx.py:168-173, used by
 * _linalg.matmul_wide_acc_prepared, src/sf/_linalg.py:311-321): B's operand
 * planes, bit slices and column statistics for the tensor-core path. */
SFB_API int64_t sfb_wide_prepared_b_bytes(int bits, int mx, int64_t N, int64_t K);

/* Prepare B (K x N codes, row stride ldb) once into `prep` (device memory
 * of sfb_wide_prepared_b_bytes() bytes) for sfb_matmul_wide_prepared; a B
 * that many calls share (a layer's weights, a replicated operand) is then
 * not re-prepared per call.  Asynchronous on `stream`. */
SFB_API int sfb_wide_prepare_b(int bits, int mx, const int16_t *B, int64_t N, int64_t K, int64_t ldb, void *prep,
                               int64_t prep_bytes, sfb_stream stream);

/* sfb_matmul_wide with B prepared by sfb_wide_prepare_b (the reference's
 * _linalg.matmul_wide_acc_prepared then POP, src/sf/_linalg.py:311-321 and
 * :201-220): one B for every batch entry; B's codes are still passed, for
 * the outputs the exact CUDA-core path recomputes.  `prep` NULL: exactly
 * sfb_matmul_wide with stride_b 0. */
SFB_API int sfb_matmul_wide_prepared(int bits, int mx, const int16_t *A, const int16_t *B, const void *prep,
                                     const int8_t *shift_arr, int shift, int16_t *out, uint8_t *flags, int64_t batch,
                                     int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t stride_a,
                                     int64_t stride_out, int64_t shift_sb, int64_t shift_sm, int64_t shift_sn,
                                     void *workspace, int64_t workspace_bytes, sfb_counts *counts,
                                     sfb_stream stream);

/* Failure-detection hook with no counterpart in the reference: the wide
 * tensor-core GEMM launches that the CALLING THREAD makes from now on bound
 * each of their pipeline waits (an mbarrier poll loop) by `polls` polls
 * (0 restores the default, 2^26), and with `stall` nonzero their MMA thread
 * first waits on a barrier that nothing arrives on.  A wait that runs out
 * adds 1 per CTA to counts->reserved[0]; the kernel still lets its copies in
 * flight land and frees its tensor memory before it returns, so the context
 * stays usable and the host reports the failure from the counts.  Tests
 * only: a stalled call's outputs are not valid.  Always returns SFB_OK. */
SFB_API int sfb_wide_wait_limit(unsigned polls, int stall);

/* sfb_matmul_wide without any device allocation, for callers that cannot
 * allocate device memory while they run: a host program that has handed all
 * of the GPU's memory to its own pool, a plugin host that forbids allocation
 * after start-up, or a loop that cannot afford the device-wide synchronisation
 * cudaMalloc / cudaFree can imply.  It has no counterpart in the reference.
 * The same arguments and results as sfb_matmul_wide, minus the workspace: the
 * scratch is a fixed 64 MiB array inside the library, held on every GPU that
 * loads the library until the process exits.  The first call on a device
 * looks up that array's address (with that device current), so make that
 * first call before any CUDA stream capture on the device; after a device
 * reset the next call looks it up again.  Problems whose scratch exceeds
 * 64 MiB (sfb_matmul_wide_workspace() > 64 MiB: 1536^3 fits, 2048^3 needs
 * about 109 MiB) are refused with SFB_ERANGE.  All calls share the one
 * array, so calls whose kernels overlap on the GPU (other streams or host
 * threads) race; serialise them. */
SFB_API int sfb_matmul_wide_noalloc(int bits, int mx, const int16_t *A, const int16_t *B, const int8_t *shift_arr,
                                    int shift, int16_t *out, uint8_t *flags, int64_t batch, int64_t M, int64_t N,
                                    int64_t K, int64_t lda, int64_t ldb, int64_t stride_a, int64_t stride_b,
                                    int64_t stride_out, int64_t shift_sb, int64_t shift_sm, int64_t shift_sn,
                                    sfb_counts *counts, sfb_stream stream);

/* The wide matmul's accumulators before POP: the reference's
 * _linalg.matmul_wide_acc (src/sf/_linalg.py:261-308).  Same operands,
 * strides and workspace as sfb_matmul_wide; acc[b * stride_acc + m * N + n]
 * receives the W-bit accumulator (int32 on both chips), clipped (nullable)
 * SFB_F_ACC_CLIPPED where it saturated; counts->acc_clipped adds those. */
SFB_API int sfb_matmul_wide_acc(int bits, int mx, const int16_t *A, const int16_t *B, int32_t *acc,
                                uint8_t *clipped, int64_t batch, int64_t M, int64_t N, int64_t K, int64_t lda,
                                int64_t ldb, int64_t stride_a, int64_t stride_b, int64_t stride_acc, void *workspace,
                                int64_t workspace_bytes, sfb_counts *counts, sfb_stream stream);

/* The wide sft linear after accumulation, per output of an (M, N) block of
 * accumulators (the reference's host runner, src/sf/torch/_core.py:68-98
 * and :162-190, with the shift rule of src/sf/_heuristic.py:123-169):
 * shift from the rule (use_rule = 1: row / column exponents, dequantized
 * row / column L2 norms, h) or the one explicit shift (use_rule = 0, no
 * redo); POP; the bias (N float64, nullable) at each output's exponent with
 * the saturating add; the redo POP; y = code 2^(exponent - (N-1)) written as
 * float32 (y32) and / or float64 (y64).  flags (nullable): SFB_F_OVERFLOW
 * where the POP or the bias add saturated, SFB_F_UNDERFLOW where a nonzero
 * total flushed to 0.  counts->overflow / underflow add those; stats (int64
 * x 4) receives redone += , bias codes clamped += , and the min / max shift
 * used by atomic min / max (start them at 127 and -128). */
SFB_API int sfb_wide_finish(int bits, int mx, const int32_t *acc, int64_t M, int64_t N, const int32_t *row_exp,
                            const int32_t *col_exp, const double *row_norm, const double *col_norm, int h,
                            int use_rule, int shift, const double *bias, float *y32, double *y64, uint8_t *flags,
                            int64_t *stats, sfb_counts *counts, sfb_stream stream);

/* Saturating sequential sum along one axis of int16 codes viewed as
 * (outer, K, inner), reduced over K from index 0: the reference's
 * _linalg.sum_codes (src/sf/_linalg.py:30-39), the Device "sum" op
 * (src/sf/_device.py:176-178).  out (outer * inner codes), flags (nullable):
 * SFB_F_OVERFLOW where some step saturated; counts->overflow adds those.
 * Computed as an ordered parallel reduction of clamp-add maps, the
 * sequential chain's bits.  inner == 1 with few outputs splits each K
 * across CTAs and needs sfb_reduce_workspace(outer, K) bytes of workspace
 * (0: none). */
SFB_API int64_t sfb_reduce_workspace(int64_t outputs, int64_t K);
SFB_API int sfb_sum(int bits, const int16_t *x, int64_t outer, int64_t K, int64_t inner, int16_t *out,
                    uint8_t *flags, void *workspace, int64_t workspace_bytes, sfb_counts *counts, sfb_stream stream);

/* 1-D dot as the reference's chain of fma (src/sf/_linalg.py:42-58): one
 * code to out[0]; flags[0] (nullable) SFB_F_OVERFLOW / SFB_F_UNDERFLOW;
 * workspace as sfb_reduce_workspace(1, n). */
SFB_API int sfb_dot(int bits, const int16_t *a, const int16_t *b, int64_t n, int16_t *out, uint8_t *flags,
                    void *workspace, int64_t workspace_bytes, sfb_counts *counts, sfb_stream stream);

/* The chip's memory format (src/sf/_vectorized.py:78-89; spec/ops.py,
 * "Memory format"): a 16-bit word with the sign at bit N-1 and |k| in the
 * low N-1 bits; the word with only the sign set reads as 0.
 * sfb_to_bits: codes -> words.  sfb_from_bits: words -> codes, and
 * counts->reserved[2] += the words with bits at or above N (the reference
 * rejects them with ValueError; their codes here are those of the low N
 * bits).  sfb_elementwise_signmag: sfb_elementwise on words in and out, the
 * conversion done in the kernel's loads and stores (no extra pass); words
 * that do not fit are counted the same way (counts is required). */
SFB_API int sfb_to_bits(int bits, const int16_t *codes, uint16_t *out, int64_t n, sfb_stream stream);
SFB_API int sfb_from_bits(int bits, const uint16_t *patterns, int16_t *codes, int64_t n, sfb_counts *counts,
                          sfb_stream stream);
SFB_API int sfb_elementwise_signmag(int op, int bits, const uint16_t *a, const uint16_t *b, const uint16_t *c,
                                    uint16_t *out, uint8_t *flags, int64_t n, int pow_n, sfb_counts *counts,
                                    sfb_stream stream);

/* Exhaustive sweep of every operand pair of one width.  No counterpart in
 * the reference's Device API: the GPU form of its exhaustive check,
 * tools/exhaustive.py:146-181.  For op in SFB_OP_ADD / SUB / MUL / DIV and
 * the rows a = a_lo .. a_hi - 1 (codes, -M <= a_lo <= a_hi <= M + 1), entry
 * a - a_lo of row_digest has ADDED to it
 *     sum over j = 0 .. 2M of  ((code(a, j - M) + M) | flags(a, j - M) << 16) * w_j   (mod 2^32)
 * with w_j = (low 32 bits of splitmix64(j)) | 1 and flags the SFB_F_* bits
 * of that pair; zero the buffer first.  Event totals add into counts.
 * Device buffers. */
SFB_API int sfb_sweep(int op, int bits, int64_t a_lo, int64_t a_hi, uint32_t *row_digest, sfb_counts *counts,
                      sfb_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* SFB200_H */
