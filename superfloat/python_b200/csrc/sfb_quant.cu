// Quantization of float tensors to sfN codes with the statistics the scale
// policy of a converted layer needs, in one pass each.
//
// sfb_scan: NaN count, +-inf count and the largest finite |x| (the inputs of
// the reference's sanitize and finite_absmax, src/sf/torch/_core.py:200-236).
// sfb_quantize: codes = cast(x / scale) per row (one scale, or one per row),
// the cast rule of src/sf/_vectorized.py:32-71 on float64 values: NaN -> 0
// (invalid), |v| >= 1 - 2^-N -> +-M (overflow), else round half to even of
// v 2^(N-1), underflow where a nonzero value rounds to 0; plus the event
// counts, the largest row L1 norm sum_k |code| and the largest |code| (the
// operands of the L1 bound, src/sf/_linalg.py:84-106).  Every division is
// IEEE double, as in NumPy, so the codes are the reference's bit for bit.
#include <math.h>

#include "sfb_common.cuh"

namespace sfb {
namespace {

constexpr int QT = 256;

template <typename T>
__device__ __forceinline__ double to_d(T v) { return (double)v; }

template <typename T>
__global__ void __launch_bounds__(QT) scan_kernel(const T *__restrict__ x, int64_t n, sfb_qstats *st) {
    unsigned long long nn = 0, ni = 0;
    double mx = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * QT + threadIdx.x; i < n; i += (int64_t)gridDim.x * QT) {
        const double v = to_d(x[i]);
        if (isnan(v)) nn++;
        else if (isinf(v)) ni++;
        else mx = fmax(mx, fabs(v));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        nn += __shfl_xor_sync(0xffffffffu, nn, o);
        ni += __shfl_xor_sync(0xffffffffu, ni, o);
        mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if ((threadIdx.x & 31) == 0) {
        if (nn) atomicAdd(&st->nan_count, nn);
        if (ni) atomicAdd(&st->inf_count, ni);
        // non-negative doubles order like their bit patterns
        if (mx > 0.0) atomicMax(reinterpret_cast<unsigned long long *>(&st->absmax),
                                (unsigned long long)__double_as_longlong(mx));
    }
}

// one warp per row (grid-stride over rows)
template <typename T>
__global__ void __launch_bounds__(QT) quant_kernel(const T *__restrict__ x, int64_t rows, int64_t cols, int64_t ld,
                                                   double scale, const double *__restrict__ row_scale, Width w,
                                                   int16_t *__restrict__ codes, int64_t ldc, sfb_qstats *st,
                                                   const sfb_qstats *__restrict__ scan, double m) {
    const int lane = threadIdx.x & 31;
    if (scan) {                                  // the scale a0 = max|x| / m from a scan pass (1 when all 0)
        const double amax = scan->absmax;
        scale = amax > 0.0 ? amax / m : 1.0;
    }
    const int64_t warp = ((int64_t)blockIdx.x * QT + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * QT) >> 5;
    const double thr = 1.0 - ldexp(1.0, -w.bits);
    const double S = (double)(1 << w.sh);
    unsigned long long over = 0, under = 0, inval = 0;
    long long best_l1 = 0;
    int best_abs = 0;
    for (int64_t r = warp; r < rows; r += nwarps) {
        const double sc = row_scale ? row_scale[r] : scale;
        long long l1 = 0;
        for (int64_t c = lane; c < cols; c += 32) {
            const double v = to_d(x[r * ld + c]) / sc;
            int k;
            if (isnan(v)) {
                k = 0;
                inval++;
            } else if (fabs(v) >= thr) {
                k = v > 0 ? w.M : -w.M;
                over++;
            } else {
                k = (int)rint(v * S);
                under += (k == 0 && v != 0.0);
            }
            codes[r * ldc + c] = (int16_t)k;
            l1 += abs(k);
            best_abs = max(best_abs, abs(k));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) l1 += __shfl_xor_sync(0xffffffffu, l1, o);
        best_l1 = max(best_l1, l1);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        over += __shfl_xor_sync(0xffffffffu, over, o);
        under += __shfl_xor_sync(0xffffffffu, under, o);
        inval += __shfl_xor_sync(0xffffffffu, inval, o);
        best_abs = max(best_abs, __shfl_xor_sync(0xffffffffu, best_abs, o));
    }
    if (lane == 0) {
        if (over) atomicAdd(&st->overflow, over);
        if (under) atomicAdd(&st->underflow, under);
        if (inval) atomicAdd(&st->invalid, inval);
        if (best_l1) atomicMax(&st->max_row_l1, best_l1);
        if (best_abs) atomicMax(&st->max_abs_code, (long long)best_abs);
    }
}

// bias codes at the layer's scale: cast(b[n] / (a s[n])), a from device memory
__global__ void __launch_bounds__(QT) bias_codes_kernel(const double *__restrict__ b, const double *__restrict__ a_dev,
                                                        const double *__restrict__ s_col, int64_t n, Width w,
                                                        int16_t *__restrict__ codes, long long *n_over) {
    const double a = *a_dev;
    const double thr = 1.0 - ldexp(1.0, -w.bits);
    const double S = (double)(1 << w.sh);
    unsigned long long over = 0;
    for (int64_t i = (int64_t)blockIdx.x * QT + threadIdx.x; i < n; i += (int64_t)gridDim.x * QT) {
        const double v = b[i] / (a * s_col[i]);
        int k;
        if (isnan(v)) {
            k = 0;
        } else if (fabs(v) >= thr) {
            k = v > 0 ? w.M : -w.M;
            over++;
        } else {
            k = (int)rint(v * S);
        }
        codes[i] = (int16_t)k;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) over += __shfl_xor_sync(0xffffffffu, over, o);
    if ((threadIdx.x & 31) == 0 && over) atomicAdd(reinterpret_cast<unsigned long long *>(n_over), over);
}

int grid_for(int64_t work) {
    const int64_t cap = (int64_t)sm_count() * (2048 / QT);
    int64_t g = (work + QT - 1) / QT;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace
}  // namespace sfb

extern "C" int sfb_scan(const void *x, int dtype, int64_t n, sfb_qstats *stats, sfb_stream stream) {
    using namespace sfb;
    if (n < 0 || (n > 0 && x == nullptr) || stats == nullptr) return set_error(SFB_EINVAL, "sfb_scan: bad argument");
    if (n == 0) return SFB_OK;
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == SFB_F32)
        scan_kernel<float><<<grid_for(n), QT, 0, st>>>((const float *)x, n, stats);
    else if (dtype == SFB_F64)
        scan_kernel<double><<<grid_for(n), QT, 0, st>>>((const double *)x, n, stats);
    else
        return set_error(SFB_EINVAL, "sfb_scan: dtype %d is not SFB_F32 / SFB_F64", dtype);
    return check_launch("sfb_scan");
}

extern "C" int sfb_quantize(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, double scale,
                            const double *row_scale, int bits, int16_t *codes, int64_t ldc, sfb_qstats *stats,
                            sfb_stream stream) {
    using namespace sfb;
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "sfb_quantize: width %d is not 4..16", bits);
    if (rows < 0 || cols < 0 || stats == nullptr) return set_error(SFB_EINVAL, "sfb_quantize: bad shape or null stats");
    if (rows == 0 || cols == 0) return SFB_OK;   // an empty view may carry any strides
    if (ld < cols || ldc < cols) return set_error(SFB_EINVAL, "sfb_quantize: ld %lld or ldc %lld below cols %lld",
                                                   (long long)ld, (long long)ldc, (long long)cols);
    if (x == nullptr || codes == nullptr) return set_error(SFB_EINVAL, "sfb_quantize: null buffer");
    if (row_scale == nullptr && !(scale > 0.0)) return set_error(SFB_EINVAL, "sfb_quantize: scale must be > 0");
    cudaStream_t st = (cudaStream_t)stream;
    const Width w = width(bits);
    const int g = grid_for(rows * 32);
    if (dtype == SFB_F32)
        quant_kernel<float><<<g, QT, 0, st>>>((const float *)x, rows, cols, ld, scale, row_scale, w, codes, ldc, stats,
                                              nullptr, 0.0);
    else if (dtype == SFB_F64)
        quant_kernel<double><<<g, QT, 0, st>>>((const double *)x, rows, cols, ld, scale, row_scale, w, codes, ldc,
                                               stats, nullptr, 0.0);
    else
        return set_error(SFB_EINVAL, "sfb_quantize: dtype %d is not SFB_F32 / SFB_F64", dtype);
    return check_launch("sfb_quantize");
}

extern "C" int sfb_quantize_auto(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                 const sfb_qstats *scan, double m, int bits, int16_t *codes, int64_t ldc,
                                 sfb_qstats *stats, sfb_stream stream) {
    using namespace sfb;
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "sfb_quantize_auto: width %d is not 4..16", bits);
    if (rows < 0 || cols < 0 || stats == nullptr || scan == nullptr || !(m > 0.0))
        return set_error(SFB_EINVAL, "sfb_quantize_auto: bad shape, null statistics or m <= 0");
    if (rows == 0 || cols == 0) return SFB_OK;
    if (ld < cols || ldc < cols) return set_error(SFB_EINVAL, "sfb_quantize_auto: ld or ldc below cols");
    if (x == nullptr || codes == nullptr) return set_error(SFB_EINVAL, "sfb_quantize_auto: null buffer");
    cudaStream_t st = (cudaStream_t)stream;
    const Width w = width(bits);
    const int g = grid_for(rows * 32);
    if (dtype == SFB_F32)
        quant_kernel<float><<<g, QT, 0, st>>>((const float *)x, rows, cols, ld, 1.0, nullptr, w, codes, ldc, stats,
                                              scan, m);
    else if (dtype == SFB_F64)
        quant_kernel<double><<<g, QT, 0, st>>>((const double *)x, rows, cols, ld, 1.0, nullptr, w, codes, ldc, stats,
                                               scan, m);
    else
        return set_error(SFB_EINVAL, "sfb_quantize_auto: dtype %d is not SFB_F32 / SFB_F64", dtype);
    return check_launch("sfb_quantize_auto");
}

extern "C" int sfb_bias_codes(int bits, const double *b, const double *a_dev, const double *s_col, int64_t n,
                              int16_t *codes, int64_t *n_over, sfb_stream stream) {
    using namespace sfb;
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "sfb_bias_codes: width %d is not 4..16", bits);
    if (n < 0) return set_error(SFB_EINVAL, "sfb_bias_codes: negative length");
    if (n == 0) return SFB_OK;
    if (b == nullptr || a_dev == nullptr || s_col == nullptr || codes == nullptr || n_over == nullptr)
        return set_error(SFB_EINVAL, "sfb_bias_codes: null argument");
    bias_codes_kernel<<<grid_for(n), QT, 0, (cudaStream_t)stream>>>(b, a_dev, s_col, n, width(bits), codes,
                                                                     reinterpret_cast<long long *>(n_over));
    return check_launch("sfb_bias_codes");
}
