// The converted layer's activation scale search on the device, in one
// cooperative launch (src/sf/torch/_core.py:200-236 sanitize / finite_absmax,
// :306-331 the search with headroom="bound"):
//
//   scan:   NaN / inf counts and the largest finite |x| (amax)
//   a0    = amax / m (1 when amax == 0), m = M / 2^(N-1)
//   cast:   codes = cast(x / a) with NaN read as 0 and +-inf as +-amax (the
//           reference's sanitize; +-max / 2^(N-1) when nothing is finite),
//           plus the row L1 / max |code| statistics
//   a     = a_bias when the bias needs more (a_bias > a0), recast
//   loop:   bound = min(rowL1 max|w|, max|x| colL1(w)) // 2^(N-1) + ceil(max(need) / a 2^(N-1))
//           stop when bound <= M, else a *= max(bound / M, 1 + 2^-20) and recast
//
// Every float64 step is the host's (IEEE division, multiplication, ceil),
// so a, the codes and the statistics are the reference's bits.  (max_i
// need_i / a == max_i(need_i) / a: division by a positive number is monotone
// under rounding.  After the bias step the bias term is at most M, so the
// bound is far below 2^53 and converts to float64 exactly.)
//
// Block 0's thread 0 makes each decision between grid-wide barriers
// (cooperative_groups grid.sync(), a cooperative launch with every block
// resident).  The result goes to a device struct the host reads once, after
// the layer's other kernels, which read the scale from it too.
#include <cooperative_groups.h>
#include <math.h>

#include <algorithm>

#include "sfb_common.cuh"

namespace cg = cooperative_groups;

namespace sfb {
namespace {

constexpr int PT = 256;
constexpr int MAX_ITER = 32;

struct Stats {                       // one pass's statistics (device scratch)
    unsigned long long nan_count, inf_count, absmax_bits, over, under, inval;
    long long max_row_l1, max_abs;
};

struct Ctrl {                        // block 0's decision, read by every block after the barrier
    long long done;
    double a_next;
};

constexpr int64_t kScratch = 2 * sizeof(Stats) + sizeof(Ctrl);

template <typename T>
__device__ void scan_pass(const T *__restrict__ x, int64_t R, int64_t K, int64_t ld, Stats *st) {
    unsigned long long nn = 0, ni = 0;
    double mx = 0.0;
    const int64_t total = R * K;
    const bool dense = ld == K;              // rows back to back: no index split per element
    for (int64_t i = (int64_t)blockIdx.x * PT + threadIdx.x; i < total; i += (int64_t)gridDim.x * PT) {
        int64_t at = i;
        if (!dense) {
            const int64_t r = i / K;
            at = r * ld + (i - r * K);
        }
        const double v = (double)x[at];
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
        if (mx > 0.0) atomicMax(&st->absmax_bits, (unsigned long long)__double_as_longlong(mx));
    }
}

// codes of x / a, one warp per row; NaN -> 0, +-inf -> +-big
template <typename T>
__device__ void cast_pass(const T *__restrict__ x, int64_t R, int64_t K, int64_t ld, double a, double big, Width w,
                          int16_t *__restrict__ codes, Stats *st) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * PT + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * PT) >> 5;
    const double thr = 1.0 - ldexp(1.0, -w.bits);
    const double S = (double)(1 << w.sh);
    unsigned long long over = 0, under = 0;
    long long best_l1 = 0;
    int best_abs = 0;
    for (int64_t r = warp; r < R; r += nwarps) {
        long long l1 = 0;
        for (int64_t c = lane; c < K; c += 32) {
            double xv = (double)x[r * ld + c];
            if (isnan(xv)) xv = 0.0;
            else if (isinf(xv)) xv = xv > 0 ? big : -big;
            const double v = xv / a;
            int k;
            if (fabs(v) >= thr) {
                k = v > 0 ? w.M : -w.M;
                over++;
            } else {
                k = (int)rint(v * S);
                under += (k == 0 && v != 0.0);
            }
            codes[r * K + c] = (int16_t)k;
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
        best_abs = max(best_abs, __shfl_xor_sync(0xffffffffu, best_abs, o));
    }
    if (lane == 0) {
        if (over) atomicAdd(&st->over, over);
        if (under) atomicAdd(&st->under, under);
        if (best_l1) atomicMax(&st->max_row_l1, best_l1);
        if (best_abs) atomicMax(&st->max_abs, (long long)best_abs);
    }
}

struct PolicyIn {
    const void *x;
    int64_t R, K, ld;
    Width w;
    long long w_max_abs, w_max_col_l1;
    int has_bias;
    double need_max, a_bias;
    int16_t *codes;
    sfb_scale_result *res;
    Stats *st;                       // 2 entries: the scan, the current cast
    Ctrl *ctrl;
};

template <typename T>
__global__ void __launch_bounds__(PT) policy_kernel(PolicyIn in) {
    cg::grid_group grid = cg::this_grid();
    const T *x = reinterpret_cast<const T *>(in.x);
    const Width w = in.w;
    const double S = (double)(1 << w.sh), m = (double)w.M / S;
    scan_pass<T>(x, in.R, in.K, in.ld, &in.st[0]);
    grid.sync();
    const double amax = __longlong_as_double((long long)in.st[0].absmax_bits);
    const bool any_inf = in.st[0].inf_count != 0;
    const double big = (any_inf && amax == 0.0) ? m : amax;       // the sanitized inf's magnitude
    const double fin = any_inf ? fmax(amax, big) : amax;         // finite_absmax of the sanitized x
    const double a0 = fin > 0.0 ? fin / m : 1.0;
    double a = a0;
    if (in.has_bias && isfinite(in.a_bias) && in.a_bias > a) a = in.a_bias;
    for (int it = 0; it < MAX_ITER; it++) {
        cast_pass<T>(x, in.R, in.K, in.ld, a, big, w, in.codes, &in.st[1]);
        grid.sync();
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            const Stats s = in.st[1];
            double ratio = 0.0;
            if (in.has_bias) ratio = in.need_max / a * S;
            const double bias_codes = isfinite(ratio) ? ceil(ratio) : 0.0;
            long long chain = 0;
            if (in.R > 0 && in.K > 0) {
                const long long r1 = s.max_row_l1 * in.w_max_abs, r2 = s.max_abs * in.w_max_col_l1;
                chain = (r1 < r2 ? r1 : r2) / (long long)S;
            }
            const double bound = (double)chain + bias_codes;
            long long done = 0;
            if (bound <= (double)w.M) {
                done = 1;
                in.res->a = a;
                in.res->a0 = a0;
                in.res->proven = chain <= w.M;
                in.res->iterations = it;
                in.res->nan_count = (long long)in.st[0].nan_count;
                in.res->inf_count = (long long)in.st[0].inf_count;
                in.res->underflow = (long long)s.under;
                in.res->err = 0;
            } else if (it == MAX_ITER - 1) {
                done = 1;
                in.res->err = 1;                                   // did not converge, as the host raises
            } else {
                const double f = bound / (double)w.M;
                a *= f > 1.0 + 0x1p-20 ? f : 1.0 + 0x1p-20;
                in.st[1] = Stats{0, 0, 0, 0, 0, 0, 0, 0};          // the next cast's statistics
            }
            in.ctrl->done = done;
            in.ctrl->a_next = a;
        }
        grid.sync();
        if (*(volatile long long *)&in.ctrl->done) break;
        a = *(volatile double *)&in.ctrl->a_next;
    }
}

}  // namespace
}  // namespace sfb

extern "C" int sfb_linear_scale(const void *x, int dtype, int64_t R, int64_t K, int64_t ld, int bits,
                                int64_t w_max_abs, int64_t w_max_col_l1, int has_bias, double need_max,
                                double a_bias, int16_t *codes, sfb_scale_result *result, void *scratch,
                                sfb_stream stream) {
    using namespace sfb;
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "sfb_linear_scale: width %d is not 4..16", bits);
    if (R < 0 || K < 0 || (K > 0 && ld < K)) return set_error(SFB_EINVAL, "sfb_linear_scale: bad shape");
    if (result == nullptr || scratch == nullptr || (R * K > 0 && (x == nullptr || codes == nullptr)))
        return set_error(SFB_EINVAL, "sfb_linear_scale: null argument");
    if (dtype != SFB_F32 && dtype != SFB_F64)
        return set_error(SFB_EINVAL, "sfb_linear_scale: dtype %d is not SFB_F32 / SFB_F64", dtype);
    cudaStream_t st = (cudaStream_t)stream;
    if (cudaMemsetAsync(scratch, 0, kScratch, st) != cudaSuccess ||
        cudaMemsetAsync(result, 0, sizeof(sfb_scale_result), st) != cudaSuccess)
        return check_launch("sfb_linear_scale (reset)");
    PolicyIn in;
    in.x = x;
    in.R = R;
    in.K = K;
    in.ld = ld;
    in.w = width(bits);
    in.w_max_abs = w_max_abs;
    in.w_max_col_l1 = w_max_col_l1;
    in.has_bias = has_bias;
    in.need_max = need_max;
    in.a_bias = a_bias;
    in.codes = codes;
    in.res = result;
    in.st = reinterpret_cast<Stats *>(scratch);
    in.ctrl = reinterpret_cast<Ctrl *>(in.st + 2);
    void *kern = dtype == SFB_F32 ? (void *)policy_kernel<float> : (void *)policy_kernel<double>;
    static int per_sm[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    int &nb = per_sm[dev][dtype == SFB_F32 ? 0 : 1];
    if (nb == 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, PT, 0) != cudaSuccess || nb < 1)
            return set_error(SFB_ECUDA, "sfb_linear_scale: occupancy query failed");
    }
    const int64_t want = std::max<int64_t>(1, (R + (PT / 32) - 1) / (PT / 32));          // a warp per row
    const int grid = (int)std::min<int64_t>(want, (int64_t)sm_count() * nb);
    void *args[] = {&in};
    if (cudaLaunchCooperativeKernel(kern, dim3(grid), dim3(PT), args, 0, st) != cudaSuccess)
        return check_launch("sfb_linear_scale");
    return check_launch("sfb_linear_scale");
}

extern "C" int64_t sfb_linear_scale_scratch(void) { return sfb::kScratch; }
