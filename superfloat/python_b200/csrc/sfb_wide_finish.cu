// The wide sft linear's step after accumulation, per output (the reference's
// host runner, src/sf/torch/_core.py:68-98 with :162-190, and the shift rule
// of src/sf/_heuristic.py:123-169):
//
//   rule:  prod  = |a_m|_2 |b_n|_2 (dequantized norms),  l2 = pow2_exp(prod)
//          target = l2 - h, raised to pow2_exp(|bias_n|) when the bias is nonzero
//          shift  = clamp(e_m + e_n - target, -32, 31)
//          redo   = clamp(e_m + e_n - pow2_exp(prod + |bias_n|), -32, 31)
//   POP of the accumulator at shift (round half to even, saturate at M);
//   with a bias, its code at the output's exponent fe = e_m + e_n - shift,
//   rint(b 2^(N-1-fe)) clamped to +-M, added with the saturating sfN add;
//   an output whose POP code or sum reached +-M, or whose bias code was
//   clamped, and whose accumulator or bias code is nonzero, is popped again
//   at the redo shift (the rule only; an explicit shift is never redone);
//   y = code 2^(fe - (N-1)) in float64, rounded once to float32 if asked.
//
// pow2_exp(m) is the smallest e with m / 2^e < 1 (frexp's exponent), 0 for
// m == 0.  Every float64 step (the product, the sum, ldexp, rint) is IEEE and
// exact or correctly rounded as in NumPy, so the bits are the reference's.
// One thread per output, grid-stride; counts and the shift range reduced per
// warp, one atomic per warp.
#include <math.h>

#include "sfb_wide_simt.cuh"

namespace sfb {
namespace {

constexpr int FT = 256;

__device__ __forceinline__ int pow2_exp(double m) {
    int e = 0;
    if (m > 0.0) frexp(m, &e);
    return e;
}

__device__ __forceinline__ int clamp_shift(int s) { return s < -32 ? -32 : (s > 31 ? 31 : s); }

struct Post {
    int y;            // the code after the bias add
    int q;            // the POP code
    bool over, under, add_sat, nz, clamped;
};

__device__ __forceinline__ Post post(long long acc, int sh, int base, bool has_bias, double b, int F, Width w) {
    Post p;
    p.q = mx_pop(acc, sh, F, w, p.over, p.under);
    p.y = p.q;
    p.add_sat = false;
    p.clamped = false;
    p.nz = acc != 0;
    if (has_bias) {
        const int fe = base - sh;
        const double raw = rint(ldexp(b, w.sh - fe));
        p.clamped = fabs(raw) > (double)w.M;
        const int bq = p.clamped ? (raw > 0.0 ? w.M : -w.M) : (int)raw;
        const int s = p.q + bq;
        const bool sat = s > w.M || s < -w.M;
        p.y = sat ? (s > 0 ? w.M : -w.M) : s;
        p.add_sat = sat || p.clamped;
        p.nz = p.nz || bq != 0;
    }
    return p;
}

struct FinishIn {
    const int32_t *acc;
    int64_t M, N;
    const int32_t *ea, *eb;
    const double *na, *nb;
    int h, rule, shift;
    const double *bias;
    float *y32;
    double *y64;
    uint8_t *flags;
    long long *stats;      // redone, bias_saturated, min shift, max shift
    Width w;
    int F;
    sfb_counts *counts;
};

__global__ void __launch_bounds__(FT) wide_finish_kernel(FinishIn in) {
    const Width w = in.w;
    const int64_t total = in.M * in.N;
    unsigned n_sat = 0, n_flush = 0, n_redo = 0, n_bsat = 0;
    int smin = 127, smax = -128;
    for (int64_t i = (int64_t)blockIdx.x * FT + threadIdx.x; i < total; i += (int64_t)gridDim.x * FT) {
        const int64_t m = i / in.N, n = i - m * in.N;
        const long long acc = in.acc[i];
        const int base = in.ea[m] + in.eb[n];
        const bool has_bias = in.bias != nullptr;
        const double b = has_bias ? in.bias[n] : 0.0;
        int sh = in.shift, shr = 0;
        if (in.rule) {
            const double prod = in.na[m] * in.nb[n];
            const int l2 = pow2_exp(prod);
            int target = l2 - in.h;
            if (has_bias && fabs(b) > 0.0) target = max(target, pow2_exp(fabs(b)));
            sh = clamp_shift(base - target);
            shr = clamp_shift(base - (has_bias ? pow2_exp(prod + fabs(b)) : l2));
        }
        Post p = post(acc, sh, base, has_bias, b, in.F, w);
        int used = sh;
        bool redo = false;
        if (in.rule) {
            redo = (abs(p.q) >= w.M || abs(p.y) >= w.M || p.add_sat) && p.nz;
            if (redo) {
                p = post(acc, shr, base, has_bias, b, in.F, w);
                used = shr;
            }
        }
        const bool sat = p.over || p.add_sat;
        const double y = ldexp((double)p.y, base - used - w.sh);
        if (in.y64) in.y64[i] = y;
        if (in.y32) in.y32[i] = (float)y;
        if (in.flags) in.flags[i] = (uint8_t)((sat ? SFB_F_OVERFLOW : 0u) | (p.under ? SFB_F_UNDERFLOW : 0u));
        n_sat += sat;
        n_flush += p.under;
        n_redo += redo;
        n_bsat += p.clamped;
        smin = min(smin, used);
        smax = max(smax, used);
    }
    n_sat = __reduce_add_sync(0xffffffffu, n_sat);
    n_flush = __reduce_add_sync(0xffffffffu, n_flush);
    n_redo = __reduce_add_sync(0xffffffffu, n_redo);
    n_bsat = __reduce_add_sync(0xffffffffu, n_bsat);
    smin = __reduce_min_sync(0xffffffffu, smin);
    smax = __reduce_max_sync(0xffffffffu, smax);
    if ((threadIdx.x & 31) == 0) {
        if (n_sat) atomicAdd(&in.counts->overflow, (unsigned long long)n_sat);
        if (n_flush) atomicAdd(&in.counts->underflow, (unsigned long long)n_flush);
        if (n_redo) atomicAdd(reinterpret_cast<unsigned long long *>(&in.stats[0]), (unsigned long long)n_redo);
        if (n_bsat) atomicAdd(reinterpret_cast<unsigned long long *>(&in.stats[1]), (unsigned long long)n_bsat);
        if (smin <= smax) {
            atomicMin(&in.stats[2], (long long)smin);
            atomicMax(&in.stats[3], (long long)smax);
        }
    }
}

}  // namespace
}  // namespace sfb

extern "C" int sfb_wide_finish(int bits, int mx, const int32_t *acc, int64_t M, int64_t N, const int32_t *row_exp,
                               const int32_t *col_exp, const double *row_norm, const double *col_norm, int h,
                               int use_rule, int shift, const double *bias, float *y32, double *y64, uint8_t *flags,
                               int64_t *stats, sfb_counts *counts, sfb_stream stream) {
    using namespace sfb;
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "sfb_wide_finish: width %d is not 4..16", bits);
    if (mx != SFB_MX_V492 && mx != SFB_MX_V481) return set_error(SFB_EINVAL, "sfb_wide_finish: unknown mx %d", mx);
    if (M < 0 || N < 0) return set_error(SFB_EINVAL, "sfb_wide_finish: negative size");
    if (!use_rule && (shift < -32 || shift > 31))
        return set_error(SFB_EINVAL, "sfb_wide_finish: shift %d is not in -32..31", shift);
    if (M == 0 || N == 0) return SFB_OK;
    if (acc == nullptr || row_exp == nullptr || col_exp == nullptr || stats == nullptr || counts == nullptr ||
        (use_rule && (row_norm == nullptr || col_norm == nullptr)) || (y32 == nullptr && y64 == nullptr))
        return set_error(SFB_EINVAL, "sfb_wide_finish: null argument");
    FinishIn in;
    in.acc = acc;
    in.M = M;
    in.N = N;
    in.ea = row_exp;
    in.eb = col_exp;
    in.na = row_norm;
    in.nb = col_norm;
    in.h = h;
    in.rule = use_rule != 0;
    in.shift = shift;
    in.bias = bias;
    in.y32 = y32;
    in.y64 = y64;
    in.flags = flags;
    in.stats = reinterpret_cast<long long *>(stats);
    in.w = width(bits);
    in.F = mx_unit(mx, bits >= 9).F;
    in.counts = counts;
    const int64_t want = (M * N + FT - 1) / FT;
    const int64_t cap = (int64_t)sm_count() * 8;
    const int grid = (int)(want < cap ? (want < 1 ? 1 : want) : cap);
    wide_finish_kernel<<<grid, FT, 0, (cudaStream_t)stream>>>(in);
    return check_launch("sfb_wide_finish");
}
