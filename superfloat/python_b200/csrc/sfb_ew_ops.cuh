// Per-element sfN arithmetic shared by the elementwise and sweep kernels:
// one output code and the events it raised.
//
// Semantics follow the reference's vectorised ops (src/sf/_vectorized.py:94-156):
//   add/sub  clip(a +- b, +-M), overflow where |a +- b| > M          (:94-99, :25-27)
//   mul      trunc(a b / S), underflow where a b != 0 truncates to 0  (:110-113)
//   div      b == 0: sign(a) M, divide; a != 0, |a| >= |b|: +-M, overflow;
//            else trunc(a S / b)                                      (:116-125)
//   fma      add(mul(a, b), c); underflow only where the add did not overflow (:128-131)
//   neg/abs  exact                                                    (:102-107)
//   sqrt     floor(sqrt(a S)), a < 0 -> 0 and invalid                 (:134-142)
//   pow      chain of mul, underflow if any step underflowed          (:145-156)
#pragma once
#include <math.h>

#include "sfb_common.cuh"

namespace sfb {
namespace ewops {

// Events one output raised; each op sets only the ones it can raise, so the
// compiler drops the others from the tally.
struct Ev {
    bool over = false, under = false, div0 = false, inval = false;
    // div only: both events in one word, 0x10000 for a divide, else 1 for
    // an overflow (a kernel that only counts adds these and splits the sum)
    unsigned pk = 0;
};

// Width constants, folded at compile time for BITS != 0 (the sf16 kernels).
template <int BITS>
__device__ __forceinline__ Width wfix(Width w) {
    if constexpr (BITS != 0) return Width{BITS, BITS - 1, (1 << (BITS - 1)) - 1};
    return w;
}

// 0 < |p| < 2^sh: a nonzero product that truncates to 0.
__device__ __forceinline__ bool small_nonzero(int p, int sh) {
    return (unsigned)(p + ((1 << sh) - 1)) <= (unsigned)((2 << sh) - 2) && p != 0;
}

template <int OP, int BITS>
__device__ __forceinline__ int ew_one(int a, int b, int c, Width w0, int pow_n, Ev &ev) {
    const Width w = wfix<BITS>(w0);
    const int M = w.M, sh = w.sh;
    if constexpr (OP == SFB_OP_ADD || OP == SFB_OP_SUB) {
        const int s = (OP == SFB_OP_ADD) ? a + b : a - b;
        const int r = clampi(s, -M, M);
        ev.over = r != s;
        return r;
    } else if constexpr (OP == SFB_OP_MUL) {
        const int p = a * b;
        ev.under = small_nonzero(p, sh);
        return tdiv_pow2(p, sh);
    } else if constexpr (OP == SFB_OP_FMA) {
        // a product that truncates to 0 leaves c unchanged and in range, so
        // the fma's underflow needs no "and not overflow" term
        const int p = a * b;
        const int s = tdiv_pow2(p, sh) + c;
        const int r = clampi(s, -M, M);
        ev.over = r != s;
        ev.under = small_nonzero(p, sh);
        return r;
    } else if constexpr (OP == SFB_OP_DIV) {
        // One quotient path for every case, mostly on the FMA and XU pipes.  The
        // operands as float32 (exact), d = max(|b|, 1), x = min(|a|, d): the
        // quotient q = floor(x 2^sh / d) is at most 2^sh, reached exactly when
        // |a| >= |b| > 0 (overflow) or b == 0 with a != 0 (divide); min(q, M)
        // with the sign of a b then gives +-M there, 0 for 0 / 0, and
        // trunc(a S / b) everywhere else.
        // With dp = d 2^-sh (exact), rcp.approx(dp) is 2^sh / d to a relative
        // error below 2^-22, so x rcp(dp) is within 2^15 2^-22 < 0.01 of the
        // quotient; the 1.5 2^23 bias rounds it to the nearest integer q0
        // (floor or floor + 1), and the sign of x - q0 dp = (x 2^sh - q0 d) 2^-sh
        // tells which.  One fused multiply-add gives that remainder exactly
        // (an integer below 2^16 in magnitude times 2^-sh).
        const float fa = (float)a, fb = (float)b;
        const float fd = fmaxf(fabsf(fb), 1.0f), fx = fminf(fabsf(fa), fd);
        const float fdp = fd * __int_as_float((127 - sh) << 23);           // d 2^-sh, exact
        float r;
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(fdp));
        const float qb = fmaf(fx, r, 12582912.0f);
        const int q0 = __float_as_int(qb) - 0x4B400000;
        const float rem = fmaf(-(qb - 12582912.0f), fdp, fx);
        const int q = q0 + (__float_as_int(rem) >> 31);                    // q0 - 1 when rem < 0
        const int m = min(q, M);
        // b == 0 and the quotient's sign read from the float copies, so the
        // integer codes are only ever converted
        const bool bz = fb == 0.0f;
        ev.over = (q >> sh) != 0 && !bz;
        ev.div0 = bz;
        ev.pk = bz ? 0x10000u : (unsigned)(q >> sh);   // q >> sh is the overflow where b != 0
        return (__float_as_int(fa) ^ __float_as_int(fb)) < 0 ? -m : m;
    } else if constexpr (OP == SFB_OP_NEG) {
        return -a;
    } else if constexpr (OP == SFB_OP_ABS) {
        return abs(a);
    } else if constexpr (OP == SFB_OP_SQRT) {
        ev.inval = a < 0;
        const int x = max(a, 0) << sh;      // < 2^30
        int r = (int)sqrtf((float)x);       // within 1 of floor(sqrt(x)) for x < 2^30
        r -= (r * r > x);
        r += ((r + 1) * (r + 1) <= x);
        return r;
    } else {  // SFB_OP_POW
        int k = a;
        bool un = false;
        for (int i = 1; i < pow_n; i++) {
            const int p = k * a;
            un |= small_nonzero(p, sh);
            k = tdiv_pow2(p, sh);
        }
        ev.under = un;
        return k;
    }
}

__device__ __forceinline__ void tally(Counts &c, const Ev &e) {
    c.over += e.over;
    c.under += e.under;
    c.div0 += e.div0;
    c.inval += e.inval;
}

__device__ __forceinline__ unsigned flag_byte(const Ev &e) {
    return (e.over ? SFB_F_OVERFLOW : 0u) | (e.under ? SFB_F_UNDERFLOW : 0u) | (e.div0 ? SFB_F_DIVIDE : 0u) |
           (e.inval ? SFB_F_INVALID : 0u);
}

// The chip's memory format (src/sf/_vectorized.py:78-89): a 16-bit word
// with the sign at bit N-1 and |k| in the low N-1 bits; the pattern with
// only the sign set reads as 0.  A pattern with bits at or above N does not
// fit the width (``bad``).
__device__ __forceinline__ int sm_to_code(unsigned p, Width w, bool &bad) {
    bad = (p >> w.bits) != 0;
    const int mag = (int)(p & (unsigned)w.M);
    return ((p >> w.sh) & 1u) ? -mag : mag;
}

__device__ __forceinline__ unsigned code_to_sm(int k, Width w) {
    return k < 0 ? ((1u << w.sh) | (unsigned)(-k)) : (unsigned)k;
}

}  // namespace ewops
}  // namespace sfb
