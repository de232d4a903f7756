// Elementwise sfN ops with per-output events, HBM-streaming on sm_100a.
//
// The per-element arithmetic (the reference's vectorised ops,
// src/sf/_vectorized.py:94-156) lives in sfb_ew_ops.cuh.
//
// Layout: int16 codes, 8 per 128-bit vector.  Each thread streams pairs of
// vectors (grid-stride, grid = SMs x resident blocks), counts events in
// registers and flushes them once per block (warp reduce + one atomic per
// counter).  Optional per-output event bytes are written 8 at a time.  The
// sf16 kernels are compiled with the width's shifts and bounds as constants;
// other widths take them at run time.
#include <math.h>

#include <algorithm>

#include "sfb_common.cuh"
#include "sfb_ew_ops.cuh"

namespace sfb {
namespace {

using namespace ewops;

constexpr int kThreads = 256;

union Vec8 {
    uint4 u;
    int16_t h[8];
};

// SM: operands and result in the chip's sign-magnitude words, converted at
// the loads and stores; patterns that do not fit the width are counted into
// counts->reserved[2].
template <int OP, int BITS, bool FLAGS, bool SM>
__global__ void __launch_bounds__(kThreads) ew_kernel(const int16_t *__restrict__ a, const int16_t *__restrict__ b,
                                                     const int16_t *__restrict__ c, int16_t *__restrict__ out,
                                                     uint8_t *__restrict__ flags, int64_t n, Width w, int pow_n,
                                                     int vec_ok, sfb_counts *counts) {
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    Counts cnt;
    constexpr bool kB = OP == SFB_OP_ADD || OP == SFB_OP_SUB || OP == SFB_OP_MUL || OP == SFB_OP_DIV ||
                        OP == SFB_OP_FMA;
    constexpr bool kC = OP == SFB_OP_FMA;
    constexpr bool kPacked = OP == SFB_OP_DIV && !FLAGS && !SM;   // div's two counts in one word
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t done = 0;
    unsigned bad = 0;
    const Width wf = wfix<BITS>(w);
    // one element: operands in (codes, or sign-magnitude words when SM), result out
    auto one = [&](int x, int y, int z, Ev &ev) -> int {
        if constexpr (SM) {
            bool b0, b1 = false, b2 = false;
            x = sm_to_code((unsigned)(uint16_t)x, wf, b0);
            if constexpr (kB) y = sm_to_code((unsigned)(uint16_t)y, wf, b1);
            if constexpr (kC) z = sm_to_code((unsigned)(uint16_t)z, wf, b2);
            bad += b0 + b1 + b2;
            return (int)code_to_sm(ew_one<OP, BITS>(x, y, z, w, pow_n, ev), wf);
        } else {
            return ew_one<OP, BITS>(x, y, z, w, pow_n, ev);
        }
    };
    if (vec_ok) {
        // two vectors per thread per iteration, loads issued before any math,
        // so each thread keeps up to 6 x 16 B in flight
        const int64_t nv = n >> 3;
        for (int64_t v = tid; v < nv; v += 2 * stride) {
            const int64_t v2 = v + stride;
            const bool has2 = v2 < nv;
            Vec8 va[2], vb[2], vc[2], vo[2];
            va[0].u = __ldcs(reinterpret_cast<const uint4 *>(a) + v);
            if constexpr (kB) vb[0].u = __ldcs(reinterpret_cast<const uint4 *>(b) + v);
            if constexpr (kC) vc[0].u = __ldcs(reinterpret_cast<const uint4 *>(c) + v);
            if (has2) {
                va[1].u = __ldcs(reinterpret_cast<const uint4 *>(a) + v2);
                if constexpr (kB) vb[1].u = __ldcs(reinterpret_cast<const uint4 *>(b) + v2);
                if constexpr (kC) vc[1].u = __ldcs(reinterpret_cast<const uint4 *>(c) + v2);
            } else {
                va[1].u = make_uint4(0, 0, 0, 0);
                vb[1].u = va[1].u;
                vc[1].u = va[1].u;
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                if (h == 1 && !has2) break;
                uint64_t fb = 0;
                unsigned pk = 0;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    Ev ev;
                    vo[h].h[j] = (int16_t)one(va[h].h[j], kB ? vb[h].h[j] : 0, kC ? vc[h].h[j] : 0, ev);
                    if constexpr (kPacked) {
                        pk += ev.pk;
                    } else {
                        tally(cnt, ev);
                    }
                    if constexpr (FLAGS) fb |= (uint64_t)flag_byte(ev) << (8 * j);
                }
                if constexpr (kPacked) {
                    cnt.over += pk & 0xFFFFu;
                    cnt.div0 += pk >> 16;
                }
                const int64_t vv = h ? v2 : v;
                __stcs(reinterpret_cast<uint4 *>(out) + vv, vo[h].u);
                if constexpr (FLAGS) __stcs(reinterpret_cast<unsigned long long *>(flags) + vv, (unsigned long long)fb);
            }
        }
        done = nv << 3;
    }
    for (int64_t i = done + tid; i < n; i += stride) {
        Ev ev;
        out[i] = (int16_t)one(a[i], kB ? b[i] : 0, kC ? c[i] : 0, ev);
        tally(cnt, ev);
        if constexpr (FLAGS) flags[i] = (uint8_t)flag_byte(ev);
    }
    if constexpr (SM) {
        bad = __reduce_add_sync(0xffffffffu, bad);
        if ((threadIdx.x & 31) == 0 && bad && counts) atomicAdd(&counts->reserved[2], (unsigned long long)bad);
    }
    flush_counts(cnt, counts, sc);
}

template <typename K>
int resident_blocks(K kernel) {
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, kThreads, 0) != cudaSuccess || nb < 1) nb = 1;
    return nb;
}

template <int OP, int BITS, bool FLAGS, bool SM>
int launch_one(const int16_t *a, const int16_t *b, const int16_t *c, int16_t *out, uint8_t *flags, int64_t n,
               Width w, int pow_n, bool vec_ok, sfb_counts *counts, cudaStream_t st) {
    auto kern = ew_kernel<OP, BITS, FLAGS, SM>;
    static const int per_sm = resident_blocks(kern);   // grid = SMs x resident blocks
    const int64_t work = vec_ok ? (n >> 4) + 1 : n;
    const int64_t max_blocks = (int64_t)sm_count() * per_sm;
    int blocks = (int)std::min<int64_t>(max_blocks, (work + kThreads - 1) / kThreads);
    if (blocks < 1) blocks = 1;
    kern<<<blocks, kThreads, 0, st>>>(a, b, c, out, flags, n, w, pow_n, vec_ok, counts);
    return check_launch("sfb_elementwise");
}

template <int OP, bool SM>
int launch(const int16_t *a, const int16_t *b, const int16_t *c, int16_t *out, uint8_t *flags, int64_t n,
           Width w, int pow_n, sfb_counts *counts, cudaStream_t st) {
    const bool vec_ok = ((uintptr_t)a % 16 == 0) && (b == nullptr || (uintptr_t)b % 16 == 0) &&
                        (c == nullptr || (uintptr_t)c % 16 == 0) && ((uintptr_t)out % 16 == 0) &&
                        (flags == nullptr || (uintptr_t)flags % 8 == 0);
    const bool f = flags != nullptr;
    if (w.bits == 16)
        return f ? launch_one<OP, 16, true, SM>(a, b, c, out, flags, n, w, pow_n, vec_ok, counts, st)
                 : launch_one<OP, 16, false, SM>(a, b, c, out, flags, n, w, pow_n, vec_ok, counts, st);
    return f ? launch_one<OP, 0, true, SM>(a, b, c, out, flags, n, w, pow_n, vec_ok, counts, st)
             : launch_one<OP, 0, false, SM>(a, b, c, out, flags, n, w, pow_n, vec_ok, counts, st);
}

template <bool SM>
int dispatch(const char *what, int op, int bits, const int16_t *a, const int16_t *b, const int16_t *c,
             int16_t *out, uint8_t *flags, int64_t n, int pow_n, sfb_counts *counts, cudaStream_t st) {
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "%s: width %d is not 4..16", what, bits);
    if (n < 0) return set_error(SFB_EINVAL, "%s: negative length %lld", what, (long long)n);
    if (n == 0) return SFB_OK;
    if (a == nullptr || out == nullptr) return set_error(SFB_EINVAL, "%s: null operand or output", what);
    const bool binary = op == SFB_OP_ADD || op == SFB_OP_SUB || op == SFB_OP_MUL || op == SFB_OP_DIV ||
                        op == SFB_OP_FMA;
    if (binary && b == nullptr) return set_error(SFB_EINVAL, "%s: op %d needs b", what, op);
    if (op == SFB_OP_FMA && c == nullptr) return set_error(SFB_EINVAL, "%s: fma needs c", what);
    if (op == SFB_OP_POW && pow_n < 1) return set_error(SFB_EINVAL, "%s: pow needs n >= 1", what);
    if (SM && counts == nullptr) return set_error(SFB_EINVAL, "%s: needs counts (pattern check)", what);
    const Width w = width(bits);
    switch (op) {
        case SFB_OP_ADD: return launch<SFB_OP_ADD, SM>(a, b, nullptr, out, flags, n, w, 0, counts, st);
        case SFB_OP_SUB: return launch<SFB_OP_SUB, SM>(a, b, nullptr, out, flags, n, w, 0, counts, st);
        case SFB_OP_MUL: return launch<SFB_OP_MUL, SM>(a, b, nullptr, out, flags, n, w, 0, counts, st);
        case SFB_OP_DIV: return launch<SFB_OP_DIV, SM>(a, b, nullptr, out, flags, n, w, 0, counts, st);
        case SFB_OP_FMA: return launch<SFB_OP_FMA, SM>(a, b, c, out, flags, n, w, 0, counts, st);
        case SFB_OP_NEG: return launch<SFB_OP_NEG, SM>(a, nullptr, nullptr, out, flags, n, w, 0, counts, st);
        case SFB_OP_ABS: return launch<SFB_OP_ABS, SM>(a, nullptr, nullptr, out, flags, n, w, 0, counts, st);
        case SFB_OP_SQRT: return launch<SFB_OP_SQRT, SM>(a, nullptr, nullptr, out, flags, n, w, 0, counts, st);
        case SFB_OP_POW: return launch<SFB_OP_POW, SM>(a, nullptr, nullptr, out, flags, n, w, pow_n, counts, st);
        default: return set_error(SFB_EINVAL, "%s: unknown op %d", what, op);
    }
}

// code <-> sign-magnitude word conversion, 8 per 128-bit vector
template <bool TO_BITS>
__global__ void __launch_bounds__(kThreads) convert_kernel(const uint16_t *__restrict__ in, uint16_t *__restrict__ out,
                                                           int64_t n, Width w, int vec_ok, sfb_counts *counts) {
    unsigned bad = 0;
    auto one = [&](uint16_t v) -> uint16_t {
        if constexpr (TO_BITS) {
            return (uint16_t)code_to_sm((int)(int16_t)v, w);
        } else {
            bool b;
            const int k = sm_to_code(v, w, b);
            bad += b;
            return (uint16_t)(int16_t)k;
        }
    };
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t done = 0;
    if (vec_ok) {
        const int64_t nv = n >> 3;
        for (int64_t v = tid; v < nv; v += stride) {
            union {
                uint4 u;
                uint16_t h[8];
            } x;
            x.u = __ldcs(reinterpret_cast<const uint4 *>(in) + v);
#pragma unroll
            for (int j = 0; j < 8; j++) x.h[j] = one(x.h[j]);
            __stcs(reinterpret_cast<uint4 *>(out) + v, x.u);
        }
        done = nv << 3;
    }
    for (int64_t i = done + tid; i < n; i += stride) out[i] = one(in[i]);
    if constexpr (!TO_BITS) {
        bad = __reduce_add_sync(0xffffffffu, bad);
        if ((threadIdx.x & 31) == 0 && bad && counts) atomicAdd(&counts->reserved[2], (unsigned long long)bad);
    }
}

template <bool TO_BITS>
int convert(const char *what, int bits, const uint16_t *in, uint16_t *out, int64_t n, sfb_counts *counts,
            cudaStream_t st) {
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "%s: width %d is not 4..16", what, bits);
    if (n < 0) return set_error(SFB_EINVAL, "%s: negative length", what);
    if (n == 0) return SFB_OK;
    if (in == nullptr || out == nullptr) return set_error(SFB_EINVAL, "%s: null buffer", what);
    const bool vec_ok = ((uintptr_t)in % 16 == 0) && ((uintptr_t)out % 16 == 0);
    const int64_t want = ((vec_ok ? (n >> 3) : n) + kThreads - 1) / kThreads;
    const int g = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sm_count() * 8));
    convert_kernel<TO_BITS><<<g, kThreads, 0, st>>>(in, out, n, width(bits), vec_ok, counts);
    return check_launch(what);
}

}  // namespace
}  // namespace sfb

extern "C" int sfb_elementwise(int op, int bits, const int16_t *a, const int16_t *b, const int16_t *c,
                               int16_t *out, uint8_t *flags, int64_t n, int pow_n, sfb_counts *counts,
                               sfb_stream stream) {
    return sfb::dispatch<false>("sfb_elementwise", op, bits, a, b, c, out, flags, n, pow_n, counts,
                                (cudaStream_t)stream);
}

extern "C" int sfb_elementwise_signmag(int op, int bits, const uint16_t *a, const uint16_t *b, const uint16_t *c,
                                       uint16_t *out, uint8_t *flags, int64_t n, int pow_n, sfb_counts *counts,
                                       sfb_stream stream) {
    auto p = [](const uint16_t *x) { return reinterpret_cast<const int16_t *>(x); };
    return sfb::dispatch<true>("sfb_elementwise_signmag", op, bits, p(a), p(b), p(c),
                               reinterpret_cast<int16_t *>(out), flags, n, pow_n, counts, (cudaStream_t)stream);
}

extern "C" int sfb_to_bits(int bits, const int16_t *codes, uint16_t *out, int64_t n, sfb_stream stream) {
    return sfb::convert<true>("sfb_to_bits", bits, reinterpret_cast<const uint16_t *>(codes), out, n, nullptr,
                              (cudaStream_t)stream);
}

extern "C" int sfb_from_bits(int bits, const uint16_t *patterns, int16_t *codes, int64_t n, sfb_counts *counts,
                             sfb_stream stream) {
    return sfb::convert<false>("sfb_from_bits", bits, patterns, reinterpret_cast<uint16_t *>(codes), n, counts,
                               (cudaStream_t)stream);
}
