// Sequential saturating reductions: sum along an axis (src/sf/_linalg.py:30-39,
// the Device "sum" op, src/sf/_device.py:176-178) and the 1-D dot as a chain of
// fma (src/sf/_linalg.py:42-58), in the reference's order (index 0 first).
//
// Each step is v -> clip(v + x, -M, M) (for dot, x = trunc(a b / 2^(N-1))).
// Such maps are closed under composition: a segment of steps is
//     v -> clip(v + s, lo, hi)
// with s the plain sum, and composing A then B gives
//     s  = sA + sB,  lo = clamp(loA + sB, loB, hiB),  hi = clamp(hiA + sB, loB, hiB).
// From v = 0 a step clips exactly when an unclipped prefix sum leaves
// [-M, M] (before the first clip the trajectory is the prefix sum), so a
// segment also carries its largest and smallest prefix sums, composing as
//     pmax = max(pmaxA, sA + pmaxB),  pmin = min(pminA, sA + pminB).
// The result is clip(s, lo, hi) and overflow is pmax > M or pmin < -M: the
// sequential chain's bits, computed as an ordered parallel reduction.
// Underflow (dot: a nonzero product truncating to 0) is an OR.
//
// Layout (outer, K, inner), reduced over K.  inner > 1: one thread per
// output walks k (loads coalesced across inner).  inner == 1: each output's
// K is cut into contiguous pieces, a CTA per piece, contiguous chunks per
// thread; chunk summaries combine in thread order inside the CTA and the
// CTA summaries in piece order in a second pass (caller workspace).
#include <algorithm>

#include "sfb_common.cuh"

namespace sfb {
namespace {

constexpr int RT = 256;
constexpr long long INF = 1ll << 62;

struct Seg {
    long long s, lo, hi, pmax, pmin;
    int under;
};

__device__ __forceinline__ long long clampll(long long v, long long lo, long long hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

__device__ __forceinline__ Seg identity() { return Seg{0, -INF, INF, -INF, INF, 0}; }

__device__ __forceinline__ Seg compose(const Seg &A, const Seg &B) {
    Seg r;
    r.s = A.s + B.s;
    r.lo = clampll(A.lo + B.s, B.lo, B.hi);
    r.hi = clampll(A.hi + B.s, B.lo, B.hi);
    r.pmax = max(A.pmax, A.s + B.pmax);
    r.pmin = min(A.pmin, A.s + B.pmin);
    r.under = A.under | B.under;
    return r;
}

__device__ __forceinline__ Seg shfl_down_seg(const Seg &v, int off) {
    Seg r;
    r.s = __shfl_down_sync(0xffffffffu, v.s, off);
    r.lo = __shfl_down_sync(0xffffffffu, v.lo, off);
    r.hi = __shfl_down_sync(0xffffffffu, v.hi, off);
    r.pmax = __shfl_down_sync(0xffffffffu, v.pmax, off);
    r.pmin = __shfl_down_sync(0xffffffffu, v.pmin, off);
    r.under = __shfl_down_sync(0xffffffffu, v.under, off);
    return r;
}

// ordered reduction of the CTA's per-thread segments (thread 0 first); the
// result is valid in thread 0
__device__ Seg cta_reduce(Seg v) {
    __shared__ Seg warps[RT / 32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const Seg o = shfl_down_seg(v, off);
        if ((lane & (2 * off - 1)) == 0 && lane + off < 32) v = compose(v, o);
    }
    if (lane == 0) warps[wid] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        v = warps[0];
        for (int w = 1; w < RT / 32; w++) v = compose(v, warps[w]);
    }
    return v;
}

// one thread's contiguous chunk [k0, k1): int32 running values (a chunk has at
// most 2^15 + 8 elements, so |s| < 2^31)
template <bool DOT>
__device__ Seg chunk_seg(const int16_t *__restrict__ a, const int16_t *__restrict__ b, int64_t k0, int64_t k1,
                         Width w, bool vec) {
    if (k0 >= k1) return identity();
    int s = 0, pmax = -(1 << 30), pmin = 1 << 30, lo = -(1 << 30), hi = 1 << 30, under = 0;
    auto step = [&](int x) {
        s += x;
        pmax = max(pmax, s);
        pmin = min(pmin, s);
        lo = clampi(lo + x, -w.M, w.M);
        hi = clampi(hi + x, -w.M, w.M);
    };
    auto value = [&](int ca, int cb) -> int {
        if constexpr (DOT) {
            const int p = ca * cb;
            under |= (p != 0) & ((unsigned)(p + ((1 << w.sh) - 1)) <= (unsigned)((2 << w.sh) - 2));
            return tdiv_pow2(p, w.sh);
        } else {
            return ca;
        }
    };
    int64_t k = k0;
    if (vec) {
        for (; k + 8 <= k1; k += 8) {
            union {
                uint4 u;
                int16_t h[8];
            } va, vb;
            va.u = __ldg(reinterpret_cast<const uint4 *>(a + k));
            if constexpr (DOT) vb.u = __ldg(reinterpret_cast<const uint4 *>(b + k));
#pragma unroll
            for (int j = 0; j < 8; j++) step(value(va.h[j], DOT ? vb.h[j] : 0));
        }
    }
    for (; k < k1; k++) step(value(a[k], DOT ? b[k] : 0));
    return Seg{s, lo, hi, pmax, pmin, under};
}

__device__ __forceinline__ void finish_one(const Seg &t, Width w, int16_t *out, uint8_t *flags, int64_t o,
                                           Counts &cnt) {
    const int r = (int)clampll(t.s, t.lo, t.hi);
    const bool over = t.pmax > w.M || t.pmin < -w.M;
    out[o] = (int16_t)r;
    if (flags) flags[o] = (uint8_t)((over ? SFB_F_OVERFLOW : 0u) | (t.under ? SFB_F_UNDERFLOW : 0u));
    cnt.over += over;
    cnt.under += t.under != 0;
}

// inner > 1: one thread per output, sequential over k
__global__ void __launch_bounds__(RT) sum_strided_kernel(const int16_t *__restrict__ x, int64_t outer, int64_t K,
                                                         int64_t inner, Width w, int16_t *__restrict__ out,
                                                         uint8_t *__restrict__ flags, sfb_counts *counts) {
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    Counts cnt;
    const int64_t total = outer * inner;
    for (int64_t o = (int64_t)blockIdx.x * RT + threadIdx.x; o < total; o += (int64_t)gridDim.x * RT) {
        const int64_t ob = o / inner, i = o - ob * inner;
        const int16_t *p = x + ob * K * inner + i;
        int acc = 0;
        bool over = false;
        for (int64_t k = 0; k < K; k++) {
            const int v = acc + p[k * inner];
            const int c = clampi(v, -w.M, w.M);
            over |= c != v;
            acc = c;
        }
        out[o] = (int16_t)acc;
        if (flags) flags[o] = over ? SFB_F_OVERFLOW : 0u;
        cnt.over += over;
    }
    flush_counts(cnt, counts, sc);
}

// inner == 1: CTA (piece, output) over K range [piece * span, ...)
template <bool DOT>
__global__ void __launch_bounds__(RT) reduce_pieces_kernel(const int16_t *__restrict__ a,
                                                           const int16_t *__restrict__ b, int64_t K, int64_t span,
                                                           int64_t chunk, Width w, int vec, Seg *__restrict__ ws,
                                                           int16_t *__restrict__ out, uint8_t *__restrict__ flags,
                                                           sfb_counts *counts) {
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    const int64_t o = blockIdx.x, piece = blockIdx.y;
    const int16_t *pa = a + o * K;
    const int16_t *pb = DOT ? b + o * K : nullptr;
    const int64_t base = piece * span, end = min(K, base + span);
    const int64_t k0 = min(end, base + (int64_t)threadIdx.x * chunk), k1 = min(end, k0 + chunk);
    const Seg t = cta_reduce(chunk_seg<DOT>(pa, pb, k0, k1, w, vec != 0));
    Counts cnt;
    if (threadIdx.x == 0) {
        if (ws) ws[o * gridDim.y + piece] = t;
        else finish_one(t, w, out, flags, o, cnt);
    }
    if (!ws) flush_counts(cnt, counts, sc);
}

__global__ void __launch_bounds__(RT) combine_pieces_kernel(const Seg *__restrict__ ws, int64_t outputs,
                                                            int pieces, Width w, int16_t *__restrict__ out,
                                                            uint8_t *__restrict__ flags, sfb_counts *counts) {
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    Counts cnt;
    for (int64_t o = (int64_t)blockIdx.x * RT + threadIdx.x; o < outputs; o += (int64_t)gridDim.x * RT) {
        Seg t = ws[o * pieces];
        for (int p = 1; p < pieces; p++) t = compose(t, ws[o * pieces + p]);
        finish_one(t, w, out, flags, o, cnt);
    }
    flush_counts(cnt, counts, sc);
}

// pieces per output: enough CTAs to fill the GPU, at least 16 elements per
// thread, chunks of at most 2^15 elements, at most 4096 pieces
struct Plan {
    int64_t pieces, span, chunk;
};

Plan plan_for(int64_t outputs, int64_t K) {
    const int64_t want = (int64_t)sm_count() * 4;
    int64_t pieces = outputs >= want ? 1 : (want + outputs - 1) / outputs;
    const int64_t most = (K + RT * 16 - 1) / (RT * 16);                 // >= 16 elements per thread
    pieces = std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(pieces, most), 4096));
    const int64_t least = (K + (int64_t)RT * 32768 - 1) / ((int64_t)RT * 32768);   // chunk <= 2^15
    pieces = std::max(pieces, least);
    int64_t span = (K + pieces - 1) / pieces;
    span = (span + 8 * RT - 1) / (8 * RT) * (8 * RT);                    // whole vectors per thread
    pieces = std::max<int64_t>(1, (K + span - 1) / span);
    return Plan{pieces, span, span / RT};
}

int launch_pieces(bool dot, const int16_t *a, const int16_t *b, int64_t outputs, int64_t K, Width w, bool vec,
                  int16_t *out, uint8_t *flags, void *workspace, int64_t ws_bytes, sfb_counts *counts,
                  cudaStream_t st, const char *what) {
    const Plan p = plan_for(outputs, K);
    if (outputs > 0x7fffffff || p.pieces > 65535)
        return set_error(SFB_ERANGE, "%s: %lld outputs x %lld pieces exceed the launch limits", what,
                         (long long)outputs, (long long)p.pieces);
    Seg *ws = nullptr;
    if (p.pieces > 1) {
        const int64_t need = outputs * p.pieces * (int64_t)sizeof(Seg);
        if (workspace == nullptr || ws_bytes < need)
            return set_error(SFB_EINVAL, "%s: workspace of %lld bytes is smaller than the %lld needed", what,
                             (long long)ws_bytes, (long long)need);
        ws = reinterpret_cast<Seg *>(workspace);
    }
    dim3 grid((unsigned)outputs, (unsigned)p.pieces);
    if (dot)
        reduce_pieces_kernel<true><<<grid, RT, 0, st>>>(a, b, K, p.span, p.chunk, w, vec, ws, out, flags, counts);
    else
        reduce_pieces_kernel<false><<<grid, RT, 0, st>>>(a, b, K, p.span, p.chunk, w, vec, ws, out, flags, counts);
    int rc = check_launch(what);
    if (rc || !ws) return rc;
    const int64_t g = std::min<int64_t>((outputs + RT - 1) / RT, (int64_t)sm_count() * 8);
    combine_pieces_kernel<<<(unsigned)std::max<int64_t>(g, 1), RT, 0, st>>>(ws, outputs, (int)p.pieces, w, out,
                                                                            flags, counts);
    return check_launch(what);
}

}  // namespace
}  // namespace sfb

extern "C" int64_t sfb_reduce_workspace(int64_t outputs, int64_t K) {
    using namespace sfb;
    if (outputs < 0 || K < 0) return set_error(SFB_EINVAL, "sfb_reduce_workspace: negative size");
    if (outputs == 0 || K == 0) return 0;
    const Plan p = plan_for(outputs, K);
    return p.pieces > 1 ? outputs * p.pieces * (int64_t)sizeof(Seg) : 0;
}

extern "C" int sfb_sum(int bits, const int16_t *x, int64_t outer, int64_t K, int64_t inner, int16_t *out,
                       uint8_t *flags, void *workspace, int64_t workspace_bytes, sfb_counts *counts,
                       sfb_stream stream) {
    using namespace sfb;
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "sfb_sum: width %d is not 4..16", bits);
    if (outer < 0 || K < 0 || inner < 0) return set_error(SFB_EINVAL, "sfb_sum: negative size");
    if (outer == 0 || inner == 0) return SFB_OK;
    if (out == nullptr || (K > 0 && x == nullptr)) return set_error(SFB_EINVAL, "sfb_sum: null operand or output");
    if (counts == nullptr) return set_error(SFB_EINVAL, "sfb_sum: null counts");
    const Width w = width(bits);
    cudaStream_t st = (cudaStream_t)stream;
    if (K == 0) {                                   // the empty sum is 0, no event
        if (cudaMemsetAsync(out, 0, (size_t)(outer * inner) * 2, st) != cudaSuccess ||
            (flags && cudaMemsetAsync(flags, 0, (size_t)(outer * inner), st) != cudaSuccess))
            return check_launch("sfb_sum");
        return SFB_OK;
    }
    if (inner > 1 || (K <= 1024 && outer >= (int64_t)sm_count() * RT)) {     // a thread per output
        const int64_t g = std::min<int64_t>((outer * inner + RT - 1) / RT, (int64_t)sm_count() * 8);
        sum_strided_kernel<<<(unsigned)std::max<int64_t>(g, 1), RT, 0, st>>>(x, outer, K, inner, w, out, flags,
                                                                             counts);
        return check_launch("sfb_sum");
    }
    const bool vec = ((uintptr_t)x % 16 == 0) && (K % 8 == 0);
    return launch_pieces(false, x, nullptr, outer, K, w, vec, out, flags, workspace, workspace_bytes, counts, st,
                         "sfb_sum");
}

extern "C" int sfb_dot(int bits, const int16_t *a, const int16_t *b, int64_t n, int16_t *out, uint8_t *flags,
                       void *workspace, int64_t workspace_bytes, sfb_counts *counts, sfb_stream stream) {
    using namespace sfb;
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "sfb_dot: width %d is not 4..16", bits);
    if (n < 0) return set_error(SFB_EINVAL, "sfb_dot: negative length");
    if (out == nullptr || (n > 0 && (a == nullptr || b == nullptr)))
        return set_error(SFB_EINVAL, "sfb_dot: null operand or output");
    if (counts == nullptr) return set_error(SFB_EINVAL, "sfb_dot: null counts");
    cudaStream_t st = (cudaStream_t)stream;
    if (n == 0) {
        if (cudaMemsetAsync(out, 0, 2, st) != cudaSuccess || (flags && cudaMemsetAsync(flags, 0, 1, st) != cudaSuccess))
            return check_launch("sfb_dot");
        return SFB_OK;
    }
    const bool vec = ((uintptr_t)a % 16 == 0) && ((uintptr_t)b % 16 == 0);
    return launch_pieces(true, a, b, 1, n, width(bits), vec, out, flags, workspace, workspace_bytes, counts, st,
                         "sfb_dot");
}
