// Chain matmul on sm_100a CUDA cores (the INT32 pipes).
//
// Per output (m, n) a chain of fma over k in increasing order
// (src/sf/_linalg.py:61-81, fma rule src/sf/_vectorized.py:128-131):
//     t   = trunc(a[m,k] b[k,n] / 2^(N-1))
//     acc = clip(acc + t, -M, M)
// overflow: some step clipped; underflow: some product a b != 0 truncated to
// t == 0 (such a step never clips, since acc is already in range).  The
// per-product floor and the per-step clip rule out an exact tensor-core
// formulation, so the chain runs on CUDA cores with k in order.  Optionally
// a bias code per column is added once after the chain with the saturating
// add (src/sf/torch/_core.py:376-378), whose overflow joins the output's, and
// the result is dequantized in float64 as y = acc / 2^(N-1) * a * s[n]
// (src/sf/torch/_core.py:381-382).
//
// Per product, on magnitudes |a|, |b| and sign masks sa, sb (0 or -1) kept
// apart in shared memory:
//     p = |a| |b|,  t = p >> (N-1),  x = t ^ sa ^ sb  (= t, or -t - 1 when negative)
// so the signed step is x plus 1 for a negative product; those +1s are
// counted per 32 k at once, popc(signword_a ^ signword_b).  Underflow is
// tracked as the running minimum of p - 1 (unsigned): it dips below
// 2^(N-1) - 1 exactly when some nonzero product is smaller than one unit.
// When the caller has proven that no partial sum can saturate (the
// reference's L1 bound; always the case under headroom="bound") the clip is
// dropped and the chain is a plain sum, any order; otherwise every step
// clips in k order and overflow is tracked per step.
//
// Tiling: a 256-thread CTA owns a 128 x 64 output tile, 8 x 4 outputs per
// thread; k-tiles of 32 staged through double-buffered shared memory.  Zero
// padding past K is neutral (a 0 product changes nothing, raises nothing).
#include "sfb_common.cuh"

namespace sfb {
namespace {

constexpr int BN = 64, BK = 32, TN = 4, THREADS = 256;

template <int BM>
struct Stage {
    uint32_t a_abs[BK][BM];   // |a|
    int32_t a_sgn[BK][BM];    // 0 or -1
    uint32_t b_abs[BK][BN];
    int32_t b_sgn[BK][BN];
    uint32_t a_sw[BM];        // sign bits of the 32 k of each row
    uint32_t b_sw[BN];
};

union Pack8 {
    uint4 u;
    int16_t h[8];
};

struct Epi {
    const int16_t *bias;      // nullable, N codes
    double a;                 // activation scale (dequant), used when y32 / y64 set
    const double *s_col;      // per-column scale (dequant)
    float *y32;               // nullable
    double *y64;              // nullable
    int16_t *codes;           // nullable
    uint8_t *flags;           // nullable
};

// TM rows per thread: 8 when the clip is proven unnecessary (BM = 128), 4 with
// the per-step clip and overflow tracking (BM = 64), to stay within registers.
template <bool SAFE, bool BITS16, int TM>
__global__ void __launch_bounds__(THREADS, 2) chain2_kernel(const int16_t *__restrict__ A, const int16_t *__restrict__ B,
                                                           int M, int N, int K, int64_t lda, int64_t ldb, int64_t sa,
                                                           int64_t sb, int64_t so, Width w0, Epi e, int vec,
                                                           sfb_counts *counts) {
    constexpr int BM = 16 * TM;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    Stage<BM> *st = reinterpret_cast<Stage<BM> *>(smem_raw);
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    const Width w = BITS16 ? Width{16, 15, 32767} : w0;
    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN), ty = tid / (BN / TN);
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int64_t z = blockIdx.z;
    A += z * sa;
    B += z * sb;

    int acc[TM][TN];
    uint32_t um[TM][TN], ov[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = 0, um[i][j] = 0xFFFFFFFFu, ov[i][j] = 0;

    // loader roles.  A: PER = 32 / (256 / BM) k of one row per thread; B: 8
    // columns of one k row per thread.  16-byte loads when the rows are aligned.
    constexpr int TPR = THREADS / BM;          // threads per A row: 2 or 4
    constexpr int PER = BK / TPR;              // k per thread: 16 or 8
    const int ar = tid / TPR, ah = tid % TPR;
    const int bk = tid >> 3, bc = (tid & 7) * 8;
    Pack8 ra[PER / 8], rb;
    auto load_regs = [&](int k0) {
        const int gm = m0 + ar;
        const int ka = k0 + ah * PER;
#pragma unroll
        for (int q = 0; q < PER / 8; q++) {
            const int kq = ka + q * 8;
            if (vec && gm < M && kq + 8 <= K) {
                ra[q].u = __ldg(reinterpret_cast<const uint4 *>(A + (int64_t)gm * lda + kq));
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++)
                    ra[q].h[j] = (gm < M && kq + j < K) ? A[(int64_t)gm * lda + kq + j] : (int16_t)0;
            }
        }
        const int gk = k0 + bk, gn0 = n0 + bc;
        if (vec && gk < K && gn0 + 8 <= N) {
            rb.u = __ldg(reinterpret_cast<const uint4 *>(B + (int64_t)gk * ldb + gn0));
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) rb.h[j] = (gk < K && gn0 + j < N) ? B[(int64_t)gk * ldb + gn0 + j] : (int16_t)0;
        }
    };
    auto store_regs = [&](Stage<BM> &s) {
        uint32_t bits = 0;
#pragma unroll
        for (int q = 0; q < PER / 8; q++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int v = ra[q].h[j];
                const int kk = ah * PER + q * 8 + j;
                s.a_abs[kk][ar] = (uint32_t)abs(v);
                s.a_sgn[kk][ar] = v >> 31;
                bits |= (uint32_t)(v < 0) << kk;
            }
#pragma unroll
        for (int o = 1; o < TPR; o <<= 1) bits |= __shfl_xor_sync(0xffffffffu, bits, o);
        if (ah == 0) s.a_sw[ar] = bits;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int v = rb.h[j];
            s.b_abs[bk][bc + j] = (uint32_t)abs(v);
            s.b_sgn[bk][bc + j] = v >> 31;
        }
    };

    const int nk = (K + BK - 1) / BK;
    if (nk > 0) {
        load_regs(0);
        store_regs(st[0]);
    }
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        Stage<BM> &cur = st[kt & 1];
        if (tid < BN) {                       // column sign words of this k-tile
            uint32_t bits = 0;
#pragma unroll 8
            for (int k = 0; k < BK; k++) bits |= (uint32_t)(cur.b_sgn[k][tid] & 1) << k;
            cur.b_sw[tid] = bits;
        }
        if (kt + 1 < nk) load_regs((kt + 1) * BK);
        __syncthreads();
#pragma unroll 2
        for (int k = 0; k < BK; k++) {
            uint32_t aa[TM];
            int32_t as_[TM];
#pragma unroll
            for (int q = 0; q < TM / 4; q++) {
                const uint4 av = *reinterpret_cast<const uint4 *>(&cur.a_abs[k][ty * TM + 4 * q]);
                const int4 sv = *reinterpret_cast<const int4 *>(&cur.a_sgn[k][ty * TM + 4 * q]);
                aa[4 * q] = av.x, aa[4 * q + 1] = av.y, aa[4 * q + 2] = av.z, aa[4 * q + 3] = av.w;
                as_[4 * q] = sv.x, as_[4 * q + 1] = sv.y, as_[4 * q + 2] = sv.z, as_[4 * q + 3] = sv.w;
            }
            const uint4 bv = *reinterpret_cast<const uint4 *>(&cur.b_abs[k][tx * TN]);
            const int4 bs = *reinterpret_cast<const int4 *>(&cur.b_sgn[k][tx * TN]);
            const uint32_t ba[TN] = {bv.x, bv.y, bv.z, bv.w};
            const int32_t bs_[TN] = {bs.x, bs.y, bs.z, bs.w};
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) {
                    const uint32_t p = aa[i] * ba[j];
                    const int32_t t = (int32_t)(p >> w.sh);
                    um[i][j] = min(um[i][j], p - 1u);
                    if (SAFE) {
                        acc[i][j] += t ^ as_[i] ^ bs_[j];             // + popc term below
                    } else {
                        const int32_t sg = as_[i] ^ bs_[j];
                        const int32_t s = acc[i][j] + ((t ^ sg) - sg);
                        const int32_t c = clampi(s, -w.M, w.M);
                        ov[i][j] |= (uint32_t)(s ^ c);
                        acc[i][j] = c;
                    }
                }
        }
        if (SAFE) {
#pragma unroll
            for (int i = 0; i < TM; i++) {
                const uint32_t sa_w = cur.a_sw[ty * TM + i];
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] += __popc(sa_w ^ cur.b_sw[tx * TN + j]);
            }
        }
        if (kt + 1 < nk) store_regs(st[(kt + 1) & 1]);
        __syncthreads();
    }

    Counts cnt;
    const uint32_t unit_m1 = (1u << w.sh) - 1u;   // um < 2^(N-1) - 1  <=>  some 0 < p < 2^(N-1)
    unsigned bad = 0;
#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int gm = m0 + ty * TM + i;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int gn = n0 + tx * TN + j;
            if (gm < M && gn < N) {
                int v = acc[i][j];
                bool o = ov[i][j] != 0;
                if (SAFE && (v > w.M || v < -w.M)) {           // the caller's proof did not hold
                    bad++;
                    v = clampi(v, -w.M, w.M);
                }
                if (e.bias) {
                    const int s = v + (int)e.bias[gn];
                    o |= (s > w.M || s < -w.M);
                    v = clampi(s, -w.M, w.M);
                }
                const bool un = um[i][j] < unit_m1;
                const int64_t idx = z * so + (int64_t)gm * N + gn;
                if (e.codes) e.codes[idx] = (int16_t)v;
                if (e.flags) e.flags[idx] = (uint8_t)((o ? SFB_F_OVERFLOW : 0u) | (un ? SFB_F_UNDERFLOW : 0u));
                if (e.y32 || e.y64) {
                    const double y = (double)v / (double)(1 << w.sh) * e.a * e.s_col[gn];
                    if (e.y32) e.y32[idx] = (float)y;
                    if (e.y64) e.y64[idx] = y;
                }
                cnt.over += o;
                cnt.under += un;
            }
        }
    }
    if (SAFE && bad && counts) atomicAdd(&counts->reserved[1], (unsigned long long)bad);
    flush_counts(cnt, counts, sc);
}

int launch_chain(int bits, const int16_t *A, const int16_t *B, const Epi &e, int64_t batch, int64_t M, int64_t N,
                 int64_t K, int64_t lda, int64_t ldb, int64_t sa, int64_t sb, int64_t so, bool safe,
                 sfb_counts *counts, cudaStream_t st, const char *what) {
    const int BM = safe ? 128 : 64;
    const int64_t mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
    if (mt > 65535 || nt > 0x7fffffff || batch > 65535 || K > 0x7fffffff || M > 0x7fffffff || N > 0x7fffffff)
        return set_error(SFB_ERANGE, "%s: %lld x %lld x %lld (batch %lld) exceeds the launch limits", what,
                         (long long)M, (long long)N, (long long)K, (long long)batch);
    dim3 grid((unsigned)nt, (unsigned)mt, (unsigned)batch);
    const int smem = safe ? 2 * (int)sizeof(Stage<128>) : 2 * (int)sizeof(Stage<64>);
    static bool attr[64][4] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    const Width w = width(bits);
    const bool b16 = bits == 16;
    const int which = (safe ? 2 : 0) + (b16 ? 1 : 0);
    auto kern = safe ? (b16 ? chain2_kernel<true, true, 8> : chain2_kernel<true, false, 8>)
                     : (b16 ? chain2_kernel<false, true, 4> : chain2_kernel<false, false, 4>);
    const int vec = (lda % 8 == 0) && (ldb % 8 == 0) && ((uintptr_t)A % 16 == 0) && ((uintptr_t)B % 16 == 0) &&
                    (sa % 8 == 0) && (sb % 8 == 0);
    if (!attr[dev][which]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_launch(what);
        attr[dev][which] = true;
    }
    kern<<<grid, THREADS, smem, st>>>(A, B, (int)M, (int)N, (int)K, lda, ldb, sa, sb, so, w, e, vec, counts);
    return check_launch(what);
}

int chain_args(const char *what, int bits, const int16_t *A, const int16_t *B, int64_t batch, int64_t M, int64_t N,
               int64_t K, int64_t lda, int64_t ldb, int64_t so) {
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "%s: width %d is not 4..16", what, bits);
    if (batch < 0 || M < 0 || N < 0 || K < 0) return set_error(SFB_EINVAL, "%s: negative size", what);
    if (K > 0 && (A == nullptr || B == nullptr)) return set_error(SFB_EINVAL, "%s: null operand", what);
    if (K > 0 && (lda < K || ldb < N)) return set_error(SFB_EINVAL, "%s: lda < K or ldb < N", what);
    if (so < M * N && batch > 1) return set_error(SFB_EINVAL, "%s: output batch entries overlap", what);
    return SFB_OK;
}

}  // namespace
}  // namespace sfb

extern "C" int sfb_matmul_chain(int bits, const int16_t *A, const int16_t *B, const int16_t *bias, int16_t *out,
                                uint8_t *flags, int64_t batch, int64_t M, int64_t N, int64_t K, int64_t lda,
                                int64_t ldb, int64_t stride_a, int64_t stride_b, int64_t stride_out,
                                sfb_counts *counts, sfb_stream stream) {
    using namespace sfb;
    int rc = chain_args("sfb_matmul_chain", bits, A, B, batch, M, N, K, lda, ldb, stride_out);
    if (rc) return rc;
    if (batch == 0 || M == 0 || N == 0) return SFB_OK;
    if (out == nullptr) return set_error(SFB_EINVAL, "sfb_matmul_chain: null output");
    Epi e{bias, 0.0, nullptr, nullptr, nullptr, out, flags};
    return launch_chain(bits, A, B, e, batch, M, N, K, lda, ldb, stride_a, stride_b, stride_out, false, counts,
                        (cudaStream_t)stream, "sfb_matmul_chain");
}

extern "C" int sfb_linear_chain(int bits, const int16_t *X, const int16_t *WT, const int16_t *bias, double a,
                                const double *s_col, int proven_no_saturation, float *y32, double *y64,
                                int16_t *codes, uint8_t *flags, int64_t R, int64_t N, int64_t K, int64_t ldx,
                                int64_t ldw, sfb_counts *counts, sfb_stream stream) {
    using namespace sfb;
    int rc = chain_args("sfb_linear_chain", bits, X, WT, 1, R, N, K, ldx, ldw, R * N);
    if (rc) return rc;
    if (R == 0 || N == 0) return SFB_OK;
    if ((y32 || y64) && s_col == nullptr) return set_error(SFB_EINVAL, "sfb_linear_chain: y needs s_col");
    if (!y32 && !y64 && !codes) return set_error(SFB_EINVAL, "sfb_linear_chain: no output requested");
    Epi e{bias, a, s_col, y32, y64, codes, flags};
    return launch_chain(bits, X, WT, e, 1, R, N, K, ldx, ldw, 0, 0, R * N, proven_no_saturation != 0, counts,
                        (cudaStream_t)stream, "sfb_linear_chain");
}
