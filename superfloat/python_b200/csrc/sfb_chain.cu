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
// Underflow is tracked as the running minimum of p - 1 (unsigned, p =
// |a| |b|): it dips below 2^(N-1) - 1 exactly when some nonzero product is
// smaller than one unit.  When the caller has proven that no partial sum can
// saturate (the reference's L1 bound; always the case under
// headroom="bound") the clip is dropped and the chain is a plain sum, any
// order; otherwise every step clips in k order and overflow is tracked per
// step.
//
// General mode (chain2_kernel): a 256-thread CTA owns a 64 x 64 output tile,
// 4 x 4 outputs per thread (or 128 threads on 32 x 64 / 16 x 64 tiles for
// small problems); k-tiles of 32 staged through double-buffered shared
// memory as |a|, |a| << (32 - (N-1)), sign(a) = +-1, |b|, sign(b) = +-1.  A
// step is t = umulhi(|a| << (32 - (N-1)), |b|) (the truncated magnitude),
// the underflow minimum of |a| |b| - 1, s = t (sa sb) + acc: four IMADs on
// the FMA pipe; and the clip to [-M, M] (two min / max) and the overflow OR
// of s ^ clip(s) on the ALU pipe, which the clip in k order keeps serial.
// Zero padding past K is neutral (a 0 product changes nothing, raises
// nothing).
//
// Proven mode (chain_pk_kernel): every partial sum stays within [-M, M], so
// two outputs (n, n+1) share one 32-bit accumulator as two 16-bit lanes and
// two products cost two IMADs, one byte permute, one LOP3, one add and one
// LOP3 for the underflow test.  Per product (lane), with c = 0x7FFF + [a == 0]:
//     p2 = |a| (|b| << (17 - N)) + (c << 16),   lane u = p2 >> 16 = t + c
// (t = trunc(|a| |b| / 2^(N-1)) < 2^15, so u < 2^16 and bit 15 of u is set
// exactly when t >= 1 or a == 0).  The byte permute gathers the two lanes'
// upper halves into one word pk; the step adds x = pk ^ sa ^ sb (sa a full
// word mask, sb per-lane 0xFFFF masks: x = u, or 0xFFFF - u when the product
// is negative) and ANDs pk | zb (zb: 0xFFFF per lane where b == 0) into the
// underflow word.  The sum of x over a 32-k block equals the wanted signed
// sum plus 32 * 0x7FFF plus popc(w_a ^ w_b) per lane, with w_a the row's
// bits (a < 0 or a == 0) and w_b the column's bits (b < 0): that correction
// is subtracted per block (lane carries only move whole units of 2^16 that
// the decode accounts for), and the final word decodes as lo = int16(low
// half), hi = (word - lo) >> 16.  Underflow of lane L: bit 15 + 16 L of the
// underflow word is clear.  A 384-thread CTA owns a 192 x 128 tile, 8 rows x
// 4 lane pairs per thread, one CTA per SM.
#include <algorithm>
#include <type_traits>

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

union Pack4 {
    uint2 u;
    int16_t h[4];
};

// V int16 codes loaded as one vector: 16 bytes (V = 8) or 8 bytes (V = 4)
template <int V>
using PackV = typename std::conditional<V == 8, Pack8, Pack4>::type;

struct Epi {
    const int16_t *bias;      // nullable, N codes
    double a;                 // activation scale (dequant), used when y32 / y64 set
    const double *a_dev;      // nullable: the scale read from device memory instead
    const double *s_col;      // per-column scale (dequant)
    float *y32;               // nullable
    double *y64;              // nullable
    int16_t *codes;           // nullable
    uint8_t *flags;           // nullable
};

// One output of either kernel: the optional saturating bias add, codes,
// flags, float64 dequantization, event counts.
__device__ __forceinline__ void emit(const Epi &e, const Width &w, int64_t idx, int gn, int v, bool o, bool un,
                                     Counts &cnt) {
    if (e.bias) {
        const int s = v + (int)e.bias[gn];
        o |= (s > w.M || s < -w.M);
        v = clampi(s, -w.M, w.M);
    }
    if (e.codes) e.codes[idx] = (int16_t)v;
    if (e.flags) e.flags[idx] = (uint8_t)((o ? SFB_F_OVERFLOW : 0u) | (un ? SFB_F_UNDERFLOW : 0u));
    if (e.y32 || e.y64) {
        const double y = (double)v / (double)(1 << w.sh) * (e.a_dev ? __ldg(e.a_dev) : e.a) * e.s_col[gn];
        if (e.y32) e.y32[idx] = (float)y;
        if (e.y64) e.y64[idx] = y;
    }
    cnt.over += o;
    cnt.under += un;
}

// General-mode operands of one k-tile, kept apart so that each step is
// multiplies on the FMA pipe and min / max / logic on the ALU pipe:
//     t   = umulhi(|a| << (32 - (N-1)), |b|)   = trunc(|a| |b| / 2^(N-1))
//     p-1 = |a| |b| - 1 (unsigned)              (the underflow minimum)
//     s   = t * (sa sb) + acc                   (sa, sb = +-1)
//     acc = clip(s, -M, M),  overflow |= s ^ acc
template <int BM, int CN = BN>
struct GStage {
    uint32_t a_abs[BK][BM];   // |a|
    uint32_t a_hi[BK][BM];    // |a| << (32 - (N-1))
    int32_t a_sgn[BK][BM];    // +1 or -1
    uint32_t b_abs[BK][CN];
    int32_t b_sgn[BK][CN];    // +1 or -1
};

// TM rows and CT columns per thread, CN columns per CTA (NT / (CN / CT) row
// groups, BM = that times TM rows): 4 x 4 outputs per thread on 64-column
// tiles, or fewer for problems so small that the outputs give too few warps.
template <bool BITS16, int TM, int NT = THREADS, int CN = BN, int CT = TN>
__global__ void __launch_bounds__(NT, 2) chain2_kernel(const int16_t *__restrict__ A, const int16_t *__restrict__ B,
                                                           int M, int N, int K, int64_t lda, int64_t ldb, int64_t sa,
                                                           int64_t sb, int64_t so, Width w0, Epi e, int vec,
                                                           sfb_counts *counts) {
    constexpr int BM = (NT / (CN / CT)) * TM;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    GStage<BM, CN> *st = reinterpret_cast<GStage<BM, CN> *>(smem_raw);
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    const Width w = BITS16 ? Width{16, 15, 32767} : w0;
    const int hi_shift = 32 - w.sh;
    const int tid = threadIdx.x;
    const int tx = tid % (CN / CT), ty = tid / (CN / CT);
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * CN;
    const int64_t z = blockIdx.z;
    A += z * sa;
    B += z * sb;

    int acc[TM][CT];
    uint32_t um[TM][CT], ov[TM][CT];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < CT; j++) acc[i][j] = 0, um[i][j] = 0xFFFFFFFFu, ov[i][j] = 0;

    // loader roles.  A: PER = 32 / (NT / BM) k of one row per thread; B: 8
    // columns of BPASS k rows per thread.  Vector loads when the rows are aligned.
    constexpr int TPR = NT / BM;               // threads per A row: 4 or 8
    constexpr int PER = BK / TPR;              // k per thread: 8 or 4
    constexpr int AV = PER < 8 ? PER : 8;      // codes per A vector load
    constexpr int BROWS = NT / (CN / 8), BPASS = BK / BROWS;
    static_assert(PER % AV == 0 && (AV == 8 || AV == 4) && BPASS * BROWS == BK, "chain2 loader shape");
    static_assert(CT == 4 || CT == 2, "four or two columns per thread");
    const int ar = tid / TPR, ah = tid % TPR;
    const int bk = tid / (CN / 8), bc = (tid % (CN / 8)) * 8;
    PackV<AV> ra[PER / AV];
    Pack8 rb[BPASS];
    auto load_regs = [&](int k0) {
        const int gm = m0 + ar;
        const int ka = k0 + ah * PER;
#pragma unroll
        for (int q = 0; q < PER / AV; q++) {
            const int kq = ka + q * AV;
            if (vec && gm < M && kq + AV <= K) {
                ra[q].u = __ldg(reinterpret_cast<const decltype(ra[q].u) *>(A + (int64_t)gm * lda + kq));
            } else {
#pragma unroll
                for (int j = 0; j < AV; j++)
                    ra[q].h[j] = (gm < M && kq + j < K) ? A[(int64_t)gm * lda + kq + j] : (int16_t)0;
            }
        }
#pragma unroll
        for (int p = 0; p < BPASS; p++) {
            const int gk = k0 + bk + p * BROWS, gn0 = n0 + bc;
            if (vec && gk < K && gn0 + 8 <= N) {
                rb[p].u = __ldg(reinterpret_cast<const uint4 *>(B + (int64_t)gk * ldb + gn0));
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++)
                    rb[p].h[j] = (gk < K && gn0 + j < N) ? B[(int64_t)gk * ldb + gn0 + j] : (int16_t)0;
            }
        }
    };
    auto store_regs = [&](GStage<BM, CN> &s) {
#pragma unroll
        for (int q = 0; q < PER / AV; q++)
#pragma unroll
            for (int j = 0; j < AV; j++) {
                const int v = ra[q].h[j];
                const int kk = ah * PER + q * AV + j;
                const uint32_t mag = (uint32_t)abs(v);
                s.a_abs[kk][ar] = mag;
                s.a_hi[kk][ar] = mag << hi_shift;
                s.a_sgn[kk][ar] = v < 0 ? -1 : 1;
            }
#pragma unroll
        for (int p = 0; p < BPASS; p++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int v = rb[p].h[j];
                s.b_abs[bk + p * BROWS][bc + j] = (uint32_t)abs(v);
                s.b_sgn[bk + p * BROWS][bc + j] = v < 0 ? -1 : 1;
            }
    };

    const int nk = (K + BK - 1) / BK;
    if (nk > 0) {
        load_regs(0);
        store_regs(st[0]);
    }
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        GStage<BM, CN> &cur = st[kt & 1];
        if (kt + 1 < nk) load_regs((kt + 1) * BK);
#pragma unroll 8
        for (int k = 0; k < BK; k++) {
            uint32_t aa[TM], ahi[TM];
            int32_t as_[TM];
            if constexpr (TM >= 4) {
#pragma unroll
                for (int q = 0; q < TM / 4; q++) {
                    const uint4 av = *reinterpret_cast<const uint4 *>(&cur.a_abs[k][ty * TM + 4 * q]);
                    const uint4 hv = *reinterpret_cast<const uint4 *>(&cur.a_hi[k][ty * TM + 4 * q]);
                    const int4 sv = *reinterpret_cast<const int4 *>(&cur.a_sgn[k][ty * TM + 4 * q]);
                    aa[4 * q] = av.x, aa[4 * q + 1] = av.y, aa[4 * q + 2] = av.z, aa[4 * q + 3] = av.w;
                    ahi[4 * q] = hv.x, ahi[4 * q + 1] = hv.y, ahi[4 * q + 2] = hv.z, ahi[4 * q + 3] = hv.w;
                    as_[4 * q] = sv.x, as_[4 * q + 1] = sv.y, as_[4 * q + 2] = sv.z, as_[4 * q + 3] = sv.w;
                }
            } else {
                static_assert(TM == 2, "two rows per thread");
                const uint2 av = *reinterpret_cast<const uint2 *>(&cur.a_abs[k][ty * TM]);
                const uint2 hv = *reinterpret_cast<const uint2 *>(&cur.a_hi[k][ty * TM]);
                const int2 sv = *reinterpret_cast<const int2 *>(&cur.a_sgn[k][ty * TM]);
                aa[0] = av.x, aa[1] = av.y;
                ahi[0] = hv.x, ahi[1] = hv.y;
                as_[0] = sv.x, as_[1] = sv.y;
            }
            uint32_t ba[CT];
            int32_t bs_[CT];
            if constexpr (CT == 4) {
                const uint4 bv = *reinterpret_cast<const uint4 *>(&cur.b_abs[k][tx * CT]);
                const int4 bs = *reinterpret_cast<const int4 *>(&cur.b_sgn[k][tx * CT]);
                ba[0] = bv.x, ba[1] = bv.y, ba[2] = bv.z, ba[3] = bv.w;
                bs_[0] = bs.x, bs_[1] = bs.y, bs_[2] = bs.z, bs_[3] = bs.w;
            } else {
                const uint2 bv = *reinterpret_cast<const uint2 *>(&cur.b_abs[k][tx * CT]);
                const int2 bs = *reinterpret_cast<const int2 *>(&cur.b_sgn[k][tx * CT]);
                ba[0] = bv.x, ba[1] = bv.y;
                bs_[0] = bs.x, bs_[1] = bs.y;
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < CT; j++) {
                    const uint32_t t = __umulhi(ahi[i], ba[j]);
                    um[i][j] = min(um[i][j], aa[i] * ba[j] + 0xFFFFFFFFu);
                    const int32_t s = (int32_t)t * (as_[i] * bs_[j]) + acc[i][j];
                    const int32_t c = clampi(s, -w.M, w.M);
                    ov[i][j] |= (uint32_t)(s ^ c);
                    acc[i][j] = c;
                }
        }
        // the other buffer was last read before the previous barrier
        if (kt + 1 < nk) store_regs(st[(kt + 1) & 1]);
        __syncthreads();
    }

    Counts cnt;
    const uint32_t unit_m1 = (1u << w.sh) - 1u;   // um < 2^(N-1) - 1  <=>  some 0 < p < 2^(N-1)
#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int gm = m0 + ty * TM + i;
#pragma unroll
        for (int j = 0; j < CT; j++) {
            const int gn = n0 + tx * CT + j;
            if (gm < M && gn < N)
                emit(e, w, z * so + (int64_t)gm * N + gn, gn, acc[i][j], ov[i][j] != 0, um[i][j] < unit_m1, cnt);
        }
    }
    flush_counts(cnt, counts, sc);
}

constexpr int PK_BN = 128, PK_BK = 32, PK_TP = 4;   // PK_TP lane pairs (8 columns) per thread

template <int BM>
struct PkStage {
    uint32_t a_mag[PK_BK][BM];            // |a|
    uint32_t a_add[PK_BK][BM];            // (0x7FFF + [a == 0]) << 16
    uint32_t a_sgn[PK_BK][BM];            // 0 or 0xFFFFFFFF
    uint32_t b_mag[PK_BK][PK_BN];         // |b| << (17 - N)
    uint32_t b_sgn[PK_BK][PK_BN / 2];     // 0xFFFF per negative lane
    uint32_t b_zero[PK_BK][PK_BN / 2];    // 0xFFFF per zero lane
    uint32_t a_w[BM];                     // bit k: a < 0 or a == 0
    uint32_t b_w[PK_BN];                  // bit k: b < 0
};

template <int TM, int NT>
constexpr int pk_smem() { return 2 * (int)sizeof(PkStage<TM * NT / 16>); }

// NT threads with TM rows each: a CTA owns a (TM NT / 16) x 128 tile, one CTA
// per SM.  The running sums are added with an IMAD by a runtime one, which
// keeps that add on the FMA pipe beside the two product IMADs while the byte
// permute and the two LOP3s use the ALU pipe.
template <int TM, int NT>
__global__ void __launch_bounds__(NT, 1) chain_pk_kernel(const int16_t *__restrict__ A,
                                                         const int16_t *__restrict__ B, int M, int N, int K,
                                                         int64_t lda, int64_t ldb, int64_t sa, int64_t sb, int64_t so,
                                                         Width w, Epi e, int vec, uint32_t one, sfb_counts *counts) {
    constexpr int PK_TM = TM, PK_BM = TM * NT / 16;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    PkStage<PK_BM> *st = reinterpret_cast<PkStage<PK_BM> *>(smem_raw);
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;               // lane pairs tx*4.., rows ty*TM..
    const int m0 = blockIdx.y * PK_BM, n0 = blockIdx.x * PK_BN;
    const int64_t z = blockIdx.z;
    A += z * sa;
    B += z * sb;
    const int bshift = 17 - w.bits;
    const int nk = (K + PK_BK - 1) / PK_BK;

    uint32_t acc[PK_TM][PK_TP], uf[PK_TM][PK_TP];
    const uint32_t acc0 = 0u - (uint32_t)nk * (32u * 0x7FFFu * 0x10001u);
#pragma unroll
    for (int i = 0; i < PK_TM; i++)
#pragma unroll
        for (int p = 0; p < PK_TP; p++) acc[i][p] = acc0, uf[i][p] = 0xFFFFFFFFu;

    // loaders: A row tid / TPR, PER k from (tid % TPR) * PER; B k-row tid / TPB, BPER columns from
    // (tid % TPB) * BPER
    constexpr int TPR = NT / PK_BM, PER = PK_BK / TPR;
    constexpr int NTB = NT < 512 ? 256 : 512;               // threads that load B
    constexpr int BPER = PK_BK * PK_BN / NTB, TPB = PK_BN / BPER;
    static_assert(PER % 8 == 0 && BPER % 8 == 0 && NT % PK_BM == 0 && NT >= NTB, "loader widths");
    const int ar = tid / TPR, ak = (tid % TPR) * PER;
    const int bk = tid / TPB, bc = (tid % TPB) * BPER;
    const bool bload = tid < NTB;
    Pack8 ra[PER / 8], rb[BPER / 8];
    auto load_regs = [&](int k0) {
        const int gm = m0 + ar;
#pragma unroll
        for (int q = 0; q < PER / 8; q++) {
            const int kq = k0 + ak + q * 8;
            if (vec && gm < M && kq + 8 <= K) {
                ra[q].u = __ldg(reinterpret_cast<const uint4 *>(A + (int64_t)gm * lda + kq));
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++)
                    ra[q].h[j] = (gm < M && kq + j < K) ? A[(int64_t)gm * lda + kq + j] : (int16_t)0;
            }
        }
        const int gk = k0 + bk;
#pragma unroll
        for (int q = 0; q < BPER / 8; q++) {
            const int gn = n0 + bc + q * 8;
            if (!bload) continue;
            if (vec && gk < K && gn + 8 <= N) {
                rb[q].u = __ldg(reinterpret_cast<const uint4 *>(B + (int64_t)gk * ldb + gn));
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++)
                    rb[q].h[j] = (gk < K && gn + j < N) ? B[(int64_t)gk * ldb + gn + j] : (int16_t)0;
            }
        }
    };
    auto store_regs = [&](PkStage<PK_BM> &s) {
        uint32_t bits = 0;
#pragma unroll
        for (int q = 0; q < PER / 8; q++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int v = ra[q].h[j];
                const int kk = ak + q * 8 + j;
                s.a_mag[kk][ar] = (uint32_t)abs(v);
                s.a_add[kk][ar] = (0x7FFFu + (uint32_t)(v == 0)) << 16;
                s.a_sgn[kk][ar] = (uint32_t)(v >> 31);
                bits |= (uint32_t)(v <= 0) << kk;
            }
#pragma unroll
        for (int o = 1; o < TPR; o <<= 1) bits |= __shfl_xor_sync(0xffffffffu, bits, o);
        if (tid % TPR == 0) s.a_w[ar] = bits;
#pragma unroll
        for (int q = 0; q < BPER / 8; q++) {
            if (!bload) continue;
            uint32_t mag[8];
#pragma unroll
            for (int j = 0; j < 8; j++) mag[j] = (uint32_t)abs((int)rb[q].h[j]) << bshift;
            *reinterpret_cast<uint4 *>(&s.b_mag[bk][bc + q * 8]) = make_uint4(mag[0], mag[1], mag[2], mag[3]);
            *reinterpret_cast<uint4 *>(&s.b_mag[bk][bc + q * 8 + 4]) = make_uint4(mag[4], mag[5], mag[6], mag[7]);
            uint32_t sg[4], zr[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int lo = rb[q].h[2 * j], hi = rb[q].h[2 * j + 1];
                sg[j] = (lo < 0 ? 0xFFFFu : 0u) | (hi < 0 ? 0xFFFF0000u : 0u);
                zr[j] = (lo == 0 ? 0xFFFFu : 0u) | (hi == 0 ? 0xFFFF0000u : 0u);
            }
            *reinterpret_cast<uint4 *>(&s.b_sgn[bk][(bc + q * 8) / 2]) = make_uint4(sg[0], sg[1], sg[2], sg[3]);
            *reinterpret_cast<uint4 *>(&s.b_zero[bk][(bc + q * 8) / 2]) = make_uint4(zr[0], zr[1], zr[2], zr[3]);
        }
    };

    if (nk > 0) {
        load_regs(0);
        store_regs(st[0]);
    }
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        PkStage<PK_BM> &cur = st[kt & 1];
        if (tid < PK_BN) {                    // column sign words of this k-tile
            const uint32_t lane_bit = (tid & 1) ? 31u : 15u;
            uint32_t bits = 0;
#pragma unroll 8
            for (int k = 0; k < PK_BK; k++) bits |= ((cur.b_sgn[k][tid >> 1] >> lane_bit) & 1u) << k;
            cur.b_w[tid] = bits;
        }
        if (kt + 1 < nk) load_regs((kt + 1) * PK_BK);
        __syncthreads();
#pragma unroll 2
        for (int k = 0; k < PK_BK; k++) {
            uint32_t am[PK_TM], ad[PK_TM], as_[PK_TM];
#pragma unroll
            for (int q = 0; q < PK_TM / 4; q++) {
                const uint4 m4 = *reinterpret_cast<const uint4 *>(&cur.a_mag[k][ty * PK_TM + 4 * q]);
                const uint4 d4 = *reinterpret_cast<const uint4 *>(&cur.a_add[k][ty * PK_TM + 4 * q]);
                const uint4 s4 = *reinterpret_cast<const uint4 *>(&cur.a_sgn[k][ty * PK_TM + 4 * q]);
                am[4 * q] = m4.x, am[4 * q + 1] = m4.y, am[4 * q + 2] = m4.z, am[4 * q + 3] = m4.w;
                ad[4 * q] = d4.x, ad[4 * q + 1] = d4.y, ad[4 * q + 2] = d4.z, ad[4 * q + 3] = d4.w;
                as_[4 * q] = s4.x, as_[4 * q + 1] = s4.y, as_[4 * q + 2] = s4.z, as_[4 * q + 3] = s4.w;
            }
            const uint4 bm0 = *reinterpret_cast<const uint4 *>(&cur.b_mag[k][tx * 2 * PK_TP]);
            const uint4 bm1 = *reinterpret_cast<const uint4 *>(&cur.b_mag[k][tx * 2 * PK_TP + 4]);
            const uint4 bs4 = *reinterpret_cast<const uint4 *>(&cur.b_sgn[k][tx * PK_TP]);
            const uint4 bz4 = *reinterpret_cast<const uint4 *>(&cur.b_zero[k][tx * PK_TP]);
            const uint32_t bm[2 * PK_TP] = {bm0.x, bm0.y, bm0.z, bm0.w, bm1.x, bm1.y, bm1.z, bm1.w};
            const uint32_t bs[PK_TP] = {bs4.x, bs4.y, bs4.z, bs4.w};
            const uint32_t bz[PK_TP] = {bz4.x, bz4.y, bz4.z, bz4.w};
#pragma unroll
            for (int i = 0; i < PK_TM; i++)
#pragma unroll
                for (int p = 0; p < PK_TP; p++) {
                    const uint32_t plo = am[i] * bm[2 * p] + ad[i];
                    const uint32_t phi = am[i] * bm[2 * p + 1] + ad[i];
                    const uint32_t pk2 = __byte_perm(plo, phi, 0x7632);
                    acc[i][p] = (pk2 ^ as_[i] ^ bs[p]) * one + acc[i][p];
                    uf[i][p] &= pk2 | bz[p];
                }
        }
#pragma unroll
        for (int i = 0; i < PK_TM; i++) {
            const uint32_t wa = cur.a_w[ty * PK_TM + i];
#pragma unroll
            for (int p = 0; p < PK_TP; p++) {
                const uint32_t nlo = __popc(wa ^ cur.b_w[tx * 2 * PK_TP + 2 * p]);
                const uint32_t nhi = __popc(wa ^ cur.b_w[tx * 2 * PK_TP + 2 * p + 1]);
                acc[i][p] -= nlo + (nhi << 16);
            }
        }
        if (kt + 1 < nk) store_regs(st[(kt + 1) & 1]);
        __syncthreads();
    }

    Counts cnt;
    unsigned bad = 0;
    // The converted layer's float output (one of y32 / y64, no codes or flags)
    // is staged through shared memory, free once the last k-tile is done, and
    // written out a row at a time by whole warps: a thread's own outputs are
    // 8 consecutive columns of 8 rows, which stored directly leave every
    // 32-byte sector of a row to 4-byte writes from several store instructions.
    const bool stage = (e.y32 != nullptr) != (e.y64 != nullptr) && !e.codes && !e.flags;
    constexpr int SROW = PK_BN + 4;                       // floats per staged row (16-byte aligned rows)
    constexpr int DROW = PK_BN + 2;                       // doubles per staged row
    static_assert(PK_BM * DROW * 8 <= (int)sizeof(PkStage<PK_BM>) * 2, "staged tile fits the stages");
    float *tile32 = reinterpret_cast<float *>(smem_raw);
    double *tile64 = reinterpret_cast<double *>(smem_raw);
    const double ascale = (e.y32 || e.y64) ? (e.a_dev ? __ldg(e.a_dev) : e.a) : 0.0;
#pragma unroll
    for (int i = 0; i < PK_TM; i++) {
        const int rl = ty * PK_TM + i, gm = m0 + rl;
        double yv[2 * PK_TP];
#pragma unroll
        for (int p = 0; p < PK_TP; p++) {
            const int lo = (int)(int16_t)(acc[i][p] & 0xFFFFu);
            const int hi = ((int)acc[i][p] - lo) >> 16;
#pragma unroll
            for (int l = 0; l < 2; l++) {
                const int gn = n0 + tx * 2 * PK_TP + 2 * p + l;
                yv[2 * p + l] = 0.0;
                if (gm < M && gn < N) {
                    int v = l ? hi : lo;
                    if (v > w.M || v < -w.M) {                // the caller's proof did not hold
                        bad++;
                        v = clampi(v, -w.M, w.M);
                    }
                    const bool un = ((uf[i][p] >> (15 + 16 * l)) & 1u) == 0;
                    if (stage) {
                        bool o = false;
                        if (e.bias) {
                            const int sum = v + (int)e.bias[gn];
                            o = sum > w.M || sum < -w.M;
                            v = clampi(sum, -w.M, w.M);
                        }
                        yv[2 * p + l] = (double)v / (double)(1 << w.sh) * ascale * e.s_col[gn];
                        cnt.over += o;
                        cnt.under += un;
                    } else {
                        emit(e, w, z * so + (int64_t)gm * N + gn, gn, v, false, un, cnt);
                    }
                }
            }
        }
        if (stage) {
            if (e.y32) {
                float4 *d = reinterpret_cast<float4 *>(tile32 + rl * SROW + tx * 2 * PK_TP);
                d[0] = make_float4((float)yv[0], (float)yv[1], (float)yv[2], (float)yv[3]);
                d[1] = make_float4((float)yv[4], (float)yv[5], (float)yv[6], (float)yv[7]);
            } else {
                double2 *d = reinterpret_cast<double2 *>(tile64 + rl * DROW + tx * 2 * PK_TP);
#pragma unroll
                for (int q = 0; q < PK_TP; q++) d[q] = make_double2(yv[2 * q], yv[2 * q + 1]);
            }
        }
    }
    if (stage) {
        __syncthreads();
        const int warp = tid >> 5, lane = tid & 31;
        for (int rl = warp; rl < PK_BM; rl += NT / 32) {
            const int gm = m0 + rl;
            if (gm >= M) break;
            const int64_t base = z * so + (int64_t)gm * N + n0;
#pragma unroll
            for (int c = lane; c < PK_BN; c += 32) {
                if (n0 + c < N) {
                    if (e.y32) e.y32[base + c] = tile32[rl * SROW + c];
                    else e.y64[base + c] = tile64[rl * DROW + c];
                }
            }
        }
    }
    if (bad && counts) atomicAdd(&counts->reserved[1], (unsigned long long)bad);
    flush_counts(cnt, counts, sc);
}

// --- general mode with K split across CTAs ---------------------------------------------------
//
// For few output tiles the general chain leaves SMs idle.  Each step
// v -> clip(v + t, -M, M) is a clamp-add map; a run of steps composes to
// v -> clip(v + s, lo, hi), and the run is clip-free for an entry v exactly
// when v + P stays in [-M, M] for every prefix sum P, i.e. v in
// [-M - pmin, M - pmax]; these compose in order (s adds, lo / hi clamp
// through the later run, pmax = max(pmaxA, sA + pmaxB), likewise pmin).  So
// each CTA summarises one piece of K for its 64 x 64 tile, and a second
// kernel composes the pieces in order from v = 0: the value is clip(s, lo,
// hi), overflow is pmax > M or pmin < -M, underflow (a nonzero product
// truncating to 0) is an OR.  The same bits as the sequential chain.

struct Piece {
    int s, lo, hi, pmax, pmin, under;
};

template <bool BITS16>
__global__ void __launch_bounds__(THREADS, 1) chain_piece_kernel(const int16_t *__restrict__ A,
                                                                 const int16_t *__restrict__ B, int M, int N, int K,
                                                                 int64_t lda, int64_t ldb, int kspan, Width w0,
                                                                 int vec, Piece *__restrict__ ws) {
    constexpr int TM = 4, BM = 64;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    Stage<BM> *st = reinterpret_cast<Stage<BM> *>(smem_raw);
    const Width w = BITS16 ? Width{16, 15, 32767} : w0;
    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN), ty = tid / (BN / TN);
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int piece = blockIdx.z;
    const int kbeg = piece * kspan, kend = min(K, kbeg + kspan);
    int sum[TM][TN], lo[TM][TN], hi[TM][TN], pmax[TM][TN], pmin[TM][TN];
    uint32_t um[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++)
            sum[i][j] = 0, lo[i][j] = -(1 << 30), hi[i][j] = 1 << 30, pmax[i][j] = -(1 << 30),
            pmin[i][j] = 1 << 30, um[i][j] = 0xFFFFFFFFu;

    constexpr int TPR = THREADS / BM, PER = BK / TPR;
    const int ar = tid / TPR, ah = tid % TPR;
    const int bk = tid >> 3, bc = (tid & 7) * 8;
    Pack8 ra[PER / 8], rb;
    auto load_regs = [&](int k0) {
        const int gm = m0 + ar;
        const int ka = k0 + ah * PER;
#pragma unroll
        for (int q = 0; q < PER / 8; q++) {
            const int kq = ka + q * 8;
            if (vec && gm < M && kq + 8 <= kend) {
                ra[q].u = __ldg(reinterpret_cast<const uint4 *>(A + (int64_t)gm * lda + kq));
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++)
                    ra[q].h[j] = (gm < M && kq + j < kend) ? A[(int64_t)gm * lda + kq + j] : (int16_t)0;
            }
        }
        const int gk = k0 + bk, gn0 = n0 + bc;
        if (vec && gk < kend && gn0 + 8 <= N) {
            rb.u = __ldg(reinterpret_cast<const uint4 *>(B + (int64_t)gk * ldb + gn0));
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++)
                rb.h[j] = (gk < kend && gn0 + j < N) ? B[(int64_t)gk * ldb + gn0 + j] : (int16_t)0;
        }
    };
    auto store_regs = [&](Stage<BM> &sg) {
#pragma unroll
        for (int q = 0; q < PER / 8; q++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int v = ra[q].h[j];
                const int kk = ah * PER + q * 8 + j;
                sg.a_abs[kk][ar] = (uint32_t)abs(v);
                sg.a_sgn[kk][ar] = v >> 31;
            }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int v = rb.h[j];
            sg.b_abs[bk][bc + j] = (uint32_t)abs(v);
            sg.b_sgn[bk][bc + j] = v >> 31;
        }
    };

    const int nk = (kend - kbeg + BK - 1) / BK;
    if (nk > 0) {
        load_regs(kbeg);
        store_regs(st[0]);
    }
    __syncthreads();
    for (int kt = 0; kt < nk; kt++) {
        Stage<BM> &cur = st[kt & 1];
        if (kt + 1 < nk) load_regs(kbeg + (kt + 1) * BK);
        const int kn = min(BK, kend - (kbeg + kt * BK));     // padded steps are skipped: they are not in the chain
        for (int k = 0; k < kn; k++) {
            uint32_t aa[TM], ba[TN];
            int32_t as_[TM], bs_[TN];
#pragma unroll
            for (int i = 0; i < TM; i++) aa[i] = cur.a_abs[k][ty * TM + i], as_[i] = cur.a_sgn[k][ty * TM + i];
#pragma unroll
            for (int j = 0; j < TN; j++) ba[j] = cur.b_abs[k][tx * TN + j], bs_[j] = cur.b_sgn[k][tx * TN + j];
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) {
                    const uint32_t p = aa[i] * ba[j];
                    const int32_t sg = as_[i] ^ bs_[j];
                    const int32_t t = (((int32_t)(p >> w.sh)) ^ sg) - sg;
                    um[i][j] = min(um[i][j], p - 1u);
                    sum[i][j] += t;
                    pmax[i][j] = max(pmax[i][j], sum[i][j]);
                    pmin[i][j] = min(pmin[i][j], sum[i][j]);
                    lo[i][j] = clampi(lo[i][j] + t, -w.M, w.M);
                    hi[i][j] = clampi(hi[i][j] + t, -w.M, w.M);
                }
        }
        if (kt + 1 < nk) store_regs(st[(kt + 1) & 1]);
        __syncthreads();
    }
    const uint32_t unit_m1 = (1u << w.sh) - 1u;
#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int gm = m0 + ty * TM + i;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int gn = n0 + tx * TN + j;
            if (gm < M && gn < N)
                ws[((int64_t)piece * M + gm) * N + gn] =
                    Piece{sum[i][j], lo[i][j], hi[i][j], pmax[i][j], pmin[i][j], um[i][j] < unit_m1 ? 1 : 0};
        }
    }
}

__global__ void __launch_bounds__(256) chain_combine_kernel(const Piece *__restrict__ ws, int pieces, int M, int N,
                                                            Width w, Epi e, sfb_counts *counts) {
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    Counts cnt;
    const int64_t total = (int64_t)M * N;
    for (int64_t o = (int64_t)blockIdx.x * 256 + threadIdx.x; o < total; o += (int64_t)gridDim.x * 256) {
        long long s = 0, lo = -(1ll << 62), hi = 1ll << 62, pmax = -(1ll << 62), pmin = 1ll << 62;
        int under = 0;
        for (int p = 0; p < pieces; p++) {
            const Piece b = ws[(int64_t)p * total + o];
            if (b.pmax == -(1 << 30)) continue;                 // an empty piece (the identity)
            lo = lo + b.s < b.lo ? b.lo : (lo + b.s > b.hi ? b.hi : lo + b.s);
            hi = hi + b.s < b.lo ? b.lo : (hi + b.s > b.hi ? b.hi : hi + b.s);
            pmax = max(pmax, s + b.pmax);
            pmin = min(pmin, s + b.pmin);
            s += b.s;
            under |= b.under;
        }
        const int v = (int)(s < lo ? lo : (s > hi ? hi : s));
        const bool over = pmax > w.M || pmin < -w.M;
        const int gn = (int)(o % N);
        emit(e, w, o, gn, v, over, under != 0, cnt);
    }
    flush_counts(cnt, counts, sc);
}

// pieces for a general chain of few tiles (1: no split)
int chain_pieces(int64_t batch, int64_t M, int64_t N, int64_t K) {
    if (batch != 1 || K < 4 * BK) return 1;
    // enough 32 x 64 tiles to occupy most SMs: the plain chain beats the pieces' summaries
    if (((M + 31) / 32) * ((N + BN - 1) / BN) >= (int64_t)sm_count() / 2) return 1;
    const int64_t tiles = ((M + 63) / 64) * ((N + BN - 1) / BN);
    const int64_t want = (2 * (int64_t)sm_count() + tiles - 1) / tiles;            // one wave at 2 CTAs per SM
    const int64_t most = std::max<int64_t>(1, K / (2 * BK));
    const int64_t p = std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(want, most), 16));
    // a piece sums at most 2^15 products in int32 (|sum| < 2^30, below the empty-piece marker)
    return (K + p - 1) / p <= 32768 - BK ? (int)p : 1;
}

int launch_chain(int bits, const int16_t *A, const int16_t *B, const Epi &e, int64_t batch, int64_t M, int64_t N,
                 int64_t K, int64_t lda, int64_t ldb, int64_t sa, int64_t sb, int64_t so, bool safe,
                 sfb_counts *counts, cudaStream_t st, const char *what) {
    constexpr int TMP = 8, NTP = 384;            // proven mode: 192 x 128 tiles, 12 warps per SM
    const int BM = safe ? TMP * NTP / 16 : 64, BNL = safe ? PK_BN : BN;
    const int64_t mt = (M + BM - 1) / BM, nt = (N + BNL - 1) / BNL;
    if (mt > 65535 || nt > 0x7fffffff || batch > 65535 || K > 0x7fffffff || M > 0x7fffffff || N > 0x7fffffff)
        return set_error(SFB_ERANGE, "%s: %lld x %lld x %lld (batch %lld) exceeds the launch limits", what,
                         (long long)M, (long long)N, (long long)K, (long long)batch);
    dim3 grid((unsigned)nt, (unsigned)mt, (unsigned)batch);
    // shared-memory limits set once per CUDA context (a device reset starts a new one)
    static unsigned long long attr[64][3] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    const unsigned long long ctx = context_id();
    const Width w = width(bits);
    const int vec = (lda % 8 == 0) && (ldb % 8 == 0) && ((uintptr_t)A % 16 == 0) && ((uintptr_t)B % 16 == 0) &&
                    (sa % 8 == 0) && (sb % 8 == 0);
    if (safe) {
        if (ctx == 0 || attr[dev][2] != ctx) {
            if (cudaFuncSetAttribute(chain_pk_kernel<TMP, NTP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     pk_smem<TMP, NTP>()) != cudaSuccess)
                return check_launch(what);
            attr[dev][2] = context_id();
        }
        chain_pk_kernel<TMP, NTP><<<grid, NTP, pk_smem<TMP, NTP>(), st>>>(A, B, (int)M, (int)N, (int)K, lda, ldb, sa,
                                                                          sb, so, w, e, vec, 1u, counts);
        return check_launch(what);
    }
    const bool b16 = bits == 16;
    if (batch * ((M + 31) / 32) * nt < (int64_t)sm_count()) {
        // so few outputs that 32 x 64 tiles would not give every SM one: 32-column tiles,
        // 32 x 32 (four rows per thread) while they still give every SM a CTA, else
        // 16 x 32 while those give half the SMs one, else 8 x 32 on 64-thread CTAs
        // (each under the default 48 KB of dynamic shared memory)
        static_assert(2 * sizeof(GStage<32, 32>) <= 48 * 1024, "default dynamic shared memory");
        const int64_t n32 = (N + 31) / 32, sms = sm_count();
        if (batch * ((M + 31) / 32) * n32 >= sms) {
            const dim3 g((unsigned)n32, (unsigned)((M + 31) / 32), (unsigned)batch);
            auto kern = b16 ? chain2_kernel<true, 4, 128, 32, 2> : chain2_kernel<false, 4, 128, 32, 2>;
            kern<<<g, 128, 2 * sizeof(GStage<32, 32>), st>>>(A, B, (int)M, (int)N, (int)K, lda, ldb, sa, sb, so, w,
                                                             e, vec, counts);
        } else if (batch * ((M + 15) / 16) * n32 >= sms / 2) {
            const dim3 g((unsigned)n32, (unsigned)((M + 15) / 16), (unsigned)batch);
            auto kern = b16 ? chain2_kernel<true, 2, 128, 32, 2> : chain2_kernel<false, 2, 128, 32, 2>;
            kern<<<g, 128, 2 * sizeof(GStage<16, 32>), st>>>(A, B, (int)M, (int)N, (int)K, lda, ldb, sa, sb, so, w,
                                                             e, vec, counts);
        } else {
            const dim3 g((unsigned)n32, (unsigned)((M + 7) / 8), (unsigned)batch);
            auto kern = b16 ? chain2_kernel<true, 2, 64, 32, 2> : chain2_kernel<false, 2, 64, 32, 2>;
            kern<<<g, 64, 2 * sizeof(GStage<8, 32>), st>>>(A, B, (int)M, (int)N, (int)K, lda, ldb, sa, sb, so, w, e,
                                                           vec, counts);
        }
        return check_launch(what);
    }
    if (batch * mt * nt < 2 * (int64_t)sm_count()) {
        // few 64 x 64 tiles: 32 x 64 tiles on 128-thread CTAs, twice the CTAs
        const dim3 g2((unsigned)nt, (unsigned)((M + 31) / 32), (unsigned)batch);
        const int smem = 2 * (int)sizeof(GStage<32>);
        auto kern = b16 ? chain2_kernel<true, 4, 128> : chain2_kernel<false, 4, 128>;
        static unsigned long long attr_s[64][2] = {};
        if (ctx == 0 || attr_s[dev][b16] != ctx) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
                return check_launch(what);
            attr_s[dev][b16] = context_id();
        }
        kern<<<g2, 128, smem, st>>>(A, B, (int)M, (int)N, (int)K, lda, ldb, sa, sb, so, w, e, vec, counts);
        return check_launch(what);
    }
    const int smem = 2 * (int)sizeof(GStage<64>);
    auto kern = b16 ? chain2_kernel<true, 4> : chain2_kernel<false, 4>;
    if (ctx == 0 || attr[dev][b16] != ctx) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_launch(what);
        attr[dev][b16] = context_id();
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
    Epi e{bias, 0.0, nullptr, nullptr, nullptr, nullptr, out, flags};
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
    Epi e{bias, a, nullptr, s_col, y32, y64, codes, flags};
    return launch_chain(bits, X, WT, e, 1, R, N, K, ldx, ldw, 0, 0, R * N, proven_no_saturation != 0, counts,
                        (cudaStream_t)stream, "sfb_linear_chain");
}

extern "C" int sfb_linear_chain_dev(int bits, const int16_t *X, const int16_t *WT, const int16_t *bias,
                                    const double *a_dev, const double *s_col, float *y32, double *y64,
                                    int16_t *codes, uint8_t *flags, int64_t R, int64_t N, int64_t K, int64_t ldx,
                                    int64_t ldw, sfb_counts *counts, sfb_stream stream) {
    using namespace sfb;
    int rc = chain_args("sfb_linear_chain_dev", bits, X, WT, 1, R, N, K, ldx, ldw, R * N);
    if (rc) return rc;
    if (R == 0 || N == 0) return SFB_OK;
    if (a_dev == nullptr) return set_error(SFB_EINVAL, "sfb_linear_chain_dev: null scale");
    if ((y32 || y64) && s_col == nullptr) return set_error(SFB_EINVAL, "sfb_linear_chain_dev: y needs s_col");
    if (!y32 && !y64 && !codes) return set_error(SFB_EINVAL, "sfb_linear_chain_dev: no output requested");
    Epi e{bias, 0.0, a_dev, s_col, y32, y64, codes, flags};
    return launch_chain(bits, X, WT, e, 1, R, N, K, ldx, ldw, 0, 0, R * N, true, counts, (cudaStream_t)stream,
                        "sfb_linear_chain_dev");
}

extern "C" int64_t sfb_matmul_chain_workspace(int64_t batch, int64_t M, int64_t N, int64_t K) {
    using namespace sfb;
    if (batch < 0 || M < 0 || N < 0 || K < 0) return set_error(SFB_EINVAL, "sfb_matmul_chain_workspace: bad size");
    const int p = chain_pieces(batch, M, N, K);
    return p > 1 ? (int64_t)p * M * N * (int64_t)sizeof(Piece) : 0;
}

extern "C" int sfb_matmul_chain_ws(int bits, const int16_t *A, const int16_t *B, const int16_t *bias, int16_t *out,
                                   uint8_t *flags, int64_t batch, int64_t M, int64_t N, int64_t K, int64_t lda,
                                   int64_t ldb, int64_t stride_a, int64_t stride_b, int64_t stride_out,
                                   void *workspace, int64_t workspace_bytes, sfb_counts *counts, sfb_stream stream) {
    using namespace sfb;
    int rc = chain_args("sfb_matmul_chain_ws", bits, A, B, batch, M, N, K, lda, ldb, stride_out);
    if (rc) return rc;
    if (batch == 0 || M == 0 || N == 0) return SFB_OK;
    if (out == nullptr) return set_error(SFB_EINVAL, "sfb_matmul_chain_ws: null output");
    Epi e{bias, 0.0, nullptr, nullptr, nullptr, nullptr, out, flags};
    cudaStream_t st = (cudaStream_t)stream;
    const int pieces = chain_pieces(batch, M, N, K);
    const int64_t need = pieces > 1 ? (int64_t)pieces * M * N * (int64_t)sizeof(Piece) : 0;
    if (pieces <= 1 || workspace == nullptr || workspace_bytes < need || M > 0x7fffffff || N > 0x7fffffff)
        return launch_chain(bits, A, B, e, batch, M, N, K, lda, ldb, stride_a, stride_b, stride_out, false, counts,
                            st, "sfb_matmul_chain_ws");
    const int kspan = (int)(((K + pieces - 1) / pieces + BK - 1) / BK * BK);
    const int np = (int)((K + kspan - 1) / kspan);
    const Width w = width(bits);
    const int vec = (lda % 8 == 0) && (ldb % 8 == 0) && ((uintptr_t)A % 16 == 0) && ((uintptr_t)B % 16 == 0);
    const int smem = 2 * (int)sizeof(Stage<64>);
    auto kern = bits == 16 ? chain_piece_kernel<true> : chain_piece_kernel<false>;
    static unsigned long long attr[64][2] = {};      // set once per CUDA context
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    const unsigned long long ctx = context_id();
    if (ctx == 0 || attr[dev][bits == 16] != ctx) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_launch("sfb_matmul_chain_ws");
        attr[dev][bits == 16] = context_id();
    }
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + 63) / 64), (unsigned)np);
    Piece *ws = reinterpret_cast<Piece *>(workspace);
    kern<<<grid, THREADS, smem, st>>>(A, B, (int)M, (int)N, (int)K, lda, ldb, kspan, w, vec, ws);
    rc = check_launch("sfb_matmul_chain_ws (pieces)");
    if (rc) return rc;
    const int64_t g = std::min<int64_t>((M * N + 255) / 256, (int64_t)sm_count() * 8);
    chain_combine_kernel<<<(unsigned)std::max<int64_t>(g, 1), 256, 0, st>>>(ws, np, (int)M, (int)N, w, e, counts);
    return check_launch("sfb_matmul_chain_ws (combine)");
}
