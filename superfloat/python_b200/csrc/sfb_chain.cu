// Chain matmul on sm_100a CUDA cores (the INT32 pipe).
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
// add (src/sf/torch/_core.py:376-378), whose overflow joins the output's.
//
// Tiling: a 256-thread block owns a 64 x 64 output tile, 4 x 4 outputs per
// thread; A and B stream through shared memory in k-tiles of 32 (zero
// padding past K is neutral: a 0 product changes nothing and raises nothing).
#include "sfb_common.cuh"

namespace sfb {
namespace {

constexpr int BM = 64, BN = 64, BK = 32, TM = 4, TN = 4, THREADS = 256;

template <bool BIAS>
__global__ void __launch_bounds__(THREADS) chain_kernel(const int16_t *__restrict__ A, const int16_t *__restrict__ B,
                                                       const int16_t *__restrict__ bias, int16_t *__restrict__ out,
                                                       uint8_t *__restrict__ flags, int M, int N, int K, int64_t lda,
                                                       int64_t ldb, int64_t sa, int64_t sb, int64_t so, Width w,
                                                       sfb_counts *counts) {
    __shared__ int4 As4[BK][BM / 4];  // As[k][m], m contiguous
    __shared__ int4 Bs4[BK][BN / 4];  // Bs[k][n], n contiguous
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    int *As = reinterpret_cast<int *>(As4);
    int *Bs = reinterpret_cast<int *>(Bs4);

    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN), ty = tid / (BN / TN);
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int64_t z = blockIdx.z;
    A += z * sa;
    B += z * sb;
    out += z * so;
    if (flags) flags += z * so;

    const int Mx = w.M, sh = w.sh;
    int acc[TM][TN];
    unsigned ovw[TM][TN], unw[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = 0, ovw[i][j] = 0, unw[i][j] = 0;

    for (int k0 = 0; k0 < K; k0 += BK) {
        // A tile: 64 rows x 32 k -> As[k][m]; 8 elements per thread
#pragma unroll
        for (int r = 0; r < (BM * BK) / THREADS; r++) {
            const int e = tid + r * THREADS;
            const int mm = e / BK, kk = e % BK;
            const int gm = m0 + mm, gk = k0 + kk;
            As[kk * BM + mm] = (gm < M && gk < K) ? (int)A[(int64_t)gm * lda + gk] : 0;
        }
        // B tile: 32 k x 64 cols -> Bs[k][n]
#pragma unroll
        for (int r = 0; r < (BK * BN) / THREADS; r++) {
            const int e = tid + r * THREADS;
            const int kk = e / BN, nn = e % BN;
            const int gk = k0 + kk, gn = n0 + nn;
            Bs[kk * BN + nn] = (gk < K && gn < N) ? (int)B[(int64_t)gk * ldb + gn] : 0;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < BK; kk++) {
            const int4 av = As4[kk][ty];
            const int4 bv = Bs4[kk][tx];
            const int a_[4] = {av.x, av.y, av.z, av.w};
            const int b_[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) {
                    const int p = a_[i] * b_[j];
                    const int t = tdiv_pow2(p, sh);
                    const int s = acc[i][j] + t;
                    const int c = clampi(s, -Mx, Mx);
                    ovw[i][j] |= (unsigned)(s ^ c);
                    unw[i][j] |= (unsigned)((p != 0) & (t == 0));
                    acc[i][j] = c;
                }
        }
        __syncthreads();
    }

    Counts cnt;
#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int gm = m0 + ty * TM + i;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int gn = n0 + tx * TN + j;
            if (gm < M && gn < N) {
                int v = acc[i][j];
                bool ov = ovw[i][j] != 0;
                if (BIAS) {
                    const int s = v + (int)bias[gn];
                    ov |= (s > Mx || s < -Mx);
                    v = clampi(s, -Mx, Mx);
                }
                const bool un = unw[i][j] != 0;
                out[(int64_t)gm * N + gn] = (int16_t)v;
                if (flags) flags[(int64_t)gm * N + gn] = (uint8_t)((ov ? SFB_F_OVERFLOW : 0u) | (un ? SFB_F_UNDERFLOW : 0u));
                cnt.over += ov;
                cnt.under += un;
            }
        }
    }
    flush_counts(cnt, counts, sc);
}

}  // namespace
}  // namespace sfb

extern "C" int sfb_matmul_chain(int bits, const int16_t *A, const int16_t *B, const int16_t *bias, int16_t *out,
                                uint8_t *flags, int64_t batch, int64_t M, int64_t N, int64_t K, int64_t lda,
                                int64_t ldb, int64_t stride_a, int64_t stride_b, int64_t stride_out,
                                sfb_counts *counts, sfb_stream stream) {
    using namespace sfb;
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "sfb_matmul_chain: width %d is not 4..16", bits);
    if (batch < 0 || M < 0 || N < 0 || K < 0) return set_error(SFB_EINVAL, "sfb_matmul_chain: negative size");
    if (batch == 0 || M == 0 || N == 0) return SFB_OK;
    if (out == nullptr || (K > 0 && (A == nullptr || B == nullptr)))
        return set_error(SFB_EINVAL, "sfb_matmul_chain: null operand or output");
    if (K > 0 && (lda < K || ldb < N)) return set_error(SFB_EINVAL, "sfb_matmul_chain: lda < K or ldb < N");
    if (stride_out < M * N && batch > 1)
        return set_error(SFB_EINVAL, "sfb_matmul_chain: output batch entries overlap");
    const int64_t mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
    if (mt > 65535 || nt > 0x7fffffff || batch > 65535 || K > 0x7fffffff || M > 0x7fffffff || N > 0x7fffffff)
        return set_error(SFB_ERANGE, "sfb_matmul_chain: %lld x %lld x %lld (batch %lld) exceeds the launch limits",
                         (long long)M, (long long)N, (long long)K, (long long)batch);
    dim3 grid((unsigned)nt, (unsigned)mt, (unsigned)batch);
    cudaStream_t st = (cudaStream_t)stream;
    const Width w = width(bits);
    if (bias)
        chain_kernel<true><<<grid, THREADS, 0, st>>>(A, B, bias, out, flags, (int)M, (int)N, (int)K, lda, ldb,
                                                     stride_a, stride_b, stride_out, w, counts);
    else
        chain_kernel<false><<<grid, THREADS, 0, st>>>(A, B, bias, out, flags, (int)M, (int)N, (int)K, lda, ldb,
                                                      stride_a, stride_b, stride_out, w, counts);
    return check_launch("sfb_matmul_chain");
}
