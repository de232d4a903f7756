// Wide (MX v4.9.2) matmul on sm_100a tensor cores: the SF16 block (sf9..sf16).
//
// The SF16-block product of 15-bit magnitudes a, w (src/sf/_linalg.py:190-198)
// is t = (a w + 80 - C) >> 8 with C = C(a mod 64, w mod 64) the dropped
// partial-product columns, C(x, y) = sum_{i<6} x_i ((y << i) mod 64).  Writing
// X = (a w - C) / 64 (an integer), t = (X + 1) >> 2, so with s = +-1 the
// product's sign, r = (X + 1) mod 4 and u = r for a positive product, 3 - r for
// a negative one (s t = (s X + 1 + [s < 0] - u) / 4 either way):
//
//     4 sum_k s t = sum_k s X - (sum_k s) / 2 + 3 K / 2 - sum_k u
//
// over the K padded to a multiple of 128 (padded products are 0 with s = +1).
// * sum s X - (sum s) / 2 is exact integer linear algebra on int8 operands:
//   the left-aligned signed codes k = s a split into limbs k = 256 h + l
//   (h signed, l unsigned) give 4 GEMMs, sum s C = sum_i (s_a bit_i(a))
//   (s_w ((w << i) mod 64)) 6 more, and (+-1) (-+32) sign planes the 11th.
//   They run as tcgen05 kind::i8 MMAs; by scale the sums are D0 = h.h
//   (x 2^16), D1 = h.l + l.h (x 2^8) and D2 = l.l - sum_i bit_i . C_i - 32
//   sum s (x 1; the C planes are stored negated), |D| < 2^31 for K <= 16384,
//   and the output needs only floor(T / 4) mod 2^32 = 2^8 D0 + D1 +
//   floor(D2 / 256) (mod 2^32), T = sum s X - (sum s) / 2.
// * sum u needs r per product: X mod 4 = (P + 2Q) mod 4 over the low bytes x
//   of a and y of w (P = sum_{i<=6} x_i y_{6-i}, Q = sum_{i<=7} x_i y_{7-i}),
//   which splits by the nibbles of x into F(x mod 16) + G(x >> 4), each a sum
//   of x's bits times two-bit words of y's bits.  Bit-sliced over 32 columns,
//   F and G are 16-entry tables of two-bit words per (k, column word), built
//   once per CTA and read by every row; w's sign and the +1 are folded into
//   the tables and a's sign is a mask applied in the same logic ops, so u for
//   32 products is two 64-bit shared-memory reads and a two-bit add (kernel
//   wide_rem_kernel), summed over k in carry-save bit-plane counters.
//
// The sum is the MX accumulator when no chunk of 8 can clip; each output is
// checked against the bound sum_k |t_k| <= min(rowL1 colmax, rowmax colL1)/256
// + K, and an output that fails it is recomputed exactly, chunk by chunk, on
// the CUDA cores (wide_tc_finish_kernel).  POP as in the CUDA-core kernel.
//
// Kernels, in stream order: prep_kernel (A and B operand planes, A's nibble
// records, B's column-sliced bits, L1 / max statistics),
// tc_gemm_kernel (128 x 256 output tiles in two phases, described at the
// kernel), wide_rem_kernel (sum u per output), wide_tc_finish_kernel.  Every
// wait on a barrier is bounded: on timeout a kernel records an error in the
// caller's counters and returns after freeing its TMEM.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "sfb_wide_simt.cuh"

namespace sfb {

int wide_simt(int bits, int mx, const int16_t *A, const int16_t *B, const int8_t *shift_arr, int shift,
              int16_t *out, uint8_t *flags, int64_t batch, int64_t M, int64_t N, int64_t K, int64_t lda,
              int64_t ldb, int64_t sa, int64_t sb, int64_t so, int64_t ssb, int64_t ssm, int64_t ssn,
              sfb_counts *counts, cudaStream_t st, int32_t *acc_out);

namespace {

constexpr int TILE = 128;          // output rows per GEMM tile and K bytes per stage
constexpr int GN = 256;            // output columns per GEMM tile
constexpr int STAGES = 4;
constexpr int GROUP_M = 8;         // row tiles per group of the GEMM's CTA order
constexpr int P1 = 3, P2 = 8;      // MMA passes per 128-k block in the two phases
constexpr int GEMM_THREADS = 192;  // TMA warp, MMA warp, four fold / epilogue warps
constexpr int NPLANES = 9;         // int8 operand planes per matrix
constexpr int STAGE_BYTES = TILE * TILE + GN * TILE;
constexpr int GEMM_SMEM = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int KMAX = 16384;        // |D| < 2^31 up to this K
constexpr unsigned kSpinLimit = 1u << 26;     // polls of one bounded wait, unless the launch gives fewer

// --- PTX wrappers --------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// bounded wait: false after `limit` polls
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned limit = kSpinLimit) {
    for (unsigned i = 0; i < limit; i++)
        if (mbar_try(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand tile in shared memory, 128-byte swizzle: rows of 128 bytes,
// 8-row groups 1024 bytes apart (SBO), the leading offset unused (1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                 // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;       // SBO
    d |= (uint64_t)1 << 46;                 // descriptor version for sm_100
    d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
    return d;
}

// kind::i8 instruction descriptor: s32 accumulate, K-major A and B, M = N = 128
__device__ __forceinline__ uint32_t idesc_i8(int a_signed, int b_signed) {
    return (2u << 4) | ((uint32_t)a_signed << 7) | ((uint32_t)b_signed << 10) | ((uint32_t)(GN >> 3) << 17) |
           ((uint32_t)(TILE >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int32_t (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = (int32_t)r[i];
}

// --- operand preparation ------------------------------------------------------------------
//
// One CTA (256 threads) per 32 rows x 128 k, staged through shared memory so
// that the codes are read with 16-byte loads and every plane row segment
// (128 k = 128 bytes) is written as one full line.  Writes the nine int8
// planes (h, l, bit_0..bit_5, sign +-1 of A; h, l, -C_0..-C_5, sign -+32 of
// B), the row / column L1 norm and maximum of the magnitudes, and for A the
// remainder's per-product record: byte 0 = (x mod 16) | 128 s, byte 1 =
// x >> 4 (x the magnitude's low byte, s its sign), two k per 32-bit word,
// laid out [k / 2][row].  For B the rows of the tile are B's columns (32 of
// them: one column word), and the kernel also writes B's low magnitude byte
// and sign as bit planes sliced over those columns, [k][plane 0..8][word], one
// warp ballot per plane and k.

constexpr int PR = 32, PK = 128;

template <bool IS_A>
__global__ void __launch_bounds__(256) prep_kernel(const int16_t *__restrict__ X, int64_t ld, int rows, int K,
                                                   int rows_pad, int Kp, int bits, uint8_t *__restrict__ planes,
                                                   uint32_t *__restrict__ rec, long long *__restrict__ l1,
                                                   int *__restrict__ mx, uint32_t *__restrict__ bn, int NWt) {
    __shared__ __align__(16) int16_t tile[PR][PK + 8];
    const int tid = threadIdx.x;
    const int r0 = blockIdx.x * PR, k0 = blockIdx.y * PK;
    const bool vec = ((reinterpret_cast<uintptr_t>(X) & 15) == 0) && (ld % 8 == 0);
    if (IS_A) {
        const int rr = tid >> 3, kk = (tid & 7) * 16, r = r0 + rr;
        const int16_t *src = X + (int64_t)r * ld + k0 + kk;
        int16_t v[16];
        if (vec && r < rows && k0 + kk + 16 <= K) {
            *reinterpret_cast<uint4 *>(v) = __ldg(reinterpret_cast<const uint4 *>(src));
            *reinterpret_cast<uint4 *>(v + 8) = __ldg(reinterpret_cast<const uint4 *>(src + 8));
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] = (r < rows && k0 + kk + j < K) ? src[j] : (int16_t)0;
        }
        *reinterpret_cast<uint4 *>(&tile[rr][kk]) = *reinterpret_cast<const uint4 *>(v);
        *reinterpret_cast<uint4 *>(&tile[rr][kk + 8]) = *reinterpret_cast<const uint4 *>(v + 8);
    } else {
        const int kl = tid >> 1, nl = (tid & 1) * 16, k = k0 + kl;
        const int16_t *src = X + (int64_t)k * ld + r0 + nl;
        int16_t v[16];
        if (vec && k < K && r0 + nl + 16 <= rows) {
            *reinterpret_cast<uint4 *>(v) = __ldg(reinterpret_cast<const uint4 *>(src));
            *reinterpret_cast<uint4 *>(v + 8) = __ldg(reinterpret_cast<const uint4 *>(src + 8));
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] = (k < K && r0 + nl + j < rows) ? src[j] : (int16_t)0;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) tile[nl + j][kl] = v[j];
    }
    __syncthreads();

    const int rr = tid >> 3, seg = tid & 7, r = r0 + rr;
    const int sh = 16 - bits;
    uint32_t pw[NPLANES][4];
#pragma unroll
    for (int p = 0; p < NPLANES; p++)
#pragma unroll
        for (int q = 0; q < 4; q++) pw[p][q] = 0;
    long long sum = 0;
    int mval = 0;
    int16_t c16[16];
    *reinterpret_cast<uint4 *>(c16) = *reinterpret_cast<const uint4 *>(&tile[rr][seg * 16]);
    *reinterpret_cast<uint4 *>(c16 + 8) = *reinterpret_cast<const uint4 *>(&tile[rr][seg * 16 + 8]);
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const int code = c16[j];
        const int a = abs(code) << sh;               // 15-bit magnitude as the SF16 block reads it
        const int s = code < 0;
        const int kt = s ? -a : a;
        const uint32_t sh8 = 8 * (j & 3);
        pw[0][j >> 2] |= ((uint32_t)(kt >> 8) & 0xFFu) << sh8;      // h (signed)
        pw[1][j >> 2] |= ((uint32_t)kt & 0xFFu) << sh8;             // l (unsigned)
#pragma unroll
        for (int i = 0; i < 6; i++) {
            int v = IS_A ? ((a >> i) & 1) : -(((a << i) & 63));     // A: bit_i(a); B: -((w << i) mod 64)
            if (s) v = -v;
            pw[2 + i][j >> 2] |= ((uint32_t)v & 0xFFu) << sh8;
        }
        const int sg = IS_A ? (s ? -1 : 1) : (s ? 32 : -32);        // product -32 s
        pw[8][j >> 2] |= ((uint32_t)sg & 0xFFu) << sh8;
        sum += a;
        mval = max(mval, a);
    }
#pragma unroll
    for (int p = 0; p < NPLANES; p++)
        *reinterpret_cast<uint4 *>(planes + ((int64_t)p * rows_pad + r) * Kp + k0 + seg * 16) =
            make_uint4(pw[p][0], pw[p][1], pw[p][2], pw[p][3]);
    // the 8 threads of a row are 8 consecutive lanes
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
        mval = max(mval, __shfl_xor_sync(0xffffffffu, mval, o));
    }
    if (seg == 0 && r < rows_pad) {
        if (sum) atomicAdd(reinterpret_cast<unsigned long long *>(l1 + r), (unsigned long long)sum);
        if (mval) atomicMax(mx + r, mval);
    }
    if (!IS_A) {
        // column-sliced bits: warp w takes k = 16 w .. 16 w + 15 of the tile
        const int lane = tid & 31, w = tid >> 5, nw = r0 / 32;
        for (int kk = 16 * w; kk < 16 * w + 16; kk++) {
            const int code = tile[lane][kk];
            const int y = (abs(code) << sh) & 255;
            uint32_t mine = 0;
#pragma unroll
            for (int p = 0; p < 8; p++) {
                const uint32_t word = __ballot_sync(0xffffffffu, (y >> p) & 1);
                if (lane == p) mine = word;
            }
            const uint32_t sw = __ballot_sync(0xffffffffu, code < 0);
            if (lane == 8) mine = sw;
            if (lane < 9) bn[((int64_t)(k0 + kk) * 9 + lane) * NWt + nw] = mine;
        }
    }
    if (IS_A) {
        // 32 rows x 64 k pairs: a warp writes one k pair for the 32 rows (128 bytes)
        const int ml = tid & 31, g = tid >> 5;
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const int kp = g * 8 + q;
            uint32_t v = 0;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int code = tile[ml][2 * kp + h];
                const int x = (abs(code) << sh) & 255;
                const uint32_t sgn = code < 0 ? 0x80u : 0u;
                v |= (((uint32_t)(x & 15) | sgn) | ((uint32_t)(x >> 4) << 8)) << (16 * h);
            }
            rec[(int64_t)(k0 / 2 + kp) * rows_pad + r0 + ml] = v;
        }
    }
}

// --- the tcgen05 GEMM: floor((sum_k s X - (sum_k s) / 2) / 4) per output ------------------------
//
// A 128 x 256 output tile needs three 256-column s32 accumulators by scale
// (D0 = h.h x 2^16, D1 = h.l + l.h x 2^8, D2 = the rest x 1), more than the
// 512 TMEM columns.  Only floor(T / 4) mod 2^32 is kept, and with 64 T =
// 2^16 D0 + 2^8 D1 + D2 that is (2^8 D0 + D1 + floor(D2 / 256)) mod 2^32.
// So the tile runs in two phases: the three h passes over all K into D0
// (columns 0..255) and D1 (256..511); four warps fold E = 2^8 D0 + D1 (mod
// 2^32) into D1's columns; the eight remaining passes accumulate D2 into
// columns 0..255; the epilogue writes E + floor(D2 / 256).
//
// Warp 0 lane 0 issues the TMA loads (A and B tiles of each pass, both
// phases, in one ring of stages); warp 1 lane 0 issues the MMAs (one thread,
// as tcgen05 requires); warps 2..5 fold and write out (warp w reaches TMEM
// lanes 32 (w mod 4) .. + 31).  Every wait is bounded: the pipeline's waits by
// `spin` polls, after which the kernel records an error in the caller's
// counters; the teardown then waits (by kSpinLimit polls) for the copies and
// the MMA commits still in flight, frees TMEM and returns.  `stall` (tests
// only) makes the MMA thread first wait on a barrier nothing arrives on, so
// a test can watch a wait run out.

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// pass it of the tile's sequence -> A plane, B plane, accumulator column, signedness, first use
struct Pass {
    int pa, pb, col, sa, sb;
    bool first;
};

__device__ __forceinline__ Pass pass_of(int it, int nkb) {
    Pass p;
    if (it < P1 * nkb) {
        const int kb = it / P1, q = it % P1;
        p.pa = q == 2 ? 1 : 0;
        p.pb = q == 1 ? 1 : 0;
        p.col = q == 0 ? 0 : GN;
        p.sa = q == 2 ? 0 : 1;
        p.sb = q == 1 ? 0 : 1;
        p.first = kb == 0 && q != 2;
    } else {
        const int j = it - P1 * nkb, kb = j / P2, q = j % P2;
        p.pa = p.pb = q == 0 ? 1 : q + 1;
        p.col = 0;
        p.sa = p.sb = q == 0 ? 0 : 1;
        p.first = kb == 0 && q == 0;
    }
    return p;
}

__global__ void __launch_bounds__(GEMM_THREADS, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                  const __grid_constant__ CUtensorMap tmB, int nkb,
                                                                  int32_t *__restrict__ SX, int Np,
                                                                  unsigned long long *__restrict__ err,
                                                                  unsigned spin, int stall) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    // bars[0..S): full, [S..2S): empty, [2S]: phase 1 done, [2S+1]: fold done, [2S+2]: all done,
    // [2S+3]: the barrier nothing arrives on (the stall test)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);
    __shared__ int s_fail;
    const uint32_t bar_p1 = smem_u32(&bars[2 * STAGES]), bar_fold = smem_u32(&bars[2 * STAGES + 1]),
                   bar_done = smem_u32(&bars[2 * STAGES + 2]), bar_never = smem_u32(&bars[2 * STAGES + 3]);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // grouped order: GROUP_M row tiles at a time sweep the column tiles, so the
    // CTAs running together share A and B tiles in L2
    const int mt = gridDim.y, nt = gridDim.x;
    const int t = blockIdx.y * nt + blockIdx.x;
    const int gsize = GROUP_M * nt, g = t / gsize, gm0 = g * GROUP_M;
    const int gm = min(GROUP_M, mt - gm0), r = t - g * gsize;
    const int m0 = (gm0 + r % gm) * TILE, n0 = (r / gm) * GN;
    if (threadIdx.x == 0) {
        s_fail = 0;
        for (int s = 0; s < STAGES; s++) {
            mbar_init(smem_u32(&bars[s]), 1);
            mbar_init(smem_u32(&bars[STAGES + s]), 1);
        }
        mbar_init(bar_p1, 1);
        mbar_init(bar_fold, 4);
        mbar_init(bar_done, 1);
        mbar_init(bar_never, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int total = nkb * (P1 + P2);

    int issued = 0;
    bool ok = true;
    if (threadIdx.x == 0) {
        // TMA producer
        for (int it = 0; it < total; it++) {
            const int s = it % STAGES, round = it / STAGES;
            if (round > 0 && !mbar_wait(smem_u32(&bars[STAGES + s]), (round - 1) & 1, spin)) {
                s_fail = 1;
                break;
            }
            if (*(volatile int *)&s_fail) break;
            const Pass p = pass_of(it, nkb);
            const int kb = it < P1 * nkb ? it / P1 : (it - P1 * nkb) / P2;
            const uint32_t full = smem_u32(&bars[s]);
            uint8_t *sa = smem + s * STAGE_BYTES;
            mbar_expect_tx(full, STAGE_BYTES);
            tma_load_3d(smem_u32(sa), &tmA, kb * TILE, m0, p.pa, full);
            tma_load_3d(smem_u32(sa + TILE * TILE), &tmB, kb * TILE, n0, p.pb, full);
            issued = it + 1;
        }
    } else if (threadIdx.x == 32) {
        // MMA issuer
        if (stall && !mbar_wait(bar_never, 0, spin)) ok = false;
        for (int it = 0; it < total && ok; it++) {
            if (it == P1 * nkb) {
                // phase 1 complete: let the fold run, then overwrite D0's columns
                mma_commit(bar_p1);
                if (!mbar_wait(bar_fold, 0, spin)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
            const int s = it % STAGES, round = it / STAGES;
            if (!mbar_wait(smem_u32(&bars[s]), round & 1, spin)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const Pass p = pass_of(it, nkb);
            const uint32_t id = idesc_i8(p.sa, p.sb);
            const uint32_t a_addr = smem_u32(smem + s * STAGE_BYTES);
            const uint32_t b_addr = a_addr + TILE * TILE;
#pragma unroll
            for (int kk = 0; kk < TILE / 32; kk++)
                mma_i8(tmem + p.col, smem_desc(a_addr + kk * 32), smem_desc(b_addr + kk * 32), id,
                       (p.first && kk == 0) ? 0u : 1u);
            mma_commit(smem_u32(&bars[STAGES + s]));
        }
        if (!ok) {
            s_fail = 1;
            mma_commit(bar_p1);                 // release the fold warps (they see s_fail)
        }
        mma_commit(bar_done);
    } else if (warp >= 2) {
        const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
        // the fold: E = 2^8 D0 + D1 (mod 2^32) into D1's columns
        // each decision is the whole warp's: the TMEM loads and stores are warp-collective
        bool fine = __all_sync(0xffffffffu, mbar_wait(bar_p1, 0, spin) && !*(volatile int *)&s_fail);
        tc_fence_after();
        if (fine) {
            for (int c = 0; c < GN / 32; c++) {
                int32_t d0[32], d1[32];
                uint32_t e[32];
                tmem_ld32(tmem + lane_base + c * 32, d0);
                tmem_ld32(tmem + lane_base + GN + c * 32, d1);
#pragma unroll
                for (int j = 0; j < 32; j++) e[j] = ((uint32_t)d0[j] << 8) + (uint32_t)d1[j];
                tmem_st32(tmem + lane_base + GN + c * 32, e);
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_fold);
        // the epilogue: E + floor(D2 / 256)
        const bool landed = __all_sync(0xffffffffu, mbar_wait(bar_done, 0, spin));
        fine = __all_sync(0xffffffffu, landed && !*(volatile int *)&s_fail);
        tc_fence_after();
        if (fine) {
            const int row = m0 + 32 * (warp & 3) + lane;
            int32_t *dst = SX + (int64_t)row * Np + n0;
            for (int c = 0; c < GN / 32; c++) {
                if (n0 + c * 32 >= Np) break;             // the last column tile runs past the padded width
                int32_t d2[32], ev[32];
                tmem_ld32(tmem + lane_base + c * 32, d2);
                tmem_ld32(tmem + lane_base + GN + c * 32, ev);
                uint32_t o[32];
#pragma unroll
                for (int j = 0; j < 32; j++) o[j] = (uint32_t)ev[j] + (uint32_t)(d2[j] >> 8);
                uint4 *d4 = reinterpret_cast<uint4 *>(dst + c * 32);       // 128-byte aligned: Np, n0, c * 32 multiples of 32
#pragma unroll
                for (int j = 0; j < 8; j++) d4[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
            }
        } else if (!landed) {
            s_fail = 1;
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (s_fail && threadIdx.x == 0) {
        atomicAdd(err, 1ull);
        // let this CTA's copies still in flight land before its shared memory is
        // released, and the MMAs (the commit on bar_done follows them) finish
        // before TMEM is freed: full-length waits, whatever `spin` was
        for (int it = issued > STAGES ? issued - STAGES : 0; it < issued; it++)
            (void)mbar_wait(smem_u32(&bars[it % STAGES]), (it / STAGES) & 1);
        (void)mbar_wait(bar_done, 0);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

// --- the remainder sum_k u --------------------------------------------------------------------
//
// One CTA per 256 rows x 128 columns: a lane owns one row, and for each of
// its four 32-column words keeps sum_k u as carry-save bit planes (bit b of
// a plane belongs to column 32 word + b).  K runs in chunks of 32, double
// buffered in shared memory: the rows' records and B's column-sliced bits
// arrive by cp.async, then every thread builds 8 entries of two table halves
// (each for one (k, word)), and the rows read them.  The kernel writes sum u per
// output; wide_tc_finish_kernel combines it with the GEMM's sum.
//
// A table entry is a two-bit word (two 32-bit planes, stored together) per
// (k, word, index).  The F half, indexed by x mod 16, holds F* = s_w ? ~F :
// F + 1; the G half, indexed by x >> 4, holds G* = s_w ? ~G : G.  Then
// u' = F* + G* (mod 4) is r for a positive w and 3 - r for a negative one,
// and u = u' ^ (3 if a < 0): a's sign is an all-ones mask folded into the
// logic ops that form the two-bit sum.  Built as sums of the nibble bits'
// terms d_i = (y_{6-i}, y_{7-i}), negated where s_w (the start values (1,
// s_w) and (s_w, s_w) are F* and G* of 0).
//
// Entry (e, table t) sits at (e * 65 + t) * 8 bytes of its half: the 16
// entries of one table fall in distinct bank pairs, so each half-warp's
// 64-bit read is one wavefront whatever the rows' indexes, and the builders
// (consecutive t) store to consecutive pairs.

constexpr int RM = 256;                    // rows per CTA: 8 warps, one row per lane
constexpr int RNW = 4;                     // 32-column words per CTA
constexpr int RKC = 32;                    // k per chunk: four blocks of 8
constexpr int RNTAB = RKC * RNW;           // tables per chunk
constexpr int RTSTR = RNTAB + 1;           // entry stride in tables (odd)
constexpr int RENT = 16;                   // entries per half: the 16 nibble values
constexpr int TAB_HALF = RENT * RTSTR * 8;    // (low, high) plane pairs
constexpr int TAB_BYTES = 2 * TAB_HALF;
constexpr int REC_BYTES = (RKC / 2) * RM * 4;
constexpr int BST_BYTES = RKC * 9 * RNW * 4;
constexpr int BUF_BYTES = TAB_BYTES + REC_BYTES + BST_BYTES;
constexpr int NPL = 17;                    // counter planes per column word
constexpr int EPI_BYTES = RNW * NPL * RM * 4;
constexpr int REM_SMEM = (2 * BUF_BYTES > EPI_BYTES) ? 2 * BUF_BYTES : EPI_BYTES;
static_assert(BUF_BYTES % 16 == 0 && TAB_BYTES % 16 == 0 && REC_BYTES % 16 == 0, "cp.async alignment");

__device__ __forceinline__ void cp16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

struct W2 {
    uint32_t lo, hi;
};

// prmt.b32 in its default mode: a selector nibble with bit 3 set replicates
// the selected byte's top bit (the __byte_perm intrinsic keeps only the low
// three bits of each nibble)
__device__ __forceinline__ uint32_t sign_bytes(uint32_t x, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(d) : "r"(x), "r"(sel));
    return d;
}

__device__ __forceinline__ W2 add2(W2 a, W2 b) { return W2{a.lo ^ b.lo, a.hi ^ b.hi ^ (a.lo & b.lo)}; }

// s + a + b = (s ^ a ^ b) + 2 maj(s, a, b), bit by bit: s keeps the sum, the carry is returned
__device__ __forceinline__ uint32_t csa(uint32_t &s, uint32_t a, uint32_t b) {
    const uint32_t c = (s & a) | (s & b) | (a & b);
    s ^= a ^ b;
    return c;
}

struct RemIn {
    const uint32_t *rec, *bn;
    uint16_t *U;          // sum u per output, [Mp][Np]
    const int32_t *SX;    // floor((sum s X - (sum s) / 2) / 4) mod 2^32, [Mp][Np]
    const long long *rowL1, *colL1;
    const int *rowMax, *colMax;
    int Mp, Np, Kp, NWt;
    const int16_t *A, *B;
    int64_t lda, ldb;
    int M, N, K;
    const int8_t *shift_arr;
    int shift;
    int64_t ssm, ssn;
    int16_t *out;
    int32_t *acc_out;     // set: store the accumulator instead of POP
    uint8_t *flags;
    Width w;
    MxUnit u;
    sfb_counts *counts;
};

// the exact chunk-by-chunk accumulation of one output (an output the bound
// does not prove clip-free)
__device__ long long exact_output(const RemIn &in, int m, int n, bool &clip) {
    const long long lo = -(1ll << 31), hi = (1ll << 31) - 1;
    long long acc = 0;
    clip = false;
    for (int k0 = 0; k0 < in.K; k0 += 8) {
        long long g = 0;
        for (int k = k0; k < min(in.K, k0 + 8); k++) {
            const int ca = in.A[(int64_t)m * in.lda + k], cb = in.B[(int64_t)k * in.ldb + n];
            const int t = mx_prod16(mx_mag(ca, in.w.bits, true), mx_mag(cb, in.w.bits, true), in.u);
            g += ((ca ^ cb) < 0) ? -t : t;
        }
        long long s = acc + g;
        if (s < lo || s > hi) clip = true;
        acc = s < lo ? lo : (s > hi ? hi : s);
    }
    return acc;
}

__global__ void __launch_bounds__(256, 2) wide_rem_kernel(RemIn in) {
    extern __shared__ __align__(16) uint8_t rsm[];
    const int tid = threadIdx.x;
    const int ml = tid;                          // this lane's row within the tile
    const int m0 = blockIdx.y * RM, nw0 = blockIdx.x * RNW, n0 = nw0 * 32;

    // carry-save counters per column word: weights 1..16 (block level), 32, 64, 128
    // (with pending words of weight 32, 64, 128), then a binary counter 256 .. 32768
    // (sum u <= 3 K < 2^16)
    uint32_t p1[RNW], p2[RNW], p4[RNW], p8[RNW], p16[RNW], h32[RNW], pend32[RNW], h64[RNW], pend64[RNW];
    uint32_t h128[RNW], pend128[RNW], hh[RNW][8];
#pragma unroll
    for (int v = 0; v < RNW; v++) {
        p1[v] = p2[v] = p4[v] = p8[v] = p16[v] = h32[v] = pend32[v] = h64[v] = pend64[v] = 0;
        h128[v] = pend128[v] = 0;
#pragma unroll
        for (int l = 0; l < 8; l++) hh[v][l] = 0;
    }

    // chunk loads: each thread copies 32 contiguous bytes of the rows' records
    // in each of RKC / 16 row groups, and 16-byte rows of B's column bits
    const int rrow = tid >> 5, rcol = (tid & 31) * 8;             // k pair row, u32 column
    const uint32_t *rsrc = in.rec + (int64_t)rrow * in.Mp + m0 + rcol;
    const uint32_t rdst = (uint32_t)(TAB_BYTES + (rrow * RM + rcol) * 4);
    const int64_t rstep = (int64_t)(RKC / 2) * in.Mp, bstep = (int64_t)RKC * 9 * in.NWt;
    const uint32_t sbase = smem_u32(rsm);
    auto load_chunk = [&](int c, int q) {
        const uint32_t d = sbase + q * BUF_BYTES;
#pragma unroll
        for (int g = 0; g < RKC / 16; g++) {
            const uint32_t *src = rsrc + c * rstep + (int64_t)g * 8 * in.Mp;
            cp16(d + rdst + g * 8 * RM * 4, src);
            cp16(d + rdst + g * 8 * RM * 4 + 16, src + 4);
        }
        for (int i = tid; i < RKC * 9; i += 256) {
            const int kk = i / 9, p = i - 9 * kk;
            cp16(d + TAB_BYTES + REC_BYTES + i * RNW * 4, in.bn + ((int64_t)kk * 9 + p) * in.NWt + nw0 + c * bstep);
        }
        cp_commit();
    };

    // table build: item -> (table t, half h, entries 8 hi .. 8 hi + 7), two
    // items per thread; every step is the same for both halves but the y
    // planes read and two masks (h and hi are uniform over a warp)
    auto build_item = [&](int q, int item) {
        const int bt = item & (RNTAB - 1), bh = (item / RNTAB) & 1, bhi = item / (2 * RNTAB);
        const int bkl = bt / RNW, bv = bt % RNW;
        const uint32_t hm = bh ? 0xFFFFFFFFu : 0u;                    // all ones for the G half
        uint8_t *buf = rsm + q * BUF_BYTES;
        const uint32_t *ys = reinterpret_cast<const uint32_t *>(buf + TAB_BYTES + REC_BYTES) + bkl * 9 * RNW + bv;
        // F: d_i = (y_{6-i}, y_{7-i}); G: d_i = (y_{2-i}, y_{3-i}), y_{-1} = 0
        const int top = 7 - 4 * bh;
        const uint32_t sw = ys[8 * RNW];
        uint32_t yv[5];
#pragma unroll
        for (int j = 0; j < 5; j++) {                                  // y_{top - j}, j = 0..4
            const int p = top - j;
            yv[j] = p >= 0 ? ys[p * RNW] : 0u;
        }
        W2 d[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t lo = yv[i + 1], hi = yv[i];
            d[i] = W2{lo, hi ^ (lo & sw)};                             // -d where w is negative
        }
        const W2 start = W2{~hm | sw, sw};                             // F: (1, s_w); G: (s_w, s_w)
        W2 e[8];
        e[0] = bhi ? add2(start, d[3]) : start;
        e[1] = add2(e[0], d[0]);
        e[2] = add2(e[0], d[1]);
        e[3] = add2(e[1], d[1]);
        e[4] = add2(e[0], d[2]);
        e[5] = add2(e[4], d[0]);
        e[6] = add2(e[4], d[1]);
        e[7] = add2(e[5], d[1]);
        uint2 *tab = reinterpret_cast<uint2 *>(buf + bh * TAB_HALF);
#pragma unroll
        for (int j = 0; j < 8; j++) tab[(bhi * 8 + j) * RTSTR + bt] = make_uint2(e[j].lo, e[j].hi);
    };
    auto build = [&](int q) {
        static_assert(4 * RNTAB == 2 * 256, "two build items per thread");
        build_item(q, tid);
        build_item(q, tid + 256);
    };

    auto hot = [&](int c, int q) {
        const uint8_t *buf = rsm + q * BUF_BYTES;
        const uint32_t *recs = reinterpret_cast<const uint32_t *>(buf + TAB_BYTES);
#pragma unroll
        for (int b = 0; b < RKC / 8; b++) {
            const uint8_t *aF[8], *aG[8];
            uint32_t sm8[8];                                           // a's sign as a mask
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t r = recs[(b * 4 + j) * RM + ml];
                const uint8_t *fk = buf + (b * 8 + 2 * j) * RNW * 8, *gk = fk + TAB_HALF;
                aF[2 * j] = fk + (r & 0xFu) * (RTSTR * 8);
                aG[2 * j] = gk + __byte_perm(r, 0, 0x4441) * (RTSTR * 8);
                sm8[2 * j] = sign_bytes(r, 0x8888);
                aF[2 * j + 1] = fk + RNW * 8 + __umulhi(r & 0xF0000u, (uint32_t)(RTSTR * 8) << 16);
                aG[2 * j + 1] = gk + RNW * 8 + __byte_perm(r, 0, 0x4443) * (RTSTR * 8);
                sm8[2 * j + 1] = sign_bytes(r, 0xAAAA);
            }
#pragma unroll
            for (int v = 0; v < RNW; v++) {
                uint32_t u0[8], u1[8];
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    const uint2 f = *reinterpret_cast<const uint2 *>(aF[kk] + v * 8);
                    const uint2 g = *reinterpret_cast<const uint2 *>(aG[kk] + v * 8);
                    u0[kk] = f.x ^ g.x ^ sm8[kk];
                    u1[kk] = f.y ^ (f.x & g.x) ^ g.y ^ sm8[kk];
                }
                // 8 words of weight 1 and 8 of weight 2 into the planes: one carry of weight 32 out
                const uint32_t c2a = csa(p1[v], u0[0], u0[1]);
                const uint32_t c4a = csa(p2[v], u1[0], u1[1]);
                const uint32_t c2b = csa(p1[v], u0[2], u0[3]);
                const uint32_t c4b = csa(p2[v], c2a, c2b);
                const uint32_t c4c = csa(p2[v], u1[2], u1[3]);
                const uint32_t c8a = csa(p4[v], c4a, c4b);
                const uint32_t c2c = csa(p1[v], u0[4], u0[5]);
                const uint32_t c4d = csa(p2[v], u1[4], u1[5]);
                const uint32_t c8b = csa(p4[v], c4c, c4d);
                const uint32_t c2d = csa(p1[v], u0[6], u0[7]);
                const uint32_t c4e = csa(p2[v], c2c, c2d);
                const uint32_t c4f = csa(p2[v], u1[6], u1[7]);
                const uint32_t c8c = csa(p4[v], c4e, c4f);
                const uint32_t c16a = csa(p8[v], c8a, c8b);
                const uint32_t c16b = p8[v] & c8c;
                p8[v] ^= c8c;
                const uint32_t c32 = csa(p16[v], c16a, c16b);
                // static per chunk: blocks 0 / 2 leave a weight-32 carry pending, 1 / 3 pair it
                // into h32; the weight-64 carries of blocks 1 and 3 pair into h64; its carry is
                // left pending in even chunks and paired into h128 in odd ones, whose carry
                // ripples up the binary counter every second chunk
                if ((b & 1) == 0) {
                    pend32[v] = c32;
                } else {
                    const uint32_t c64 = csa(h32[v], pend32[v], c32);
                    pend32[v] = 0;
                    if (b == 1) {
                        pend64[v] = c64;
                    } else {
                        const uint32_t c128 = csa(h64[v], pend64[v], c64);
                        pend64[v] = 0;
                        if ((c & 1) == 0) {
                            pend128[v] = c128;
                        } else {
                            uint32_t cc = csa(h128[v], pend128[v], c128);
                            pend128[v] = 0;
#pragma unroll
                            for (int l = 0; l < 8; l++) {
                                const uint32_t t = hh[v][l] & cc;
                                hh[v][l] ^= cc;
                                cc = t;
                            }
                        }
                    }
                }
            }
        }
    };

    const int nch = in.Kp / RKC;
    load_chunk(0, 0);
    cp_wait_all();
    __syncthreads();
    build(0);
    __syncthreads();
    for (int c = 0; c < nch; c++) {
        const int q = c & 1;
        if (c + 1 < nch) load_chunk(c + 1, q ^ 1);
        hot(c, q);
        cp_wait_all();
        __syncthreads();
        if (c + 1 < nch) build(q ^ 1);
        __syncthreads();
    }

    // the planes to shared memory, [word][plane][row]; then one thread per output
    uint32_t *pl = reinterpret_cast<uint32_t *>(rsm);
#pragma unroll
    for (int v = 0; v < RNW; v++) {
        uint32_t *d = pl + (v * NPL) * RM + ml;
        d[0 * RM] = p1[v];
        d[1 * RM] = p2[v];
        d[2 * RM] = p4[v];
        d[3 * RM] = p8[v];
        d[4 * RM] = p16[v];
        d[5 * RM] = h32[v];
        d[6 * RM] = h64[v];
        d[7 * RM] = h128[v];
        d[8 * RM] = pend128[v];
#pragma unroll
        for (int l = 0; l < 8; l++) d[(9 + l) * RM] = hh[v][l];
    }
    __syncthreads();

    // sum u per output (< 3 Kp <= 49152) as 16 bits, [row][column]
    const int nl = tid & 127, vw = nl >> 5, bit = nl & 31;
    for (int i = 0; i < RM / 2; i++) {
        const int mloc = 2 * i + (tid >> 7);
        const uint32_t *src = pl + (vw * NPL) * RM + mloc;
        uint32_t U = 0;
#pragma unroll
        for (int l = 0; l < NPL; l++) {
            const int wt = l < 8 ? l : l - 1;                    // planes 7 and 8 both weigh 128
            U += ((src[l * RM] >> bit) & 1u) << wt;
        }
        in.U[(int64_t)(m0 + mloc) * in.Np + n0 + nl] = (uint16_t)U;
    }
}

// The accumulator of each output from the GEMM's sum and the remainder's,
// the per-output clip bound (outputs it does not prove are recomputed
// exactly on the CUDA cores) and POP.  With T = sum s X - (sum s) / 2, the
// accumulator is (T + 3 Kp / 2 - U) / 4, a multiple of 4 before the division,
// so T mod 4 = (U - 3 Kp / 2) mod 4 and the accumulator is floor(T / 4) +
// ((T mod 4) + 3 Kp / 2 - U) / 4: exact modulo 2^32 from the 32-bit
// floor(T / 4), and so exact for every output the bound proves (|acc| < 2^31).
// POP of a 32-bit accumulator (every output here: proven below 2^31, or the
// clamped W = 32 accumulator), as mx_pop with 32-bit shifts.
__device__ __forceinline__ int mx_pop32(int acc, int shift, int F, Width w, bool &over, bool &under) {
    const int e = shift - F + w.bits - 1;
    const uint32_t mag = acc < 0 ? 0u - (uint32_t)acc : (uint32_t)acc;
    uint32_t q;
    if (e >= 0) {
        over = e >= 16 ? mag != 0 : mag > ((uint32_t)w.M >> e);
        q = over ? (uint32_t)w.M : mag << e;
    } else {
        const int d = -e;
        if (d >= 32) {
            q = 0;
        } else {
            const uint32_t fl = mag >> d, rem = mag & ((1u << d) - 1u), half = 1u << (d - 1);
            q = fl + ((rem > half) || (rem == half && (fl & 1u)));
        }
        over = q > (uint32_t)w.M;
        if (over) q = (uint32_t)w.M;
    }
    under = acc != 0 && q == 0;
    return acc < 0 ? -(int)q : (int)q;
}

// One block per 256 columns and a stride of rows.  A row whose L1 norm times
// the block's largest column magnitude is within the clip bound needs no
// per-output test (the bound is only ever used conservatively).
__global__ void __launch_bounds__(256) wide_tc_finish_kernel(RemIn in) {
    __shared__ unsigned sc[5];
    __shared__ int s_cmax[8];
    zero_counts_smem(sc);
    Counts cnt;
    const long long lim = (1ll << 31) - 1;
    const int h = 3 * in.Kp / 2;
    const int n = blockIdx.x * 256 + threadIdx.x;
    const bool nin = n < in.N;
    const int cmx = nin ? in.colMax[n] : 0;
    const long long cl1 = nin ? in.colL1[n] : 0;
    int bm = cmx;
#pragma unroll
    for (int o = 16; o; o >>= 1) bm = max(bm, __shfl_xor_sync(0xffffffffu, bm, o));
    if ((threadIdx.x & 31) == 0) s_cmax[threadIdx.x >> 5] = bm;
    __syncthreads();
    bm = s_cmax[0];
#pragma unroll
    for (int i = 1; i < 8; i++) bm = max(bm, s_cmax[i]);
    // four rows per step, their loads issued together
    for (int m0 = blockIdx.y; m0 < in.M; m0 += 4 * gridDim.y) {
        if (!nin) continue;
        int Uv[4];
        uint32_t tv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int m = m0 + j * gridDim.y;
            const int64_t at = (int64_t)min(m, in.M - 1) * in.Np + n;
            Uv[j] = in.U[at];
            tv[j] = (uint32_t)in.SX[at];
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int m = m0 + j * gridDim.y;
            if (m >= in.M) break;
            const long long rl1 = in.rowL1[m];
            const bool row_safe = ((rl1 * (long long)bm) >> 8) + in.K <= lim;
            const int64_t o = (int64_t)m * in.N + n;
            const int U = Uv[j];
            int S = (int32_t)(tv[j] + (uint32_t)((((U - h) & 3) + h - U) >> 2));
            bool cl = false;
            if (!row_safe) {
                const long long b1 = rl1 * (long long)cmx;
                const long long b2 = (long long)in.rowMax[m] * cl1;
                if (((b1 < b2 ? b1 : b2) >> 8) + in.K > lim) S = (int)exact_output(in, m, n, cl);
            }
            if (in.acc_out) {
                in.acc_out[o] = S;
                if (in.flags) in.flags[o] = (uint8_t)(cl ? SFB_F_ACC_CLIPPED : 0u);
                cnt.clip += cl;
                continue;
            }
            const int sft =
                in.shift_arr ? (int)in.shift_arr[(int64_t)m * in.ssm + (int64_t)n * in.ssn] : in.shift;
            bool over, under;
            const int qv = mx_pop32(S, sft, in.u.F, in.w, over, under);
            over |= cl;
            in.out[o] = (int16_t)qv;
            if (in.flags)
                in.flags[o] = (uint8_t)((over ? SFB_F_OVERFLOW : 0u) | (under ? SFB_F_UNDERFLOW : 0u) |
                                        (cl ? SFB_F_ACC_CLIPPED : 0u));
            cnt.over += over;
            cnt.under += under;
            cnt.clip += cl;
        }
    }
    flush_counts(cnt, in.counts, sc);
}

// --- host side -------------------------------------------------------------------------------

struct Layout {
    int64_t Mp, Np, Kp, KW;
    int64_t off_pa, off_pb, off_ra, off_bn, off_l1a, off_l1b, off_mxa, off_mxb, off_sx, off_u, total;
};

int64_t up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

Layout layout_for(int64_t M, int64_t N, int64_t K) {
    Layout L;
    L.Mp = up(M, RM);               // the remainder kernel's row tile (a multiple of TILE)
    L.Np = up(N, GN);               // whole GEMM column tiles (a multiple of the other kernels' 128)
    L.Kp = up(K, TILE);
    L.KW = L.Kp / 32;
    int64_t o = 0;
    auto take = [&](int64_t bytes) {
        const int64_t at = o;
        o = up(o + bytes, 1024);
        return at;
    };
    L.off_pa = take(NPLANES * L.Mp * L.Kp);
    L.off_pb = take(NPLANES * L.Np * L.Kp);
    L.off_ra = take(2 * L.Kp * L.Mp);
    L.off_bn = take(4 * 9 * L.Kp * (L.Np / 32));
    L.off_l1a = take(8 * L.Mp);
    L.off_l1b = take(8 * L.Np);
    L.off_mxa = take(4 * L.Mp);
    L.off_mxb = take(4 * L.Np);
    L.off_sx = take(4 * L.Mp * L.Np);
    L.off_u = take(2 * L.Mp * L.Np);
    L.total = o + 1024;            // slack for aligning the caller's base
    return L;
}

// The calling thread's wait settings for the GEMM launches it makes
// (sfb_wide_wait_limit): 0 polls = kSpinLimit, and the stall test off.
// The GEMM runs on a second stream beside the remainder kernel (they read
// the prepared planes and write different outputs; the finish kernel waits
// for both), so that each kernel's last, partly filled wave overlaps the
// other's work.  One such stream and its two events per host thread and
// device, made again when the device's context changes.  The no-allocation
// entry point launches everything on the caller's stream (t_serial).
struct SideStream {
    unsigned long long ctx;
    cudaStream_t s;
    cudaEvent_t fork, join;
};
thread_local SideStream t_side[64] = {};
thread_local bool t_serial = false;

SideStream *side_stream(int dev) {
    const unsigned long long ctx = context_id();
    SideStream &ss = t_side[dev];
    if (ss.s != nullptr && ctx != 0 && ss.ctx == ctx) return &ss;
    ss = SideStream{};
    if (cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
        (void)cudaGetLastError();
        ss = SideStream{};
        return nullptr;
    }
    ss.ctx = context_id();
    return &ss;
}

thread_local unsigned t_wait_polls = 0;
thread_local int t_wait_stall = 0;

// The prepared form of a B operand (sfb_wide_prepare_b): its nine int8
// planes, column-sliced bit planes and column statistics, laid out as in the
// workspace but in a buffer of their own, so that a B used by many calls
// (a layer's weights) is prepared once.
struct BLayout {
    int64_t Np, Kp, off_pb, off_bn, off_l1b, off_mxb, total;
};

BLayout blayout_for(int64_t N, int64_t K) {
    BLayout L;
    L.Np = up(N, GN);
    L.Kp = up(K, TILE);
    int64_t o = 0;
    auto take = [&](int64_t bytes) {
        const int64_t at = o;
        o = up(o + bytes, 1024);
        return at;
    };
    L.off_pb = take(NPLANES * L.Np * L.Kp);
    L.off_bn = take(4 * 9 * L.Kp * (L.Np / 32));
    L.off_l1b = take(8 * L.Np);
    L.off_mxb = take(4 * L.Np);
    L.total = o + 1024;            // slack for aligning the caller's base
    return L;
}

bool b_eligible(int bits, int mx, int64_t N, int64_t K) {
    return mx == SFB_MX_V492 && bits >= 9 && bits <= 16 && K >= 1 && K <= KMAX && N >= 1 && up(N, TILE) <= (1 << 20);
}

bool eligible(int bits, int mx, int64_t M, int64_t N, int64_t K) {
    return mx == SFB_MX_V492 && bits >= 9 && bits <= 16 && K >= 1 && K <= KMAX && M >= 1 && N >= 1 &&
           (double)M * (double)N * (double)K >= (double)(1 << 22) && up(M, TILE) <= (1 << 20) &&
           up(N, TILE) <= (1 << 20);
}

typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

int make_map(CUtensorMap *map, void *base, int64_t rows_pad, int64_t Kp, int box_rows) {
    EncodeTiled enc = encoder();
    if (!enc) return set_error(SFB_ECUDA, "sfb_matmul_wide: cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)rows_pad, (cuuint64_t)NPLANES};
    const cuuint64_t strides[2] = {(cuuint64_t)Kp, (cuuint64_t)(Kp * rows_pad)};
    const cuuint32_t box[3] = {TILE, (cuuint32_t)box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(SFB_ECUDA, "sfb_matmul_wide: tensor map encoding failed (%d)", (int)r);
    return SFB_OK;
}

}  // namespace

int64_t wide_tc_workspace(int bits, int mx, int64_t batch, int64_t M, int64_t N, int64_t K) {
    (void)batch;
    if (!eligible(bits, mx, M, N, K)) return 0;
    return layout_for(M, N, K).total;
}

int wide_tc_try(int bits, int mx, const int16_t *A, const int16_t *B, const int8_t *shift_arr, int shift,
                int16_t *out, uint8_t *flags, int64_t batch, int64_t M, int64_t N, int64_t K, int64_t lda,
                int64_t ldb, int64_t sa, int64_t sb, int64_t so, int64_t ssb, int64_t ssm, int64_t ssn, void *ws,
                int64_t ws_bytes, sfb_counts *counts, cudaStream_t st, bool *handled, int32_t *acc_out,
                const void *bprep) {
    *handled = false;
    if (!eligible(bits, mx, M, N, K)) return SFB_OK;
    if (bprep && batch > 1 && sb != 0)
        return set_error(SFB_EINVAL, "sfb_matmul_wide: a prepared B serves one matrix (stride_b must be 0)");
    const Layout L = layout_for(M, N, K);
    if (ws == nullptr || ws_bytes < L.total)
        return set_error(SFB_EINVAL, "sfb_matmul_wide: workspace of %lld bytes is smaller than the %lld needed",
                         (long long)ws_bytes, (long long)L.total);
    if (counts == nullptr) return set_error(SFB_EINVAL, "sfb_matmul_wide: the tensor-core path needs counts");
    // the kernels' shared-memory limits, set once per CUDA context (a device
    // reset starts a new context, which needs them again)
    static unsigned long long smem_ctx[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    const unsigned long long ctx = context_id();
    if (ctx == 0 || smem_ctx[dev] != ctx) {
        if (cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM) !=
                cudaSuccess ||
            cudaFuncSetAttribute(wide_rem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 REM_SMEM) != cudaSuccess)
            return check_launch("sfb_matmul_wide (attributes)");
        smem_ctx[dev] = context_id();
    }
    uint8_t *base = reinterpret_cast<uint8_t *>(((uintptr_t)ws + 1023) & ~(uintptr_t)1023);
    uint8_t *pa = base + L.off_pa, *pb = base + L.off_pb;
    uint32_t *ra = reinterpret_cast<uint32_t *>(base + L.off_ra);
    uint32_t *bn = reinterpret_cast<uint32_t *>(base + L.off_bn);
    long long *l1a = reinterpret_cast<long long *>(base + L.off_l1a);
    long long *l1b = reinterpret_cast<long long *>(base + L.off_l1b);
    int *mxa = reinterpret_cast<int *>(base + L.off_mxa), *mxb = reinterpret_cast<int *>(base + L.off_mxb);
    if (bprep) {                   // B's planes, bit slices and statistics from its prepared buffer
        const BLayout BL = blayout_for(N, K);
        uint8_t *bb = reinterpret_cast<uint8_t *>(((uintptr_t)bprep + 1023) & ~(uintptr_t)1023);
        pb = bb + BL.off_pb;
        bn = reinterpret_cast<uint32_t *>(bb + BL.off_bn);
        l1b = reinterpret_cast<long long *>(bb + BL.off_l1b);
        mxb = reinterpret_cast<int *>(bb + BL.off_mxb);
    }
    int32_t *SX = reinterpret_cast<int32_t *>(base + L.off_sx);
    CUtensorMap tmA, tmB;
    int rc = make_map(&tmA, pa, L.Mp, L.Kp, TILE);
    if (rc) return rc;
    rc = make_map(&tmB, pb, L.Np, L.Kp, GN);
    if (rc) return rc;
    const Width w = width(bits);
    for (int64_t z = 0; z < batch; z++) {
        if (cudaMemsetAsync(base + L.off_l1a, 0, L.off_sx - L.off_l1a, st) != cudaSuccess)
            return check_launch("sfb_matmul_wide (stats reset)");
        prep_kernel<true><<<dim3((unsigned)(L.Mp / PR), (unsigned)(L.Kp / PK)), 256, 0, st>>>(
            A + z * sa, lda, (int)M, (int)K, (int)L.Mp, (int)L.Kp, bits, pa, ra, l1a, mxa, nullptr, 0);
        if (!bprep)
            prep_kernel<false><<<dim3((unsigned)(L.Np / PR), (unsigned)(L.Kp / PK)), 256, 0, st>>>(
                B + z * sb, ldb, (int)N, (int)K, (int)L.Np, (int)L.Kp, bits, pb, nullptr, l1b, mxb, bn,
                (int)(L.Np / 32));
        RemIn in;
        in.rec = ra;
        in.bn = bn;
        in.SX = SX;
        in.rowL1 = l1a;
        in.colL1 = l1b;
        in.rowMax = mxa;
        in.colMax = mxb;
        in.Mp = (int)L.Mp;
        in.Np = (int)L.Np;
        in.Kp = (int)L.Kp;
        in.NWt = (int)(L.Np / 32);
        in.A = A + z * sa;
        in.B = B + z * sb;
        in.lda = lda;
        in.ldb = ldb;
        in.M = (int)M;
        in.N = (int)N;
        in.K = (int)K;
        in.shift_arr = shift_arr ? shift_arr + z * ssb : nullptr;
        in.shift = shift;
        in.ssm = ssm;
        in.ssn = ssn;
        in.out = out ? out + z * so : nullptr;
        in.acc_out = acc_out ? acc_out + z * so : nullptr;
        in.flags = flags ? flags + z * so : nullptr;
        in.w = w;
        in.u = mx_unit(mx, true);
        in.counts = counts;
        in.U = reinterpret_cast<uint16_t *>(base + L.off_u);
        SideStream *side = t_serial ? nullptr : side_stream(dev);
        cudaStream_t gst = st;
        if (side && cudaEventRecord(side->fork, st) == cudaSuccess &&
            cudaStreamWaitEvent(side->s, side->fork, 0) == cudaSuccess)
            gst = side->s;
        tc_gemm_kernel<<<dim3((unsigned)((L.Np + GN - 1) / GN), (unsigned)(L.Mp / TILE)), GEMM_THREADS, GEMM_SMEM, gst>>>(
            tmA, tmB, (int)(L.Kp / TILE), SX, (int)L.Np, &counts->reserved[0], t_wait_polls ? t_wait_polls : kSpinLimit,
            t_wait_stall);
        wide_rem_kernel<<<dim3((unsigned)(L.Np / (RNW * 32)), (unsigned)(L.Mp / RM)), 256, REM_SMEM, st>>>(in);
        if (gst != st &&
            (cudaEventRecord(side->join, gst) != cudaSuccess || cudaStreamWaitEvent(st, side->join, 0) != cudaSuccess))
            return check_launch("sfb_matmul_wide (stream join)");
        const int64_t fx = (N + 255) / 256;
        const dim3 fgrid((unsigned)fx, (unsigned)std::max<int64_t>(1, std::min<int64_t>(M, (int64_t)sm_count() * 8 / fx)));
        wide_tc_finish_kernel<<<fgrid, 256, 0, st>>>(in);
        rc = check_launch("sfb_matmul_wide (tensor-core path)");
        if (rc) return rc;
    }
    *handled = true;
    return SFB_OK;
}

int64_t wide_tc_prepared_b_bytes(int bits, int mx, int64_t N, int64_t K) {
    return b_eligible(bits, mx, N, K) ? blayout_for(N, K).total : 0;
}

int wide_tc_prepare_b(int bits, int mx, const int16_t *B, int64_t N, int64_t K, int64_t ldb, void *prep,
                      int64_t prep_bytes, cudaStream_t st) {
    if (!b_eligible(bits, mx, N, K)) return SFB_OK;        // no prepared form: calls read B's codes
    const BLayout BL = blayout_for(N, K);
    if (prep == nullptr || prep_bytes < BL.total)
        return set_error(SFB_EINVAL, "sfb_wide_prepare_b: buffer of %lld bytes is smaller than the %lld needed",
                         (long long)prep_bytes, (long long)BL.total);
    if (B == nullptr || ldb < N) return set_error(SFB_EINVAL, "sfb_wide_prepare_b: null B or ldb < N");
    uint8_t *bb = reinterpret_cast<uint8_t *>(((uintptr_t)prep + 1023) & ~(uintptr_t)1023);
    if (cudaMemsetAsync(bb + BL.off_l1b, 0, BL.off_mxb + 4 * BL.Np - BL.off_l1b, st) != cudaSuccess)
        return check_launch("sfb_wide_prepare_b (stats reset)");
    prep_kernel<false><<<dim3((unsigned)(BL.Np / PR), (unsigned)(BL.Kp / PK)), 256, 0, st>>>(
        B, ldb, (int)N, (int)K, (int)BL.Np, (int)BL.Kp, bits, bb + BL.off_pb, nullptr,
        reinterpret_cast<long long *>(bb + BL.off_l1b), reinterpret_cast<int *>(bb + BL.off_mxb),
        reinterpret_cast<uint32_t *>(bb + BL.off_bn), (int)(BL.Np / 32));
    return check_launch("sfb_wide_prepare_b");
}

}  // namespace sfb

// --- the wide matmul without any device allocation ------------------------------------------
//
// For callers that cannot allocate device memory on their hot path: a host
// program that has handed all of the GPU's memory to its own pool, a plugin
// host that forbids allocations once it has started, or a loop that cannot
// afford the device-wide synchronisation cudaMalloc / cudaFree can imply.
// The tensor-core path's scratch (operand planes, remainder bit planes, row /
// column statistics, partial sums) lives in the fixed array below instead of
// a caller workspace.  Every GPU that loads this library holds the array until
// the process exits.  The array keeps the previous call's contents; the path
// clears what must start at zero (the row / column statistics) and overwrites
// everything else.  Calls share the one array, so two calls whose kernels
// overlap on the GPU (different streams, or different host threads) race.

namespace {

constexpr int64_t kNoAllocScratchBytes = 64ll << 20;   // 64 MiB per device

static __device__ __align__(256) unsigned char g_wide_scratch[kNoAllocScratchBytes];

}  // namespace

extern "C" int sfb_wide_wait_limit(unsigned polls, int stall) {
    sfb::t_wait_polls = polls;
    sfb::t_wait_stall = stall != 0;
    return SFB_OK;
}

extern "C" int sfb_matmul_wide_noalloc(int bits, int mx, const int16_t *A, const int16_t *B,
                                       const int8_t *shift_arr, int shift, int16_t *out, uint8_t *flags,
                                       int64_t batch, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                       int64_t stride_a, int64_t stride_b, int64_t stride_out, int64_t shift_sb,
                                       int64_t shift_sm, int64_t shift_sn, sfb_counts *counts, sfb_stream stream) {
    using namespace sfb;
    // The array's device address, looked up by the first call on each device
    // with that device current (so that first call belongs before any stream
    // capture), and again whenever the device's CUDA context has changed: a
    // device reset reloads the library's module and the array may then sit at
    // another address.
    struct Slot {
        unsigned long long ctx;
        void *ptr;
    };
    static Slot scratch[64] = {};
    static std::mutex lock;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return set_error(SFB_ECUDA, "sfb_matmul_wide_noalloc: no current CUDA device");
    void *ptr = nullptr;
    {
        std::lock_guard<std::mutex> g(lock);
        Slot &slot = scratch[dev];
        const unsigned long long ctx = context_id();
        if (slot.ptr == nullptr || ctx == 0 || slot.ctx != ctx) {
            slot.ptr = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&slot.ptr, g_wide_scratch);
            if (e != cudaSuccess) {
                slot.ptr = nullptr;
                return set_error(SFB_ECUDA, "sfb_matmul_wide_noalloc: scratch lookup failed: %s", cudaGetErrorString(e));
            }
            slot.ctx = context_id();     // the lookup makes the device's context current if none was
        }
        ptr = slot.ptr;
    }
    const int64_t need = sfb_matmul_wide_workspace(bits, mx, batch, M, N, K);
    if (need < 0) return (int)need;
    if (need > kNoAllocScratchBytes)
        return set_error(SFB_ERANGE,
                         "sfb_matmul_wide_noalloc: %lld x %lld x %lld needs %lld bytes of scratch, more than the "
                         "%lld this entry point holds; use sfb_matmul_wide with a workspace",
                         (long long)M, (long long)N, (long long)K, (long long)need, (long long)kNoAllocScratchBytes);
    sfb::t_serial = true;                // everything on the caller's stream: no stream or event is made
    const int rc = sfb_matmul_wide(bits, mx, A, B, shift_arr, shift, out, flags, batch, M, N, K, lda, ldb, stride_a,
                                   stride_b, stride_out, shift_sb, shift_sm, shift_sn, ptr, kNoAllocScratchBytes,
                                   counts, stream);
    sfb::t_serial = false;
    return rc;
}
