// Exhaustive sweep of every operand pair of one width (the reference's
// tools/exhaustive.py:146-181, on the GPU).
//
// Rows are the a codes of [a_lo, a_hi); every row pairs a with all 2M+1
// codes b_j = j - M and evaluates the op with the elementwise kernels' own
// per-element arithmetic (sfb_ew_ops.cuh).  Nothing per pair is stored: each
// row folds into one 32-bit digest
//     sum_j ((code + M) | flags << 16) * w_j   (mod 2^32),
// w_j = the low word of splitmix64(j), made odd, and the events are totalled.
// A wrong code or flag at one pair changes the digest by a nonzero multiple
// (below 2^20) of an odd weight, which is never 0 mod 2^32, so a single
// wrong pair is always seen; several cancel with probability about 2^-32.
//
// A CTA owns RB consecutive rows and one span of j; its threads stride
// over the span, compute w_j once and apply it to the RB rows (one
// multiply-add per pair), keeping RB running digests in registers; a warp
// shuffle reduction and one 32-bit atomic add per row and warp add the
// span's share to the row (the digest is a sum, so spans add).  A launch of
// few rows (a rank's share of a multi-GPU sweep) splits j into as many spans
// as it takes to give every SM several CTAs.  The sweep is bound by
// instruction issue (about 2^32 pairs per op at sf16), with 4 bytes written
// per row.
#include <algorithm>

#include "sfb_common.cuh"
#include "sfb_ew_ops.cuh"

namespace sfb {
namespace {

using namespace ewops;

constexpr int SW_THREADS = 256, RB = 16;

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long x) {
    unsigned long long z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

template <int OP, int BITS>
__global__ void __launch_bounds__(SW_THREADS) sweep_kernel(Width w, int a_lo, int a_hi, int jspan,
                                                          uint32_t *__restrict__ row_digest, sfb_counts *counts) {
    __shared__ unsigned sc[5];
    zero_counts_smem(sc);
    const int M = w.M, n = 2 * w.M + 1;
    const int r0 = a_lo + blockIdx.x * RB;
    uint32_t dg[RB];
#pragma unroll
    for (int r = 0; r < RB; r++) dg[r] = 0;
    Counts cnt;
    const int j0 = blockIdx.y * jspan, j1 = min(n, j0 + jspan);
    for (int j = j0 + threadIdx.x; j < j1; j += SW_THREADS) {
        const uint32_t wj = (uint32_t)splitmix64((unsigned long long)j) | 1u;
        const int b = j - M;
#pragma unroll
        for (int r = 0; r < RB; r++) {
            const int a = r0 + r;
            if (a < a_hi) {
                Ev ev;
                const int k = ew_one<OP, BITS>(a, b, 0, w, 0, ev);
                dg[r] += ((uint32_t)(k + M) | (flag_byte(ev) << 16)) * wj;
                tally(cnt, ev);
            }
        }
    }
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < RB; r++) {
#pragma unroll
        for (int o = 16; o; o >>= 1) dg[r] += __shfl_xor_sync(0xffffffffu, dg[r], o);
        const int a = r0 + r;
        if (lane == 0 && a < a_hi) atomicAdd(&row_digest[a - a_lo], dg[r]);
    }
    flush_counts(cnt, counts, sc);
}

template <int OP>
void launch_sweep(int bits, int a_lo, int a_hi, uint32_t *rd, sfb_counts *counts, cudaStream_t st) {
    const int rows = (a_hi - a_lo + RB - 1) / RB;
    const Width w = width(bits);
    const int n = 2 * w.M + 1;
    auto kern = bits == 16 ? sweep_kernel<OP, 16> : sweep_kernel<OP, 0>;
    auto resident = [](decltype(kern) k) {
        int b = 0;
        return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k, SW_THREADS, 0) == cudaSuccess && b > 0 ? b : 1;
    };
    static const int per_sm16 = resident(sweep_kernel<OP, 16>), per_sm0 = resident(sweep_kernel<OP, 0>);
    const int per_sm = bits == 16 ? per_sm16 : per_sm0;
    // j spans: enough CTAs for four waves, each span at least 8 strides of the block
    const int want = 4 * sm_count() * per_sm;
    const int most = std::max(1, n / (8 * SW_THREADS));
    const int spans = std::min(most, std::max(1, (want + rows - 1) / rows));
    const int jspan = (n + spans - 1) / spans;
    kern<<<dim3((unsigned)rows, (unsigned)spans), SW_THREADS, 0, st>>>(w, a_lo, a_hi, jspan, rd, counts);
}

}  // namespace
}  // namespace sfb

extern "C" int sfb_sweep(int op, int bits, int64_t a_lo, int64_t a_hi, uint32_t *row_digest, sfb_counts *counts,
                         sfb_stream stream) {
    using namespace sfb;
    if (bits < 4 || bits > 16) return set_error(SFB_EINVAL, "sfb_sweep: width %d is not 4..16", bits);
    const int64_t M = (1 << (bits - 1)) - 1;
    if (a_lo < -M || a_hi > M + 1 || a_lo > a_hi)
        return set_error(SFB_EINVAL, "sfb_sweep: rows [%lld, %lld) are not within [-%lld, %lld]", (long long)a_lo,
                         (long long)a_hi, (long long)M, (long long)M);
    if (a_lo == a_hi) return SFB_OK;
    if (row_digest == nullptr) return set_error(SFB_EINVAL, "sfb_sweep: null row digest buffer");
    cudaStream_t st = (cudaStream_t)stream;
    switch (op) {
        case SFB_OP_ADD: launch_sweep<SFB_OP_ADD>(bits, (int)a_lo, (int)a_hi, row_digest, counts, st); break;
        case SFB_OP_SUB: launch_sweep<SFB_OP_SUB>(bits, (int)a_lo, (int)a_hi, row_digest, counts, st); break;
        case SFB_OP_MUL: launch_sweep<SFB_OP_MUL>(bits, (int)a_lo, (int)a_hi, row_digest, counts, st); break;
        case SFB_OP_DIV: launch_sweep<SFB_OP_DIV>(bits, (int)a_lo, (int)a_hi, row_digest, counts, st); break;
        default: return set_error(SFB_EINVAL, "sfb_sweep: op %d is not add, sub, mul or div", op);
    }
    return check_launch("sfb_sweep");
}
