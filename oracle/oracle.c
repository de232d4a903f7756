/* C restatement of the reference's chain and wide accumulation (oracle; test
 * infrastructure only, never linked into the product).
 *
 *   orc_matmul_chain  : src/sf/_linalg.py:61-81 (one fma chain per output,
 *                       k increasing; fma rule of src/sf/_vectorized.py:128-131)
 *   orc_wide_acc      : src/sf/_linalg.py:261-308 with the SF16-block product
 *                       of src/sf/_linalg.py:190-198 walked bit by bit, as defined
 *
 * Codes are int64 signed codes in [-M, M].  Each call computes rows [r0, r1);
 * the Python side splits rows over threads (ctypes releases the GIL).
 */
#include <stdint.h>
#include <stdlib.h>

static inline int64_t clamp64(int64_t v, int64_t lo, int64_t hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

/* out[m, n] = chain over k of clip(acc + trunc(a[m,k] b[k,n] / S)).
 * A: M x K row-major, B: K x N row-major. */
void orc_matmul_chain(int64_t r0, int64_t r1, int bits, const int64_t *A, const int64_t *B, int64_t M, int64_t N,
                      int64_t K, int64_t *out, uint8_t *over, uint8_t *under) {
    const int64_t S = (int64_t)1 << (bits - 1), MX = S - 1;
    (void)M;
    for (int64_t m = r0; m < r1; m++) {
        for (int64_t n = 0; n < N; n++) {
            int64_t acc = 0;
            uint8_t o = 0, u = 0;
            for (int64_t k = 0; k < K; k++) {
                const int64_t p = A[m * K + k] * B[k * N + n];
                const int64_t mag = (p < 0 ? -p : p) / S;
                const int64_t t = p < 0 ? -mag : mag;
                const int64_t s = acc + t;
                const int ov = s > MX || s < -MX;
                o |= (uint8_t)ov;
                u |= (uint8_t)(!ov && p != 0 && t == 0);
                acc = clamp64(s, -MX, MX);
            }
            out[m * N + n] = acc;
            over[m * N + n] = o;
            under[m * N + n] = u;
        }
    }
}

/* SF16-block product magnitude: partial-product rows bit_i(a) (w << i) with the
 * columns below tk dropped, plus comp, masked to 30 bits, cut to F fraction bits. */
static inline int64_t prod16(int64_t a, int64_t w, int tk, int64_t comp, int F) {
    const int64_t keep = ~(((int64_t)1 << tk) - 1);
    int64_t r = comp;
    for (int i = 0; i < 15; i++)
        if ((a >> i) & 1) r += (w << i) & keep;
    return (r & (((int64_t)1 << 30) - 1)) >> (30 - F);
}

/* Wide accumulators: am / bm magnitudes as the block reads them (A: M x K,
 * B: K x N), an / bn 1 where the code is negative.  blk16 selects the
 * SF16-block product; otherwise products are exact.  Chunks of 8 k, one clip
 * at [lo, hi] per chunk. */
void orc_wide_acc(int64_t r0, int64_t r1, const int64_t *am, const uint8_t *an, const int64_t *bm, const uint8_t *bn,
                  int64_t M, int64_t N, int64_t K, int blk16, int tk, int64_t comp, int F,
                  int64_t lo, int64_t hi, int64_t *acc, uint8_t *clip) {
    (void)M;
    for (int64_t m = r0; m < r1; m++) {
        for (int64_t n = 0; n < N; n++) {
            int64_t s = 0;
            uint8_t c = 0;
            for (int64_t k0 = 0; k0 < K; k0 += 8) {
                const int64_t k1 = k0 + 8 < K ? k0 + 8 : K;
                int64_t g = 0;
                for (int64_t k = k0; k < k1; k++) {
                    const int64_t a = am[m * K + k], w = bm[k * N + n];
                    const int64_t t = blk16 ? prod16(a, w, tk, comp, F) : a * w;
                    g += (an[m * K + k] ^ bn[k * N + n]) ? -t : t;
                }
                s += g;
                if (s < lo) { s = lo; c = 1; }
                else if (s > hi) { s = hi; c = 1; }
            }
            acc[m * N + n] = s;
            clip[m * N + n] = c;
        }
    }
}
