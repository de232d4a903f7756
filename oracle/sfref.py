"""NumPy restatement of the reference's sfN arithmetic (oracle; test infrastructure).

Codes are signed integers k in [-M, M], M = 2^(N-1) - 1, value k / 2^(N-1)
(reference src/sf/_format.py:1-11, :21-60).  Every op returns
``(codes int64, events)`` where ``events`` maps an event name to a boolean
mask over the output, the shape the reference's vectorised ops return
(src/sf/_vectorized.py:1-11).
"""
from __future__ import annotations

import numpy as np

EVENTS = ("overflow", "underflow", "divide", "invalid")


def consts(bits: int):
    """(M, S) for sfN: M = 2^(N-1) - 1 the largest code, S = 2^(N-1) one unit
    (src/sf/_format.py:40-48)."""
    if not 4 <= bits <= 16:
        raise ValueError(f"sf width must be 4..16, got {bits}")
    S = 1 << (bits - 1)
    return S - 1, S


def _i64(x):
    return np.asarray(x, dtype=np.int64)


def _tdiv(num, den):
    """Integer quotient rounded toward zero (src/sf/_vectorized.py:19-22)."""
    num, den = _i64(num), _i64(den)
    mag = np.abs(num) // np.abs(den)
    return np.where((num < 0) ^ (den < 0), -mag, mag)


# --- elementwise ops (src/sf/_vectorized.py:94-156) -------------------------------------

def add(bits, a, b):
    """clip(a + b) with overflow where |a + b| > M (_vectorized.py:94-95, :25-27)."""
    M, _ = consts(bits)
    s = _i64(a) + _i64(b)
    return np.clip(s, -M, M), {"overflow": np.abs(s) > M}


def sub(bits, a, b):
    """clip(a - b), as add (_vectorized.py:98-99)."""
    M, _ = consts(bits)
    s = _i64(a) - _i64(b)
    return np.clip(s, -M, M), {"overflow": np.abs(s) > M}


def neg(bits, a):
    """Exact negation, no event (_vectorized.py:102-103)."""
    return -_i64(a), {}


def abs_(bits, a):
    """Exact magnitude, no event (_vectorized.py:106-107)."""
    return np.abs(_i64(a)), {}


def mul(bits, a, b):
    """trunc(a b / S); underflow where a nonzero product truncates to 0
    (_vectorized.py:110-113)."""
    _, S = consts(bits)
    p = _i64(a) * _i64(b)
    k = _tdiv(p, S)
    return k, {"underflow": (p != 0) & (k == 0)}


def div(bits, a, b):
    """Saturating division (_vectorized.py:116-125):
    b == 0        -> sign(a) M (0 for 0/0), divide event;
    a != 0 and |a| >= |b| -> +-M with the quotient's sign, overflow event;
    otherwise     -> trunc(a S / b)."""
    M, S = consts(bits)
    a, b = np.broadcast_arrays(_i64(a), _i64(b))
    zero = b == 0
    q = _tdiv(a * S, np.where(zero, 1, b))
    over = ~zero & (a != 0) & (np.abs(a) >= np.abs(b))
    sat = np.where(np.sign(a) == np.sign(b), M, -M)
    out = np.where(zero, np.sign(a) * M, np.where(over, sat, q))
    return out, {"overflow": over, "divide": zero}


def fma(bits, a, b, c):
    """add(mul(a, b), c): two roundings, not fused; the product's underflow is
    reported only where the add did not overflow (_vectorized.py:128-131)."""
    p, ep = mul(bits, a, b)
    s, es = add(bits, p, c)
    return s, {"overflow": es["overflow"], "underflow": ep["underflow"] & ~es["overflow"]}


def sqrt(bits, a):
    """floor(sqrt(a S)) for a >= 0; 0 and an invalid event for a < 0
    (_vectorized.py:134-142).  Integer square root, exact."""
    _, S = consts(bits)
    a = _i64(a)
    bad = a < 0
    x = np.where(bad, 0, a) * S
    r = np.floor(np.sqrt(x.astype(np.float64))).astype(np.int64)
    r = np.where(r * r > x, r - 1, r)
    r = np.where((r + 1) * (r + 1) <= x, r + 1, r)
    return np.where(bad, 0, r), {"invalid": bad}


def pow_int(bits, a, n: int):
    """a ** n as a left-to-right chain of ``mul`` (_vectorized.py:145-156).
    The reference stops early once every element is 0; later steps would
    only multiply zeros, which raises no event, so running all n - 1 steps
    gives the same codes and masks."""
    if n < 1:
        raise ValueError("pow needs n >= 1")
    a = _i64(a)
    k = a.copy()
    under = np.zeros(k.shape, bool)
    for _ in range(n - 1):
        k, ev = mul(bits, k, a)
        under |= ev["underflow"]
    return k, {"underflow": under}


OPS = {"add": add, "sub": sub, "mul": mul, "div": div, "fma": fma,
       "neg": neg, "abs": abs_, "sqrt": sqrt}


def ew(op: str, bits: int, *operands, **kw):
    if op == "pow":
        return pow_int(bits, *operands, **kw)
    return OPS[op](bits, *operands)


# --- chain accumulation (src/sf/_linalg.py:30-111) -----------------------------------------

def cast_float(bits, values, scale=1.0):
    """float -> codes of ``values / scale`` (scale a number or a per-row
    column vector), src/sf/_vectorized.py:59-71: NaN -> 0 (invalid),
    |v| >= 1 - 2^-N -> +-M (overflow, inf included), else round half to
    even of v 2^(N-1), underflow where a nonzero value rounds to 0."""
    M, S = consts(bits)
    v = np.asarray(values).astype(np.float64) / np.asarray(scale, dtype=np.float64)
    nan = np.isnan(v)
    over = (np.abs(v) >= 1.0 - 2.0 ** -bits) & ~nan
    fits = ~over & ~nan
    k = np.zeros(v.shape, dtype=np.int64)
    k[fits] = np.rint(v[fits] * S).astype(np.int64)
    k[over] = np.sign(v[over]).astype(np.int64) * M
    under = fits & (k == 0) & (v != 0)
    return k, {"overflow": over, "underflow": under, "invalid": nan}


def sum_chain(bits, a, axis=0):
    """Sequential saturating sum from index 0 (_linalg.py:30-40)."""
    a = np.moveaxis(_i64(a), axis, 0)
    acc = np.zeros(a.shape[1:], np.int64)
    over = np.zeros(a.shape[1:], bool)
    for k in range(a.shape[0]):
        acc, ev = add(bits, acc, a[k])
        over |= ev["overflow"]
    return acc, {"overflow": over}


def matmul_chain(bits, A, B):
    """(..., M, K) @ (..., K, N), one fma chain per output in increasing k:
    acc = clip(acc + trunc(a_k b_k / S)) (_linalg.py:61-81).  Overflow marks
    outputs where any step saturated; underflow outputs where a product
    truncated to 0 on a step that did not saturate (the fma rule)."""
    A, B = _i64(A), _i64(B)
    K = A.shape[-1]
    shape = np.broadcast_shapes(A.shape[:-2], B.shape[:-2]) + (A.shape[-2], B.shape[-1])
    acc = np.zeros(shape, np.int64)
    over = np.zeros(shape, bool)
    under = np.zeros(shape, bool)
    for k in range(K):
        acc, ev = fma(bits, A[..., :, k:k + 1], B[..., k:k + 1, :], acc)
        over |= ev["overflow"]
        under |= ev["underflow"]
    return acc, {"overflow": over, "underflow": under}


def chain_bound(bits, A, B) -> int:
    """The reference's L1 bound on every partial sum, in codes (_linalg.py:84-106):
    min(max_i ||a_i||_1 max|b|, max|a| max_j ||b_j||_1) // S."""
    _, S = consts(bits)
    A, B = np.abs(_i64(A)), np.abs(_i64(B))
    if A.size == 0 or B.size == 0 or A.shape[-1] == 0:
        return 0
    r = int(A.sum(axis=-1).max()) * int(B.max())
    c = int(A.max()) * int(B.sum(axis=-2).max())
    return min(r, c) // S


# --- wide accumulation: the MX engine (src/sf/_linalg.py:114-369) --------------------------

# The accumulator units per chip (_linalg.py:144-147): W accumulator bits,
# F fraction bits, tk the first kept partial-product column, comp the
# constant added to each SF16-block product.
MX_UNITS = {
    "v4.9.2": {16: dict(W=32, F=22, tk=6, comp=80), 8: dict(W=32, F=14, tk=None, comp=None)},
    "v4.8.1": {16: dict(W=25, F=19, tk=9, comp=1024), 8: dict(W=20, F=14, tk=None, comp=None)},
}
MX_DEFAULT = "v4.9.2"
SHIFT_MIN, SHIFT_MAX = -32, 31


def mx_block(bits: int) -> int:
    """sf9..sf16 run on the SF16 block, sf4..sf8 on the SF8 block (_linalg.py:178-180)."""
    return 16 if bits >= 9 else 8


def mx_mags(bits, codes):
    """|code| left-aligned in the 16-bit word's 15-bit magnitude field, or the
    top byte's 7-bit field on the SF8 block (_linalg.py:183-187)."""
    m = np.abs(_i64(codes)) << (16 - bits)
    return m >> 8 if mx_block(bits) == 8 else m


def mx_product16(am, wm, unit):
    """SF16-block product magnitude (_linalg.py:190-198): the 15 partial-product
    rows bit_i(a) (w << i) with columns below tk dropped, plus comp, masked to
    30 bits and cut to F fraction bits.  Walked bit by bit, as defined."""
    am, wm = _i64(am), _i64(wm)
    keep = ~np.int64((1 << unit["tk"]) - 1)
    acc = np.full(np.broadcast_shapes(am.shape, wm.shape), unit["comp"], np.int64)
    for i in range(15):
        acc = acc + ((am >> i) & 1) * ((wm << i) & keep)
    return (acc & ((1 << 30) - 1)) >> (30 - unit["F"])


def wide_acc(bits, A, B, mx=MX_DEFAULT, chunk_cols=256):
    """MX accumulators before POP (_linalg.py:261-308): per output, K in
    chunks of 8; a chunk's signed products are summed exactly, added to the
    W-bit accumulator, which saturates at +-(2^(W-1)) once per chunk.
    Returns (acc int64, clipped bool, F)."""
    A, B = _i64(A), _i64(B)
    blk = mx_block(bits)
    u = MX_UNITS[mx][blk]
    lo, hi = -(1 << (u["W"] - 1)), (1 << (u["W"] - 1)) - 1
    am, bm = mx_mags(bits, A), mx_mags(bits, B)
    an, bn = A < 0, B < 0
    K = A.shape[-1]
    shape = np.broadcast_shapes(A.shape[:-2], B.shape[:-2]) + (A.shape[-2], B.shape[-1])
    acc = np.zeros(shape, np.int64)
    clip = np.zeros(shape, bool)
    N = shape[-1]
    for n0 in range(0, N, chunk_cols):
        cs = slice(n0, min(N, n0 + chunk_cols))
        s = np.zeros(shape[:-1] + (cs.stop - cs.start,), np.int64)
        c = np.zeros(s.shape, bool)
        for k0 in range(0, K, 8):
            ks = slice(k0, min(K, k0 + 8))
            a_ = am[..., :, ks][..., :, :, None]
            b_ = bm[..., ks, cs][..., None, :, :]
            t = mx_product16(a_, b_, u) if blk == 16 else a_ * b_
            ng = an[..., :, ks][..., :, :, None] ^ bn[..., ks, cs][..., None, :, :]
            s = s + np.where(ng, -t, t).sum(axis=-2)
            c |= (s < lo) | (s > hi)
            s = np.clip(s, lo, hi)
        acc[..., cs] = s
        clip[..., cs] = c
    return acc, clip, u["F"]


def wide_pop(bits, acc, shift, frac):
    """POP (_linalg.py:201-220): acc 2^(shift - frac) in sfN codes, rounded
    half to even on the magnitude, saturated at M, sign restored (never -0).
    Returns (codes, overflow (q > M before the clamp), underflow (acc != 0,
    q == 0))."""
    M, _ = consts(bits)
    acc = _i64(acc)
    e = np.broadcast_to(_i64(shift) - frac + bits - 1, acc.shape)
    mag = np.abs(acc)
    d = np.maximum(-e, 1)
    fl = mag >> d
    rem = mag - (fl << d)
    half = np.int64(1) << (d - 1)
    rnd = fl + ((rem > half) | ((rem == half) & (fl & 1 == 1)))
    q = np.where(e >= 0, mag << np.maximum(e, 0), rnd)
    over = q > M
    q = np.minimum(q, M)
    return np.where(acc < 0, -q, q), over, (acc != 0) & (q == 0)


def check_shift(shift):
    """An int in [-32, 31] or an integer array of them (_linalg.py:223-247)."""
    if shift is None:
        return 0
    if isinstance(shift, (bool, np.bool_)):
        raise TypeError("shift must be an int or an array of ints, got bool")
    if isinstance(shift, (int, np.integer)):
        if not SHIFT_MIN <= int(shift) <= SHIFT_MAX:
            raise ValueError(f"shift must be between {SHIFT_MIN} and {SHIFT_MAX}, got {shift}")
        return int(shift)
    arr = np.asarray(shift)
    if arr.dtype == bool or not np.issubdtype(arr.dtype, np.integer):
        raise TypeError(f"shift must be an int or an array of ints, got an array of {arr.dtype}")
    if arr.size and (arr.min() < SHIFT_MIN or arr.max() > SHIFT_MAX):
        raise ValueError("every shift must be between -32 and 31")
    arr = arr.astype(np.int64)
    return int(arr) if arr.ndim == 0 else arr


def matmul_wide(bits, A, B, shift=0, mx=MX_DEFAULT, acc_fn=None):
    """(..., M, K) @ (..., K, N) on the MX engine (_linalg.py:330-348):
    overflow = accumulator clipped or POP saturated; underflow = a nonzero
    total rounded to 0.  ``acc_fn`` replaces ``wide_acc`` (the C oracle)."""
    shift = check_shift(shift)
    acc, clip, F = (acc_fn or wide_acc)(bits, A, B, mx)
    if not isinstance(shift, int):
        shift = np.broadcast_to(shift, acc.shape)
    q, over, under = wide_pop(bits, acc, shift, F)
    return q, {"overflow": clip | over, "underflow": under}


def wide_acc_safe(bits, A, B, mx=MX_DEFAULT) -> bool:
    """Host proof that no accumulator can clip (_linalg.py:351-369): the L1
    relaxation of sum |t|, each SF16 term at most |a||w| / 2^(30-F) + 1."""
    A, B = _i64(A), _i64(B)
    if A.size == 0 or B.size == 0 or A.shape[-1] == 0:
        return True
    blk = mx_block(bits)
    am, bm = mx_mags(bits, A), mx_mags(bits, B)
    l1 = min(int(am.sum(axis=-1).max()) * int(bm.max()), int(am.max()) * int(bm.sum(axis=-2).max()))
    u = MX_UNITS[mx][blk]
    bound = l1 // (1 << (30 - u["F"])) + A.shape[-1] if blk == 16 else l1
    return bound <= (1 << (u["W"] - 1)) - 1


# --- the exact decomposition the B200 wide kernel uses, stated on the CPU ----------------

def t16_closed(am, wm):
    """v4.9.2 SF16-block product in closed form: with x = a mod 64, y = w mod 64,
    C[x][y] = sum_{i+j<6} 2^(i+j) x_i y_j (the dropped columns), the product is
    (a w + 80 - C) >> 8.  Equal to ``mx_product16`` for every 15-bit pair."""
    am, wm = _i64(am), _i64(wm)
    x, y = am & 63, wm & 63
    C = np.zeros(np.broadcast_shapes(x.shape, y.shape), np.int64)
    for i in range(6):
        C = C + ((x >> i) & 1) * ((y << i) & 63)
    return (am * wm + 80 - C) >> 8


# --- the wide sft linear: exponents, guard, shift rule, bias after POP, redo ---------------
# (src/sf/_heuristic.py:32-169, src/sf/torch/_core.py:55-99, :177-190, :463-600)

WIDE_MARGIN = 2


def h_for(K: int) -> int:
    """Bits taken back below the L2 bound for dot length K (_heuristic.py:32-37)."""
    K = int(K)
    return 0 if K < 1 else max(0, (K.bit_length() - 1) // 2 - WIDE_MARGIN)


def pow2_exp(m):
    """Smallest integer e with m / 2^e < 1, 0 where m == 0 (_heuristic.py:40-48)."""
    m = np.asarray(m, dtype=np.float64)
    out = np.zeros(m.shape, np.int64)
    nz = m > 0
    out[nz] = np.frexp(m[nz])[1]
    return out


def _pow2_codes(bits, x, e):
    M, S = consts(bits)
    P = bits - 1
    return np.clip(np.rint(np.ldexp(x, (P - e).astype(np.int64))), -M, M).astype(np.int64)


def quantize_pow2(bits, x, axis=-1):
    """One power-of-two exponent per slice: e = pow2_exp(max |x|), codes =
    rint(x 2^(N-1-e)) clamped (_heuristic.py:51-66).  Returns (q, e, underflow)."""
    x = np.asarray(x, dtype=np.float64)
    mx = np.abs(x).max(axis=axis) if x.shape[axis] else np.zeros(np.delete(x.shape, axis))
    e = pow2_exp(mx)
    q = _pow2_codes(bits, x, np.expand_dims(e, axis))
    return q, e, int(np.count_nonzero((q == 0) & (x != 0)))


def code_norms(codes, axis):
    """L2 norms of integer code vectors (exact sums of squares, _heuristic.py:69-72)."""
    c = np.moveaxis(np.asarray(codes, dtype=np.float64), axis, -1)
    return np.sqrt(np.einsum("...i,...i->...", c, c))


def col_norm_max(bits, qb):
    """Largest column norm of the block magnitudes of (K, N) codes (_heuristic.py:75-82)."""
    bm = mx_mags(bits, qb).astype(np.float64)
    return float(np.sqrt((bm * bm).sum(axis=-2)).max()) if bm.size else 0.0


def acc_guard(bits, x, qa, ea, bmax, mx=MX_DEFAULT):
    """Raise token exponents until the Cauchy-Schwarz bound of every
    accumulator is below the unit's limit (_heuristic.py:85-120).
    Returns (qa, ea, raised)."""
    blk = mx_block(bits)
    u = MX_UNITS[mx][blk]
    hi = (1 << (u["W"] - 1)) - 1
    K = qa.shape[-1]
    raised = np.zeros(ea.shape, bool)
    for _ in range(64):
        am = mx_mags(bits, qa).astype(np.float64)
        an = np.sqrt((am * am).sum(axis=-1))
        prod = an * bmax
        bound = (prod / float(1 << (30 - u["F"])) + K) if blk == 16 else prod
        bad = bound * (1 + 1e-12) + 1 > hi
        if not bad.any():
            return qa, ea, int(np.count_nonzero(raised))
        ea = np.where(bad, ea + 1, ea)
        raised |= bad
        qa = np.where(bad[:, None], _pow2_codes(bits, x, ea[:, None]), qa)
    raise RuntimeError("accumulator guard did not converge")


def wide_plan(bits, na, nb, ea, eb, K, bias_abs=None):
    """Per output shift and redo shift (_heuristic.py:123-169) from the
    dequantized row / column norms.  Returns (shift, shift_l2, h)."""
    h = h_for(K)
    prod = na[:, None] * nb[None, :]
    l2 = pow2_exp(prod)
    base = ea[:, None] + eb[None, :]
    if bias_abs is None:
        target = l2 - h
    else:
        ba = np.broadcast_to(np.asarray(bias_abs, dtype=np.float64), base.shape)
        target = np.where(ba > 0, np.maximum(l2 - h, pow2_exp(ba)), l2 - h)
    shift = np.clip(base - target, SHIFT_MIN, SHIFT_MAX)
    l2_redo = l2 if bias_abs is None else pow2_exp(prod + np.asarray(bias_abs, dtype=np.float64))
    return shift, np.clip(base - l2_redo, SHIFT_MIN, SHIFT_MAX), h


def bias_codes(bits, b, fe):
    """The bias at each output's exponent: rint(b 2^(N-1-fe)) clamped
    (_core.py:182-190).  Returns (codes, clamped)."""
    M, _ = consts(bits)
    with np.errstate(over="ignore"):
        raw = np.rint(np.ldexp(np.asarray(b, dtype=np.float64), (bits - 1 - fe).astype(np.int64)))
    return np.clip(raw, -M, M).astype(np.int64), np.abs(raw) > M


def wide_finish(bits, acc, F, base, shift, shift_redo, bias=None):
    """POP at ``shift``, the bias added with the saturating add, and a second
    POP at ``shift_redo`` where the code or the sum reached +-M or the bias
    code clamped, on a nonzero output (_core.py:68-98, :162-179).
    Returns (y codes, used shift, saturated, flushed, redo mask)."""
    M, _ = consts(bits)
    acc = _i64(acc)

    def post(sh):
        """(sum, pop overflow, pop underflow, add saturated, nonzero, pop codes) at shift ``sh``."""
        q, over, under = wide_pop(bits, acc, sh, F)
        if bias is None:
            return q, over, under, np.zeros(q.shape, bool), acc != 0, q
        bq, clamped = bias_codes(bits, np.broadcast_to(bias, q.shape), base - sh)
        y, ev = add(bits, q, bq)
        return y, over, under, ev["overflow"] | clamped, (acc != 0) | (bq != 0), q

    y, over, under, add_sat, nz, q = post(shift)
    used = np.broadcast_to(shift, acc.shape).copy()
    redo = np.zeros(acc.shape, bool)
    if shift_redo is not None:
        redo = ((np.abs(q) >= M) | (np.abs(y) >= M) | add_sat) & nz
        if redo.any():
            y2, over2, under2, add_sat2, _, _ = post(shift_redo)
            y = np.where(redo, y2, y)
            add_sat = np.where(redo, add_sat2, add_sat)
            over = np.where(redo, over2, over)
            under = np.where(redo, under2, under)
            used = np.where(redo, shift_redo, used)
    return y, used, over | add_sat, under, redo


def _wide_core(bits, x, qa, ea, in_under, qb, eb, w_under, bias, shift, mx, acc_fn):
    """Guard, plan, accumulation, finish and dequantization shared by the
    linear and the activation matmul (_core.py:463-534)."""
    P = bits - 1
    qa, ea, raised = acc_guard(bits, x, qa, ea, col_norm_max(bits, qb), mx)
    base = ea[:, None] + eb[None, :]
    if shift is None:
        na = code_norms(qa, -1) * np.ldexp(1.0, (ea - P).astype(np.int64))
        nb = code_norms(qb, -2) * np.ldexp(1.0, (eb - P).astype(np.int64))
        sh, sh_redo, h = wide_plan(bits, na, nb, ea, eb, x.shape[-1], None if bias is None else np.abs(bias))
    else:
        sh, sh_redo, h = np.full(base.shape, int(check_shift(shift))), None, None
    acc, clipped, F = (acc_fn or wide_acc)(bits, qa, qb, mx)
    y, used, sat, under, redo = wide_finish(bits, acc, F, base, sh, sh_redo, bias)
    fe = base - used
    with np.errstate(over="ignore"):
        yf = np.ldexp(y.astype(np.float64), (fe - P).astype(np.int64))
    bsat = 0 if bias is None else int(np.count_nonzero(bias_codes(bits, np.broadcast_to(bias, fe.shape), fe)[1]))
    return yf, {"saturated": int(sat.sum()), "exact": True, "underflow": int(under.sum()),
                "input_underflow": in_under, "weight_underflow": w_under, "bias_saturated": bsat,
                "headroom_bits": 0.0, "outputs": int(y.size),
                "act_scale": float(np.ldexp(1.0, int(ea.max()))) if ea.size else 1.0, "accumulate": "wide",
                "shift_min": int(used.min()) if used.size else None,
                "shift_max": int(used.max()) if used.size else None, "h": h, "redone": int(redo.sum()),
                "flushed": int(under.sum()), "acc_clipped": int(clipped.sum()), "guard_raised": raised}


def wide_linear(x, w, b, bits, shift=None, mx=MX_DEFAULT, acc_fn=None):
    """y = x W^T + b on the MX engine with the wide rule (_core.py:569-600):
    per-token and per-channel power-of-two exponents, the guard, the plan,
    one accumulation, POP + bias + redo, float64 dequantization.  ``acc_fn``
    replaces ``wide_acc`` (the C oracle).  Returns (y float64, status dict)."""
    x = np.asarray(x, dtype=np.float64)
    qa, ea, in_under = quantize_pow2(bits, x, -1)
    qw, ew, w_under = quantize_pow2(bits, np.asarray(w, dtype=np.float64), -1)
    bias = None if b is None else np.asarray(b, dtype=np.float64)
    return _wide_core(bits, x, qa, ea, in_under, qw.T, ew, w_under, bias, shift, mx, acc_fn)


def wide_matmul(a, b, bits, shift=None, mx=MX_DEFAULT, acc_fn=None):
    """(M, K) @ (K, N) of two activations on the MX engine: one exponent per
    row of a and per column of b (_core.py:537-557)."""
    a = np.asarray(a, dtype=np.float64)
    qa, ea, ua = quantize_pow2(bits, a, -1)
    qb, eb, ub = quantize_pow2(bits, np.asarray(b, dtype=np.float64), -2)
    return _wide_core(bits, a, qa, ea, ua + ub, qb, eb, 0, None, shift, mx, acc_fn)


# --- the chip's sign-magnitude memory format (src/sf/_vectorized.py:78-89) ----------------

def to_bits(bits, codes):
    """Signed codes -> sign-magnitude words: sign at bit N-1, |k| below it."""
    k = _i64(codes)
    return np.where(k < 0, (1 << (bits - 1)) | (-k), k).astype(np.uint16)


def from_bits(bits, words):
    """Sign-magnitude words -> codes (the sign-only word reads as 0).
    Returns (codes, fits): ``fits`` False where a word has bits at or above N."""
    M, _ = consts(bits)
    b = _i64(words)
    mag = b & M
    return np.where((b >> (bits - 1)) & 1, -mag, mag), (b >= 0) & (b < (1 << bits))
