"""The SF linear / matmul of converted layers, with the scale policy, on the B200.

Same steps and the same float64 arithmetic as the reference's torch core
(src/sf/torch/_core.py:336-433), run on the GPU:

1. ``sanitize``: NaN / inf in x, W, b go through the error policy
   (src/sf/torch/_core.py:200-232);
2. weight scale ``s_w`` per tensor or per channel and ``W_code = cast(W / s_w)``
   (:256-296); cached per weight tensor version, since inference weights do
   not change between calls;
3. activation scale ``a``: ``a0 = max|x| / max``, then with
   ``headroom="bound"`` raised until the L1 bound proves that no chain step and
   no bias add can saturate (:306-331);
4. the chain matmul ``x_code @ W_code^T`` and the one saturating bias add,
   fused in libsfb200's chain kernel (exact per-output events);
5. ``y = acc / 2^(N-1) * a * s_w`` in float64.

Every float64 operation here (division, multiplication, round half to even)
is IEEE correctly rounded on the GPU as in NumPy, so the codes, scales and
outputs are the reference's, bit for bit.
"""
from __future__ import annotations

import math
import weakref
from collections import OrderedDict
from dataclasses import dataclass

import numpy as np
import torch

from .. import _config, _errstate, _lib
from .._device import get_device
from .._format import FORMATS, SFFormat

WSCALES = ("per_tensor", "per_channel")
HEADROOMS = ("bound", "none")
ACCUMULATES = ("chain", "wide")
_MAX_ITER = 32


@dataclass
class CoreResult:
    y: torch.Tensor
    saturated: int | None
    exact: bool
    underflow: int | None
    input_underflow: int
    weight_underflow: int
    bias_saturated: int
    headroom_bits: float
    outputs: int
    act_scale: float = 1.0
    accumulate: str = "chain"
    shift_min: int | None = None
    shift_max: int | None = None
    h: int | None = None
    redone: int = 0
    flushed: int | None = None
    acc_clipped: int | None = None
    guard_raised: int = 0


def check_args(bits, wscale=None, headroom=None, accumulate=None) -> SFFormat:
    if accumulate is not None and accumulate not in ACCUMULATES:
        raise ValueError(f"accumulate must be one of {ACCUMULATES}, got {accumulate!r}")
    if bits not in FORMATS:
        raise ValueError(f"unsupported SF width {bits}")
    if wscale is not None and wscale not in WSCALES:
        raise ValueError(f"scale must be one of {WSCALES}, got {wscale!r}")
    if headroom is not None and headroom not in HEADROOMS:
        raise ValueError(f"headroom must be one of {HEADROOMS}, got {headroom!r}")
    return FORMATS[bits]


def target():
    """The target the torch path runs on (``default_device``)."""
    dev = get_device(_config.get("default_device"))
    if not hasattr(dev, "run_device"):
        from .._errors import SFUnsupportedError
        raise SFUnsupportedError(f"{dev.name} cannot run the torch path (no device-resident entry)")
    return dev


# --- elementwise helpers on float64 device tensors --------------------------------------------

def finite_absmax(x: torch.Tensor) -> float:
    if x.numel() == 0:
        return 0.0
    fin = torch.isfinite(x)
    if not bool(fin.any()):
        return 0.0
    return float(torch.where(fin, x.abs(), torch.zeros((), dtype=x.dtype, device=x.device)).max())


def sanitize(x: torch.Tensor, fmt: SFFormat, what: str) -> torch.Tensor:
    """NaN -> invalid event, +-inf -> overflow event; under a non-raising policy
    NaN becomes 0 and +-inf the tensor's largest finite magnitude (or +-max)."""
    nan = torch.isnan(x)
    inf = torch.isinf(x)
    n_nan, n_inf = int(nan.sum()), int(inf.sum())
    if n_nan:
        _errstate.handle("invalid", f"{fmt.name} {what}: invalid (NaN) in {n_nan} of {x.numel()} element(s)")
    if n_inf:
        _errstate.handle("overflow", f"{fmt.name} {what}: ±inf in {n_inf} of {x.numel()} element(s) (saturates)")
    if n_nan:
        x = torch.where(nan, torch.zeros((), dtype=x.dtype, device=x.device), x)
    if n_inf:
        big = finite_absmax(x)
        if big == 0.0:
            big = fmt.max_code / fmt.scale
        x = torch.where(inf, torch.sign(x) * big, x)
    return x


def cast(fmt: SFFormat, v: torch.Tensor):
    """float64 values -> int16 codes: round half to even, saturate at
    |v| >= 1 - 2^-N, NaN -> 0.  Returns (codes, {event: count tensor})."""
    nan = torch.isnan(v)
    over = (v.abs() >= 1.0 - 2.0 ** -fmt.bits) & ~nan
    fits = ~over & ~nan
    k = torch.round(torch.where(fits, v, torch.zeros((), dtype=v.dtype, device=v.device)) * fmt.scale)
    k = torch.where(over, torch.sign(v) * fmt.max_code, k)
    under = fits & (k == 0) & (v != 0)
    return k.to(torch.int16), {"overflow": over.sum(), "underflow": under.sum(), "invalid": nan.sum()}


# --- weights -----------------------------------------------------------------------------------

def weight_scales(fmt: SFFormat, w: torch.Tensor, wscale: str) -> torch.Tensor:
    """One positive scale per output row from the finite magnitudes
    (src/sf/torch/_core.py:277-289)."""
    m = fmt.max_code / fmt.scale
    fin = torch.where(torch.isfinite(w), w.abs(), torch.zeros((), dtype=w.dtype, device=w.device))
    N = w.shape[0]
    if wscale == "per_tensor":
        amax = float(fin.max()) if w.numel() else 0.0
        return torch.full((N,), amax / m if amax > 0 else 1.0, dtype=torch.float64, device=w.device)
    amax = fin.max(dim=1).values if w.numel() else torch.zeros(N, dtype=torch.float64, device=w.device)
    return torch.where(amax > 0, amax / m, torch.ones((), dtype=torch.float64, device=w.device))


@dataclass
class PreparedWeight:
    """A weight as the chain kernel reads it: W_code^T (K, N) int16, the
    scales, and the L1 statistics the headroom bound needs."""

    kwT: torch.Tensor
    s_w: torch.Tensor
    w_under: int
    max_abs: int          # max |W_code|
    max_col_l1: int       # max_n sum_k |W_code[n, k]|


def _stats_buf(dev, n=1):
    return torch.zeros(n, _lib.QSTATS_WORDS, dtype=torch.int64, device=dev)


def prepare_weight(fmt: SFFormat, w: torch.Tensor, wscale: str) -> PreparedWeight:
    """W_code = cast(W / s_w) per output row, with the statistics the bound
    needs (one fused pass, sfb_quantize)."""
    s = weight_scales(fmt, w, wscale)
    N, K = w.shape
    codes = torch.empty(N, K, dtype=torch.int16, device=w.device)
    st = _stats_buf(w.device)
    if w.numel():
        _lib.quantize(w.contiguous(), N, K, K, 1.0, s.contiguous(), fmt.bits, codes, K, st[0])
    q = _lib.qstats_view(st[0].cpu())
    return PreparedWeight(codes.t().contiguous(), s, q["underflow"], q["max_abs"], q["max_row_l1"])


class WeightCache:
    """Prepared weights keyed by the tensor's storage, shape, strides and
    version counter (an in-place update prepares it again), with a weak
    reference to the owning tensor so a new tensor at a freed address is never
    mistaken for the old one.  Least recently used entries go first."""

    def __init__(self, max_entries: int = 512):
        self.items = OrderedDict()
        self.max_entries = max_entries
        self.hits = self.misses = 0

    @staticmethod
    def _owner(w):
        while w._base is not None:
            w = w._base
        return w

    @staticmethod
    def _key(fmt, w, wscale, dev):
        return (w.untyped_storage().data_ptr(), w.storage_offset(), tuple(w.shape), tuple(w.stride()),
                w._version, w.dtype, str(w.device), fmt.bits, wscale, str(dev))

    def peek(self, fmt, w: torch.Tensor, wscale: str, dev):
        """The prepared weight when it is cached (so finite), else None."""
        hit = self.items.get(self._key(fmt, w, wscale, dev))
        if hit is not None and hit[0]() is not None:
            self.hits += 1
            return hit[1]
        return None

    def get(self, fmt, w: torch.Tensor, wscale: str, dev) -> PreparedWeight:
        key = self._key(fmt, w, wscale, dev)
        hit = self.items.get(key)
        if hit is not None and hit[0]() is not None:
            self.items.move_to_end(key)
            self.hits += 1
            return hit[1]
        self.misses += 1
        wd = w.detach().to(device=dev, dtype=torch.float64)
        finite = bool(torch.isfinite(wd).all())
        wd = sanitize(wd, fmt, "linear weight")
        pw = prepare_weight(fmt, wd, wscale)
        if finite:                                  # a NaN / inf weight raises its events on every call
            self.items[key] = (weakref.ref(self._owner(w)), pw)
        while len(self.items) > self.max_entries:
            self.items.popitem(last=False)
        return pw

    def clear(self):
        self.items.clear()


weight_cache = WeightCache()


# --- the activation scale ------------------------------------------------------------------

class _Quantized:
    """Codes of x / a from one sfb_quantize pass, with the cast's underflow
    count and the L1 statistics (the events dict of ``cast``).  ``done``:
    codes and host statistics of a pass already run (the fused first pass)."""

    def __init__(self, fmt, x2d: torch.Tensor, a: float, done=None):
        if done is not None:
            self.codes, q = done
        else:
            R, K = x2d.shape
            self.codes = torch.empty(R, K, dtype=torch.int16, device=x2d.device)
            st = _stats_buf(x2d.device)
            _lib.quantize(x2d, R, K, x2d.stride(0), a, None, fmt.bits, self.codes, K, st[0])
            q = _lib.qstats_view(st[0].cpu())
        self.events = {"overflow": q["overflow"], "underflow": q["underflow"], "invalid": q["invalid"]}
        self.row_l1, self.max_abs = q["max_row_l1"], q["max_abs"]

    def bound(self, fmt, b_max_abs, b_max_col_l1) -> int:
        if self.codes.numel() == 0:
            return 0
        return min(self.row_l1 * b_max_abs, self.max_abs * b_max_col_l1) // fmt.scale


def activation_fused(fmt, x2d: torch.Tensor, amax: float, b_max_abs: int, b_max_col_l1: int, bias_over_scale,
                     headroom: str, first=None):
    """The activation scale search (src/sf/torch/_core.py:306-331) on a
    float32 / float64 (R, K) device tensor, each cast one sfb_quantize pass
    (``first``: the pass at a0 already run, as (codes, host statistics)).
    Returns (codes, events, a, a0, proven): ``proven`` when the L1 bound shows
    that no chain step can saturate."""
    m = fmt.max_code / fmt.scale
    a0 = amax / m if amax > 0 else 1.0
    a = a0
    q = _Quantized(fmt, x2d, a, done=first)
    if headroom == "none":
        return q.codes, q.events, a, a0, q.bound(fmt, b_max_abs, b_max_col_l1) <= fmt.max_code
    a_bias = bias_over_scale(None)
    if a_bias is not None and math.isfinite(a_bias) and a_bias > a:
        a = a_bias
        q = _Quantized(fmt, x2d, a)
    for _ in range(_MAX_ITER):
        ratio = bias_over_scale(a)
        bias_codes = int(math.ceil(ratio)) if ratio is not None and math.isfinite(ratio) else 0
        chain = q.bound(fmt, b_max_abs, b_max_col_l1)
        bound = chain + bias_codes
        if bound <= fmt.max_code:
            return q.codes, q.events, a, a0, chain <= fmt.max_code
        a *= max(bound / fmt.max_code, 1.0 + 2.0 ** -20)
        q = _Quantized(fmt, x2d, a)
    raise RuntimeError("sf: headroom search did not converge")


def _scanned(x: torch.Tensor, cuda, fmt, what: str):
    """x on the device as contiguous float32 / float64, with its finite
    max |x|: one sfb_scan pass; the error policy (``sanitize``) runs only when
    the scan found a NaN or an inf."""
    x = x.detach().to(device=cuda)
    if x.dtype not in (torch.float32, torch.float64):
        x = x.to(torch.float32)                            # float16 / bfloat16 widen exactly
    x = x.contiguous()
    st = _stats_buf(cuda)
    _lib.scan(x, st[0])
    sc = _lib.qstats_view(st[0].cpu())
    if sc["nan"] or sc["inf"]:
        x = sanitize(x.to(torch.float64), fmt, what)
        return x, finite_absmax(x)
    return x, sc["absmax"]


class BiasCache:
    """A layer's bias as the scale search reads it, per bias version and
    prepared weight: the sanitized float64 bias on the device, and on the
    host |b| / s_w and the scale that fits the largest finite ratio.  Biases
    holding NaN / inf are not cached (their events fire on every call)."""

    def __init__(self, max_entries: int = 512):
        self.items = OrderedDict()
        self.max_entries = max_entries

    @staticmethod
    def _key(fmt, b, pw, cuda):
        return (b.untyped_storage().data_ptr(), b.storage_offset(), tuple(b.shape), tuple(b.stride()), b._version,
                b.dtype, str(b.device), id(pw), fmt.bits, str(cuda))

    def peek(self, fmt, b: torch.Tensor, pw: PreparedWeight, cuda):
        """(bias float64, need, a_bias, max need) when cached (so finite), else None."""
        hit = self.items.get(self._key(fmt, b, pw, cuda))
        if hit is not None and hit[0]() is not None and hit[1]() is pw:
            return hit[2]
        return None

    def get(self, fmt, b: torch.Tensor, pw: PreparedWeight, cuda):
        key = self._key(fmt, b, pw, cuda)
        hit = self.items.get(key)
        if hit is not None and hit[0]() is not None and hit[1]() is pw:
            self.items.move_to_end(key)
            return hit[2]
        bd = b.detach().to(device=cuda, dtype=torch.float64)
        finite = bool(torch.isfinite(bd).all())
        bd = sanitize(bd, fmt, "linear bias")
        need = (bd.abs() / pw.s_w).cpu().numpy()            # may hold inf; host float64, as the reference
        fin = np.isfinite(need)
        a_bias = float(need[fin].max()) / (fmt.max_code / fmt.scale) if fin.any() else 0.0
        val = (bd, need, a_bias, float(need.max()) if need.size else 0.0)
        if finite:
            owner = b
            while owner._base is not None:
                owner = owner._base
            self.items[key] = (weakref.ref(owner), weakref.ref(pw), val)
            while len(self.items) > self.max_entries:
                self.items.popitem(last=False)
        return val

    def clear(self):
        self.items.clear()


bias_cache = BiasCache()


# --- linear ----------------------------------------------------------------------------------

def linear(x: torch.Tensor, w: torch.Tensor, b, bits: int, wscale: str = "per_tensor",
           headroom: str = "bound", dev=None, out_dtype=torch.float32) -> CoreResult:
    """x: (R, K), w: (N, K), b: (N,) or None, any float dtype, any device;
    the result ``y`` (float32, or float64 when ``out_dtype`` is) is on the
    target's CUDA device, rounded once from the float64 dequantization."""
    fmt = check_args(bits, wscale, headroom)
    dev = dev or target()
    cuda = dev.torch_device
    S, M = fmt.scale, fmt.max_code
    x = x.detach().to(device=cuda)
    if x.dtype not in (torch.float32, torch.float64):
        x = x.to(torch.float32)                            # float16 / bfloat16 widen exactly
    x = x.contiguous()
    R, K = x.shape
    m = M / S
    if headroom == "bound":
        r = _linear_on_device(fmt, x, w, b, wscale, cuda, out_dtype)
        if r is not None:
            return r
    # the scan and the first quantize (scale max|x| / m, taken on the device): one statistics read
    st = _stats_buf(cuda, 2)
    kx0 = torch.empty(R, K, dtype=torch.int16, device=cuda)
    _lib.scan(x, st[0])
    _lib.quantize_auto(x, R, K, K, st[0], m, fmt.bits, kx0, K, st[1])
    host = st.cpu()
    sc, q0 = _lib.qstats_view(host[0]), _lib.qstats_view(host[1])
    first = None
    if sc["nan"] or sc["inf"]:                              # the policy decides; then the finite values
        x = sanitize(x.to(torch.float64), fmt, "linear input")
        amax = finite_absmax(x)
    else:
        amax = sc["absmax"]
        first = (kx0, q0)
    pw = weight_cache.get(fmt, w, wscale, cuda)
    bd = need = None
    if b is not None:
        bd, need, a_bias, _ = bias_cache.get(fmt, b, pw, cuda)
    if b is not None and bd.numel():
        def bias_over_scale(a):
            if a is None:
                return a_bias
            with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
                return float((need / a).max() * S)
    else:
        def bias_over_scale(a):
            return None if a is None else 0.0

    kx, ev_x, a, a0, proven = activation_fused(fmt, x, amax, pw.max_abs, pw.max_col_l1, bias_over_scale, headroom,
                                               first=first)
    kb = None
    cnt = torch.zeros(_lib.N_COUNTS + 1, dtype=torch.int64, device=cuda)   # + the bias codes' saturations
    if b is not None:
        kb, ev_b = cast(fmt, bd / (a * pw.s_w))
        cnt[_lib.N_COUNTS] = ev_b["overflow"]
    N = pw.kwT.shape[1]
    y = torch.empty(R, N, dtype=torch.float64 if out_dtype == torch.float64 else torch.float32, device=cuda)
    _lib.linear_chain(fmt.bits, kx, pw.kwT, kb, a, pw.s_w, proven,
                      y if y.dtype == torch.float32 else None, y if y.dtype == torch.float64 else None,
                      None, None, cnt, R, N, K, K, N)
    c = cnt.cpu().numpy()
    _lib.check_counts(c[:_lib.N_COUNTS])
    return CoreResult(y=y, saturated=int(c[0]), exact=True, underflow=int(c[1]),
                      input_underflow=int(ev_x["underflow"]), weight_underflow=pw.w_under,
                      bias_saturated=int(c[_lib.N_COUNTS]), headroom_bits=math.log2(a / a0) if a0 > 0 else 0.0,
                      outputs=R * N, act_scale=a)


device_path_calls = 0          # layers completed by _linear_on_device (the tests read it)


def _linear_on_device(fmt, x, w, b, wscale, cuda, out_dtype):
    """The whole layer queued on the device with one host read at the end:
    the scale search (sfb_linear_scale), the bias codes and the chain read the
    scale from device memory.  Runs when the weight (and bias) are prepared
    and so finite; returns None otherwise, and when the input held NaN / inf,
    so that the host path applies the error policy in the reference's order."""
    pw = weight_cache.peek(fmt, w, wscale, cuda)
    if pw is None:
        return None
    bias = None
    if b is not None:
        bias = bias_cache.peek(fmt, b, pw, cuda)
        if bias is None:
            return None
    R, K = x.shape
    N = pw.kwT.shape[1]
    kx = torch.empty(R, K, dtype=torch.int16, device=cuda)
    words = torch.zeros(_lib.N_COUNTS + 1 + _lib.SCALE_RESULT_WORDS, dtype=torch.int64, device=cuda)
    cnt, n_over, res = words[:_lib.N_COUNTS], words[_lib.N_COUNTS:_lib.N_COUNTS + 1], words[_lib.N_COUNTS + 1:]
    scratch = torch.empty(_lib.linear_scale_scratch(), dtype=torch.uint8, device=cuda)
    has_bias = bias is not None and bias[0].numel() > 0
    need_max, a_bias = (bias[3], bias[2]) if has_bias else (0.0, 0.0)
    _lib.linear_scale(x, R, K, K, fmt.bits, pw.max_abs, pw.max_col_l1, has_bias, need_max, a_bias, kx, res, scratch)
    a_dev = res[0:1].view(torch.float64)
    kb = None
    if bias is not None:
        kb = torch.empty(N, dtype=torch.int16, device=cuda)
        _lib.bias_codes(fmt.bits, bias[0], a_dev, pw.s_w, N, kb, n_over)
    y = torch.empty(R, N, dtype=torch.float64 if out_dtype == torch.float64 else torch.float32, device=cuda)
    _lib.linear_chain_dev(fmt.bits, kx, pw.kwT, kb, a_dev, pw.s_w, y if y.dtype == torch.float32 else None,
                          y if y.dtype == torch.float64 else None, cnt, R, N, K, K, N)
    host = words.cpu()
    c = host.numpy()
    r = c[_lib.N_COUNTS + 1:]
    nan_count, inf_count, err = int(r[4]), int(r[5]), int(r[7])
    if nan_count or inf_count:
        return None
    if err:
        raise RuntimeError("sf: headroom search did not converge")
    _lib.check_counts(c[:_lib.N_COUNTS])
    a, a0 = (float(v) for v in host[_lib.N_COUNTS + 1:_lib.N_COUNTS + 3].view(torch.float64))
    global device_path_calls
    device_path_calls += 1
    return CoreResult(y=y, saturated=int(c[0]), exact=True, underflow=int(c[1]), input_underflow=int(r[6]),
                      weight_underflow=pw.w_under, bias_saturated=int(c[_lib.N_COUNTS]),
                      headroom_bits=math.log2(a / a0) if a0 > 0 else 0.0, outputs=R * N, act_scale=a)


def matmul(a_val: torch.Tensor, b_val: torch.Tensor, bits: int, headroom: str = "bound", dev=None) -> CoreResult:
    """(..., M, K) @ (..., K, N) of two activations, both with a dynamic
    per-tensor scale, headroom on ``a`` (src/sf/torch/_core.py:412-433)."""
    fmt = check_args(bits, None, headroom)
    dev = dev or target()
    cuda = dev.torch_device
    S, M = fmt.scale, fmt.max_code
    m = M / S
    a_val, _amax = _scanned(a_val, cuda, fmt, "matmul left operand")
    b_val = sanitize(b_val.detach().to(device=cuda, dtype=torch.float64), fmt, "matmul right operand")
    bmax = finite_absmax(b_val)
    s_b = bmax / m if bmax > 0 else 1.0
    kb, ev_b = cast(fmt, b_val / s_b)
    if kb.numel() and kb.shape[-2]:
        ab = kb.abs().to(torch.int64)
        st = torch.stack([ab.max(), ab.sum(-2).max()]).cpu()
        b_max, b_l1 = int(st[0]), int(st[1])
    else:
        b_max = b_l1 = 0
    K = a_val.shape[-1]
    ka, ev_a, a, a0, _ = activation_fused(fmt, a_val.reshape(-1, K), _amax, b_max, b_l1,
                                          lambda _a: None if _a is None else 0.0, headroom)
    ka = ka.reshape(a_val.shape)
    acc, cnt, _ = dev.run_device("matmul", fmt, ka, kb)
    c = cnt.cpu()
    y = acc.to(torch.float64) / S * a * s_b
    return CoreResult(y=y, saturated=int(c[0]), exact=True, underflow=int(c[1]),
                      input_underflow=int(ev_a["underflow"]) + int(ev_b["underflow"]), weight_underflow=0,
                      bias_saturated=0, headroom_bits=math.log2(a / a0) if a0 > 0 else 0.0,
                      outputs=int(acc.numel()), act_scale=a)


def fake_quantize(x: torch.Tensor, bits: int, mode: str, scale: float):
    """Values snapped to the SF grid (src/sf/torch/_core.py:438-460).
    Returns (values float64, codes, scale, event counts)."""
    fmt = check_args(bits)
    if mode == "none":
        s = 1.0
    elif mode == "dynamic":
        amax = finite_absmax(x)
        s = amax / (fmt.max_code / fmt.scale) if amax > 0 else 1.0
    elif mode == "fixed":
        if not (scale > 0 and math.isfinite(scale)):
            raise ValueError("scale must be a positive finite float")
        s = float(scale)
    else:
        raise ValueError(f"unknown quantize mode {mode!r}")
    codes, ev = cast(fmt, x / s)
    return codes.to(torch.float64) / fmt.scale * s, codes, s, ev


def dequantize_weight(fmt, w: torch.Tensor, wscale: str) -> torch.Tensor:
    s = weight_scales(fmt, w, wscale)
    codes, _ = cast(fmt, w / s[:, None])
    return codes.to(torch.float64) / fmt.scale * s[:, None]
