"""Pre-flight gate for heavy ops: decide on the host what can be decided.

Mirrors the reference's gate (src/sf/_preflight.py:57-220):

* known answers read off the inputs: div0 (div) and invalid (sqrt) counts;
* range bound: ``safe`` (no element can saturate), ``certain`` (every element
  must saturate: refused under ``config(preflight="raise")``), else
  ``unknown``;
* probe for the undecidable band: a sample of the real inputs (the same
  sample rule as the reference) is run, and if every probed output
  saturates the op is ``suspected`` (warned by default, refused or verified
  under ``config(suspect=...)``).

The bounds are O(inputs) NumPy reductions on the host codes; the probe and
the replay run the sampled op on the target itself.
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass, field

import numpy as np

from . import _config, _errstate
from ._errors import SFOverflowError, SFOverflowWarning, SFPreflightWarning
from ._format import SFFormat


@dataclass
class Verdict:
    kind: str
    reason: str = ""
    events: dict = field(default_factory=dict)


def _maxabs(c):
    c = np.asarray(c)
    return int(np.abs(c).max()) if c.size else 0


def _minabs(c):
    c = np.asarray(c)
    return int(np.abs(c).min()) if c.size else 0


def chain_bound(fmt: SFFormat, a, b) -> int:
    """L1 bound on every partial sum of the chain matmul, in codes
    (src/sf/_linalg.py:84-106)."""
    a, b = np.abs(np.asarray(a, np.int64)), np.abs(np.asarray(b, np.int64))
    if a.size == 0 or b.size == 0 or a.shape[-1] == 0:
        return 0
    r = int(a.sum(axis=-1).max()) * int(b.max())
    c = int(a.max()) * int(b.sum(axis=-2).max())
    return min(r, c) // fmt.scale


def mx_mags(fmt: SFFormat, codes):
    m = np.abs(np.asarray(codes, np.int64)) << (16 - fmt.bits)
    return m if fmt.bits >= 9 else m >> 8


def wide_acc_safe(fmt: SFFormat, a, b, mx="v4.9.2") -> bool:
    """No accumulator of the wide matmul can reach its limit
    (src/sf/_linalg.py:351-369)."""
    a, b = np.asarray(a, np.int64), np.asarray(b, np.int64)
    if a.size == 0 or b.size == 0 or a.shape[-1] == 0:
        return True
    am, bm = mx_mags(fmt, a), mx_mags(fmt, b)
    l1 = min(int(am.sum(axis=-1).max()) * int(bm.max()), int(am.max()) * int(bm.sum(axis=-2).max()))
    W, F = {("v4.9.2", True): (32, 22), ("v4.9.2", False): (32, 14),
            ("v4.8.1", True): (25, 19), ("v4.8.1", False): (20, 14)}[(mx, fmt.bits >= 9)]
    bound = l1 // (1 << (30 - F)) + a.shape[-1] if fmt.bits >= 9 else l1
    return bound <= (1 << (W - 1)) - 1


def check(op, fmt: SFFormat, *ops, **kw) -> Verdict:
    M, S = fmt.max_code, fmt.scale
    ev = {}
    if any(np.size(o) == 0 for o in ops):
        return Verdict("safe", "no live elements", ev)
    if op == "div":
        shape = np.broadcast_shapes(*(np.shape(o) for o in ops))
        ev["div0"] = int(np.count_nonzero(np.broadcast_to(np.asarray(ops[1]) == 0, shape)))
    if op == "sqrt":
        ev["invalid"] = int(np.count_nonzero(np.asarray(ops[0]) < 0))
    if op in ("add", "sub"):
        a, b = _maxabs(ops[0]), _maxabs(ops[1])
        if a + b <= M:
            return Verdict("safe", "max|a| + max|b| <= max", ev)
        pa, pb = np.asarray(ops[0]), np.asarray(ops[1])
        sb = -pb if op == "sub" else pb
        if _minabs(pa) + _minabs(pb) > M and ((np.all(pa > 0) and np.all(sb > 0)) or
                                               (np.all(pa < 0) and np.all(sb < 0))):
            return Verdict("certain", "every element of a and b overflows", ev)
        return Verdict("unknown", "", ev)
    if op in ("mul", "neg", "abs"):
        return Verdict("safe", "cannot overflow", ev)
    if op == "fma":
        a, b, c = (_maxabs(o) for o in ops)
        if (a * b) // S + c <= M:
            return Verdict("safe", "trunc(max|a| max|b|) + max|c| <= max", ev)
        return Verdict("unknown", "", ev)
    if op == "div":
        shape = np.broadcast_shapes(*(np.shape(o) for o in ops))
        a, b = (np.broadcast_to(np.asarray(o), shape) for o in ops)
        nz = b != 0
        if nz.any() and np.all(np.abs(a[nz]) >= np.abs(b[nz])) and np.all(a[nz] != 0):
            return Verdict("certain", "|a| >= |b| for every element", ev)
        if nz.all() and np.all(np.abs(a) < np.abs(b)):
            return Verdict("safe", "|a| < |b| everywhere", ev)
        return Verdict("unknown", "", ev)
    if op in ("sqrt", "pow"):
        return Verdict("safe", f"{op} cannot overflow", ev)
    if op == "matmul":
        if chain_bound(fmt, ops[0], ops[1]) <= M:
            return Verdict("safe", "L1 bound: no partial sum can exceed max", ev)
        return Verdict("unknown", "", ev)
    if op == "sum":                                 # src/sf/_preflight.py:105-109
        a = np.asarray(ops[0])
        K = a.shape[kw.get("axis", 0)] if a.ndim else 1
        if K * _maxabs(a) <= M:
            return Verdict("safe", "K * max|a| <= max", ev)
        return Verdict("unknown", "", ev)
    return Verdict("unknown", "", ev)


def probe(op, fmt, dev, *ops, **kw):
    """The reference's sample (src/sf/_preflight.py:114-152), run on ``dev``:
    True when every probed output saturates."""
    n = _config.get("probe_size")
    rng = np.random.default_rng(0)
    if op in ("add", "sub", "fma", "div"):
        shape = np.broadcast_shapes(*(np.shape(o) for o in ops))
        flat = [np.broadcast_to(np.asarray(o), shape).reshape(-1) for o in ops]
        total = flat[0].size
        if total == 0:
            return False
        idx = np.unique(np.concatenate([rng.integers(0, total, min(n, total)),
                                        np.argsort(np.abs(flat[0]))[-8:], np.argsort(np.abs(flat[1]))[-8:],
                                        np.argsort(np.abs(flat[0]))[:8]]))
        _, masks = dev.evaluate(op, fmt, *(f[idx] for f in flat))
        return bool(masks["overflow"].all())
    if op == "matmul":
        a, b = np.asarray(ops[0]), np.asarray(ops[1])
        a2 = a.reshape(-1, a.shape[-2], a.shape[-1])[0]
        b2 = b.reshape(-1, b.shape[-2], b.shape[-1])[0]
        if a2.shape[0] == 0 or b2.shape[1] == 0:
            return False
        rows, cols = min(8, a2.shape[0]), min(8, b2.shape[1])
        ra = np.unique(np.concatenate([rng.integers(0, a2.shape[0], rows), np.argsort(np.abs(a2).max(axis=1))[-2:]]))
        cb = np.unique(np.concatenate([rng.integers(0, b2.shape[1], cols), np.argsort(np.abs(b2).max(axis=0))[-2:]]))
        _, masks = dev.evaluate("matmul", fmt, a2[ra], b2[:, cb])
        return bool(masks["overflow"].all())
    return None


def replay_all_saturate(op, fmt, dev, *ops, **kw) -> bool:
    _, masks = dev.evaluate(op, fmt, *ops, **kw)
    over = masks.get("overflow")
    return over is not None and np.size(over) > 0 and bool(np.all(over))


def decide(v: Verdict, op, fmt, dev, *ops, **kw) -> Verdict:
    """Probe, then apply ``suspect=`` and ``preflight=`` (src/sf/_preflight.py:184-220)."""
    if v.kind == "unknown" and _config.get("probe"):
        if probe(op, fmt, dev, *ops, **kw):
            v = Verdict("suspected", "golden-vector probe: every probed output saturates", v.events)
    if v.kind == "suspected":
        policy = _config.get("suspect")
        if policy == "verify":
            v = Verdict("certain", "host replay: every output saturates", v.events) \
                if replay_all_saturate(op, fmt, dev, *ops, **kw) else Verdict("unknown", "", v.events)
        elif policy == "raise":
            raise SFOverflowError(f"pre-flight: {op} on {fmt.name} is suspected to saturate on every element "
                                  f"({v.reason}); not launched (sf.config(suspect=...) controls this)")
        elif policy == "warn":
            warnings.warn(f"pre-flight: {op} on {fmt.name} is suspected to saturate on every element "
                          f"({v.reason}); launching anyway", SFPreflightWarning,
                          stacklevel=_errstate.user_stacklevel())
    if v.kind == "certain":
        policy = _config.get("preflight")
        msg = f"pre-flight: {op} on {fmt.name} would saturate on every element ({v.reason}); not launched"
        if policy == "raise":
            raise SFOverflowError(msg)
        if policy == "warn":
            warnings.warn(msg, SFOverflowWarning, stacklevel=_errstate.user_stacklevel())
    return v
