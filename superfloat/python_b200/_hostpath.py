"""Elementwise ops on host-resident codes: chunked and double-buffered.

A caller whose codes live in host memory (int16, pinned) gets the same
kernels with the copies hidden behind them: the element range is cut into
chunks (the last few smaller, so that the drain after the last copy in is
short), and each chunk's host-to-device copies, kernel and device-to-host copy
are queued on one of two streams, so one chunk's copies overlap the other's
kernel and the copy engines run both directions at once.  Status counts
accumulate on the device and are read once at the end.
"""
from __future__ import annotations

import numpy as np

from . import _lib

_ARITY = {"add": 2, "sub": 2, "mul": 2, "div": 2, "fma": 3, "neg": 1, "abs": 1, "sqrt": 1, "pow": 1}


def cuts(n: int, chunk: int) -> list:
    """``[lo, hi)`` ranges covering ``n`` elements for the pipeline: full
    chunks, then the last two chunks' worth halved step by step down to
    chunk / 8.  After the last host-to-device copy only the smallest chunk's
    kernel and copy back are left, so one op's drain is short.  Every ``lo``
    is a multiple of 8 codes (16 bytes), which keeps the kernel's vector path."""
    small = max(chunk // 8, 8)
    out, lo = [], 0
    while lo < n:
        rem = n - lo
        if rem > 2 * chunk:
            m = chunk
        elif rem > small:
            m = min(chunk, (rem // 2 + 7) & ~7)
        else:
            m = rem
        out.append((lo, lo + m))
        lo += m
    return out


class HostPipeline:
    """Device staging for host-buffer elementwise ops on one B200Device."""

    def __init__(self, dev, chunk: int = 1 << 24, slots: int = 2):
        import torch
        self.dev = dev
        self.chunk = chunk
        d = dev.torch_device
        self.streams = [torch.cuda.Stream(device=d) for _ in range(slots)]
        self.ins = [[torch.empty(chunk, dtype=torch.int16, device=d) for _ in range(3)] for _ in range(slots)]
        self.outs = [torch.empty(chunk, dtype=torch.int16, device=d) for _ in range(slots)]
        self.flags = [torch.empty(chunk, dtype=torch.uint8, device=d) for _ in range(slots)]
        self.counts = [torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device=d) for _ in range(slots)]

    def run(self, op, fmt, *xs, out, flags_out=None, pow_n: int = 0, layout: str = "codes"):
        """``out[i] = op(xs...)[i]`` over host int16 tensors of equal length
        (pinned for the copies to overlap).  Returns the event counts (numpy
        int64[8]); per-output event bytes go to ``flags_out`` when given.
        ``layout="signmag"``: operands and result are the chip's
        sign-magnitude words (carried in int16 tensors), converted inside the
        kernel; ValueError when a word does not fit the width."""
        if layout not in ("codes", "signmag"):
            raise ValueError(f"layout must be 'codes' or 'signmag', got {layout!r}")
        import torch
        n = out.numel()
        for c in self.counts:
            c.zero_()
        cur = torch.cuda.current_stream(self.dev.torch_device)
        for s in self.streams:
            s.wait_stream(cur)
        for k, (lo, hi) in enumerate(cuts(n, self.chunk)):
            m = hi - lo
            slot = k % len(self.streams)
            st = self.streams[slot]
            with torch.cuda.stream(st):
                ins = [self.ins[slot][i][:m] for i in range(len(xs))]
                for dst, src in zip(ins, xs):
                    dst.copy_(src[lo:hi], non_blocking=True)
                o = self.outs[slot][:m]
                fl = self.flags[slot][:m] if flags_out is not None else None
                b = ins[1] if len(ins) > 1 else None
                c = ins[2] if len(ins) > 2 else None
                if layout == "signmag":
                    _lib.elementwise_signmag(op, fmt.bits, ins[0], b, c, o, fl, self.counts[slot], pow_n=pow_n,
                                             stream=st)
                else:
                    _lib.elementwise(op, fmt.bits, ins[0], b, c, o, fl, self.counts[slot], pow_n=pow_n, stream=st)
                out[lo:hi].copy_(o, non_blocking=True)
                if flags_out is not None:
                    flags_out[lo:hi].copy_(fl, non_blocking=True)
        for s in self.streams:
            cur.wait_stream(s)
        total = self.counts[0].clone()
        for c in self.counts[1:]:
            total += c
        res = total.cpu().numpy()
        _lib.check_counts(res)
        if layout == "signmag":
            _lib.check_patterns(res, fmt.bits)
        return res


def plugin_run(dev, pipe: HostPipeline, op, fmt, *operands, n_pow: int = 0):
    """The ``Device.run`` contract (int64 codes in, int64 codes and boolean
    masks out) for equal-shape operands, through the host pipeline: narrowing
    and widening on the host with torch's threaded copies, the rest on the GPU."""
    import torch
    ops = [np.ascontiguousarray(o, dtype=np.int64) for o in operands]
    shape = ops[0].shape
    n = ops[0].size
    xs = []
    for o in ops:
        t = torch.empty(n, dtype=torch.int16, pin_memory=True)
        t.copy_(torch.from_numpy(o.reshape(-1)))
        xs.append(t)
    out = torch.empty(n, dtype=torch.int16, pin_memory=True)
    fl = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    counts = pipe.run(op, fmt, *xs, out=out, flags_out=fl, pow_n=n_pow)
    codes = torch.empty(n, dtype=torch.int64)
    codes.copy_(out)
    from ._device import OP_EVENTS, _EVENT_BIT
    masks = {e: ((fl & _EVENT_BIT[e]) != 0).numpy().reshape(shape) for e in OP_EVENTS[op]}
    return codes.numpy().reshape(shape), masks, counts
