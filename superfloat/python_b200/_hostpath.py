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


class MultiOpPipeline:
    """Several elementwise ops over the same host-resident operands (int16
    codes in pinned host memory), chunked over several streams: per chunk
    each distinct operand is copied in once, every op runs on it, and every
    result is copied back, so an operand that several ops read crosses PCIe
    once per chunk.  One chunk's copies overlap the other streams' kernels,
    and the copy engines run both directions at once.  Status counts
    accumulate per op and stream on the device and come back with the last
    copies of each stream.

    ``run_async`` only queues a call and returns a ``Pending`` whose
    ``result()`` waits for it and gives the counts, so a caller can queue the
    next call's copies before reading this one's counts: consecutive calls
    then keep the copy engines busy instead of draining between calls."""

    def __init__(self, dev, names, ops, chunk: int = 1 << 23, slots: int = 4):
        import torch
        self.dev = dev
        self.chunk = chunk
        self.names = list(names)                 # operand names
        self.ops = list(ops)                     # (op, (operand names...)) in run order
        d = dev.torch_device
        self.streams = [torch.cuda.Stream(device=d) for _ in range(slots)]
        self.ins = [{nm: torch.empty(chunk, dtype=torch.int16, device=d) for nm in self.names}
                    for _ in range(slots)]
        self.outs = [[torch.empty(chunk, dtype=torch.int16, device=d) for _ in self.ops] for _ in range(slots)]

    class Pending:
        def __init__(self, done, host_counts, dev_counts):
            self.done, self.host_counts, self.dev_counts = done, host_counts, dev_counts

        def result(self):
            """Wait for the call; its event counts per op (numpy int64[ops, 8])."""
            for ev in self.done:
                ev.synchronize()
            res = self.host_counts.numpy().sum(0)
            for c in res:
                _lib.check_counts(c)
            return res

    def run_async(self, fmt, inputs: dict, outputs: list) -> "MultiOpPipeline.Pending":
        """Queue ``outputs[i][j] = ops[i](inputs...)[j]`` for host int16
        tensors of one length (pinned for the copies to overlap)."""
        import torch
        n = inputs[self.names[0]].numel()
        d = self.dev.torch_device
        cur = torch.cuda.current_stream(d)
        counts = torch.zeros(len(self.streams), len(self.ops), _lib.N_COUNTS, dtype=torch.int64, device=d)
        host_counts = torch.empty(counts.shape, dtype=torch.int64, pin_memory=True)
        for st in self.streams:
            st.wait_stream(cur)                  # the zeroed counts
        for k, (lo, hi) in enumerate(cuts(n, self.chunk)):
            m = hi - lo
            slot = k % len(self.streams)
            st = self.streams[slot]
            with torch.cuda.stream(st):
                dev_in = {nm: self.ins[slot][nm][:m] for nm in self.names}
                for nm in self.names:
                    dev_in[nm].copy_(inputs[nm][lo:hi], non_blocking=True)
                for i, (op, args) in enumerate(self.ops):
                    xs = [dev_in[a] for a in args] + [None] * (3 - len(args))
                    o = self.outs[slot][i][:m]
                    _lib.elementwise(op, fmt.bits, xs[0], xs[1], xs[2], o, None, counts[slot, i], stream=st)
                    outputs[i][lo:hi].copy_(o, non_blocking=True)
        done = []
        for slot, st in enumerate(self.streams):
            with torch.cuda.stream(st):
                host_counts[slot].copy_(counts[slot], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(st)
                done.append(ev)
        counts.record_stream(cur)
        for st in self.streams:
            counts.record_stream(st)
        return MultiOpPipeline.Pending(done, host_counts, counts)

    def run(self, fmt, inputs: dict, outputs: list):
        """``run_async`` and wait: the event counts per op (numpy int64[ops, 8])."""
        return self.run_async(fmt, inputs, outputs).result()


class PluginStager:
    """The ``Device.run`` contract (int64 NumPy codes in, int64 codes and
    boolean event masks out) for large equal-shape elementwise calls.

    The element range runs in chunks through ``slots`` staging slots, each a
    set of pinned host buffers and device buffers allocated once and reused
    by every call.  Per chunk the host narrows the int64 operands into the
    slot's pinned int16 buffers (torch's threaded casting copy); the slot's
    stream copies them in, runs the kernel, splits the event byte into one
    bool mask per event, and copies the int16 result and the masks back; the
    host then widens the result into the caller's int64 output and copies
    the masks into its boolean arrays.  With three slots the host's narrowing of one
    chunk and widening of another overlap the GPU's work on a third.  Status
    counts accumulate per slot on the device and are read once per call.
    One call at a time per stager (a lock)."""

    MAX_EVENTS = 2                  # events an op reports (fma: overflow, underflow)

    def __init__(self, dev, chunk: int = 1 << 23, slots: int = 4):
        import threading
        import torch
        self.dev = dev
        self.chunk = chunk
        d = dev.torch_device
        E = self.MAX_EVENTS
        self.streams = [torch.cuda.Stream(device=d) for _ in range(slots)]
        self.done = [torch.cuda.Event() for _ in range(slots)]
        self.h_in = [[torch.empty(chunk, dtype=torch.int16, pin_memory=True) for _ in range(3)]
                     for _ in range(slots)]
        self.h_out = [torch.empty(chunk, dtype=torch.int16, pin_memory=True) for _ in range(slots)]
        self.h_mask = [torch.empty(E, chunk, dtype=torch.bool, pin_memory=True) for _ in range(slots)]
        self.d_in = [[torch.empty(chunk, dtype=torch.int16, device=d) for _ in range(3)] for _ in range(slots)]
        self.d_out = [torch.empty(chunk, dtype=torch.int16, device=d) for _ in range(slots)]
        self.d_fl = [torch.empty(chunk, dtype=torch.uint8, device=d) for _ in range(slots)]
        self.d_mask = [torch.empty(E, chunk, dtype=torch.bool, device=d) for _ in range(slots)]
        self.d_tmp = [torch.empty(chunk, dtype=torch.uint8, device=d) for _ in range(slots)]
        self.counts = torch.zeros(slots, _lib.N_COUNTS, dtype=torch.int64, device=d)
        self.lock = threading.Lock()

    def run(self, op, bits, operands, events, event_bits, pow_n: int = 0):
        """``operands``: C-contiguous int64 arrays of one shape.  Returns
        (int64 codes, {event: bool mask}, counts int64[8]) of that shape."""
        import warnings
        import torch
        shape = operands[0].shape
        n = operands[0].size
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")                # read-only caller arrays: only read here
            flat = [torch.from_numpy(o.reshape(-1)) for o in operands]
        codes = np.empty(n, dtype=np.int64)
        masks = {e: np.empty(n, dtype=bool) for e in events}
        t_codes = torch.from_numpy(codes)
        t_masks = {e: torch.from_numpy(m) for e, m in masks.items()}
        nslot = len(self.streams)
        with self.lock:
            self.counts.zero_()
            cur = torch.cuda.current_stream(self.dev.torch_device)
            for st in self.streams:
                st.wait_stream(cur)
            pending = []

            evs = list(t_masks)
            if len(evs) > self.MAX_EVENTS:
                raise ValueError(f"{op} reports {len(evs)} events; the stager carries {self.MAX_EVENTS}")

            def finish(item):
                slot, lo, hi = item
                m = hi - lo
                self.done[slot].synchronize()
                t_codes[lo:hi].copy_(self.h_out[slot][:m])                 # int16 -> int64
                for i, e in enumerate(evs):
                    t_masks[e][lo:hi].copy_(self.h_mask[slot][i, :m])       # bool bytes, a plain copy

            try:
                for k, lo in enumerate(range(0, n, self.chunk)):
                    hi = min(n, lo + self.chunk)
                    m = hi - lo
                    slot = k % nslot
                    if len(pending) == nslot:
                        finish(pending.pop(0))                              # frees this slot
                    hin = self.h_in[slot]
                    for i, src in enumerate(flat):
                        hin[i][:m].copy_(src[lo:hi])                        # int64 -> int16
                    st = self.streams[slot]
                    with torch.cuda.stream(st):
                        din = self.d_in[slot]
                        for i in range(len(flat)):
                            din[i][:m].copy_(hin[i][:m], non_blocking=True)
                        b = din[1][:m] if len(flat) > 1 else None
                        c = din[2][:m] if len(flat) > 2 else None
                        _lib.elementwise(op, bits, din[0][:m], b, c, self.d_out[slot][:m], self.d_fl[slot][:m],
                                         self.counts[slot], pow_n=pow_n, stream=st)
                        self.h_out[slot][:m].copy_(self.d_out[slot][:m], non_blocking=True)
                        # each event's mask as bool bytes, split from the event byte on the device
                        for i, e in enumerate(evs):
                            tmp = self.d_tmp[slot][:m]
                            torch.bitwise_and(self.d_fl[slot][:m], event_bits[e], out=tmp)
                            torch.ne(tmp, 0, out=self.d_mask[slot][i, :m])
                        for i in range(len(evs)):
                            self.h_mask[slot][i, :m].copy_(self.d_mask[slot][i, :m], non_blocking=True)
                        self.done[slot].record(st)
                    pending.append((slot, lo, hi))
                while pending:
                    finish(pending.pop(0))
            except BaseException:
                # copies of this call may still read the pinned slots: let them
                # finish before the next call refills them
                for st in self.streams:
                    st.synchronize()
                raise
            for st in self.streams:
                cur.wait_stream(st)
            res = self.counts.sum(0).cpu().numpy()
        _lib.check_counts(res)
        return codes.reshape(shape), {e: mk.reshape(shape) for e, mk in masks.items()}, res
