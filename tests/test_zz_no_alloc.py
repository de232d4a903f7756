"""sfb_matmul_wide_noalloc: the wide matmul for callers that cannot allocate
device memory while they run (a program that gave all GPU memory to its own
pool, a plugin host that forbids allocation after start-up, a loop that cannot
take the synchronisation an allocation can imply).  Its scratch is a fixed
64 MiB array inside the library, so it must give exactly what
sfb_matmul_wide gives with a caller workspace, call after call, even though
the array keeps the previous call's contents.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.  It passes alone in a fresh
process and after the other tests."""
import ctypes

import numpy as np
import pytest

from superfloat.python_b200 import _lib

pytestmark = pytest.mark.gpu


def _call(lib, name, bits, A, B, out, flags, counts, shift, workspace=None):
    import torch
    M, K = A.shape
    N = B.shape[1]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())                        # noqa: E731
    args = [bits, 0, p(A), p(B), None, shift, p(out), p(flags), 1, M, N, K, K, N, 0, 0, M * N, 0, 0, 0]
    if name == "sfb_matmul_wide":
        args += [p(workspace), workspace.numel()]
    args += [p(counts), stream]
    return getattr(lib, name)(*args)


def test_noalloc_equals_the_workspace_entry_point_twice(gpu):
    import torch
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(2024)
    # two calls in a row, the second at a smaller, ragged shape: its padding
    # rows / columns and its scratch layout differ from the first call's, so
    # whatever the first call left in the array must not leak into it
    for call, (M, N, K) in enumerate(((1536, 1536, 1536), (1000, 1100, 900))):
        need = lib.sfb_matmul_wide_workspace(16, 0, 1, M, N, K)
        assert 0 < need <= 64 << 20                   # the tensor-core path, within the fixed scratch
        ws = torch.empty(need, dtype=torch.uint8, device=dev)      # a fresh workspace for the reference call
        A = torch.from_numpy(rng.integers(-3000 * (call + 1), 3000 * (call + 1) + 1, (M, K))).to(torch.int16).to(dev)
        B = torch.from_numpy(rng.integers(-32767, 32768, (K, N))).to(torch.int16).to(dev)
        shift = -call
        outs = []
        for name in ("sfb_matmul_wide", "sfb_matmul_wide_noalloc"):
            out = torch.empty(M, N, dtype=torch.int16, device=dev)
            flags = torch.empty(M, N, dtype=torch.uint8, device=dev)
            counts = torch.zeros(8, dtype=torch.int64, device=dev)
            rc = _call(lib, name, 16, A, B, out, flags, counts, shift, workspace=ws)
            assert rc == 0, (name, _lib.last_error())
            torch.cuda.synchronize()
            outs.append((out.cpu().numpy(), flags.cpu().numpy(), counts.cpu().numpy()))
        (o1, f1, c1), (o2, f2, c2) = outs
        np.testing.assert_array_equal(o2, o1)         # integer codes: the tolerance is exact equality
        np.testing.assert_array_equal(f2, f1)
        np.testing.assert_array_equal(c2, c1)
        assert c1[5] == 0 and c1[0] > 0               # no device error; some outputs saturate


def test_noalloc_refuses_problems_beyond_its_scratch(gpu):
    import torch
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    M = N = K = 2048
    assert lib.sfb_matmul_wide_workspace(16, 0, 1, M, N, K) > 64 << 20
    A = torch.zeros(M, K, dtype=torch.int16, device=dev)
    B = torch.zeros(K, N, dtype=torch.int16, device=dev)
    out = torch.empty(M, N, dtype=torch.int16, device=dev)
    flags = torch.empty(M, N, dtype=torch.uint8, device=dev)
    counts = torch.zeros(8, dtype=torch.int64, device=dev)
    rc = _call(lib, "sfb_matmul_wide_noalloc", 16, A, B, out, flags, counts, 0)
    assert rc == _lib.SFB_ERANGE
    assert b"more than the" in lib.sfb_last_error()
