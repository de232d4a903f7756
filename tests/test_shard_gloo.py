"""Multi-rank host logic on CPU: world_size 2 over gloo, each rank computing
its row block with the oracle; gathered results equal the single-process
ones (matmul rows, sweep rows, event counts, max of times)."""
import os
import socket

import numpy as np


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from oracle import sfref
        from superfloat.python_b200 import _shard
        rng = np.random.default_rng(7)
        A = rng.integers(-32767, 32768, (2, 37, 23))
        B = rng.integers(-32767, 32768, (2, 23, 11))

        def compute(Ab, Bb):
            k, ev = sfref.matmul_chain(16, Ab.numpy(), Bb.numpy())
            fl = ev["overflow"].astype(np.uint8) | (ev["underflow"].astype(np.uint8) << 1)
            cnt = torch.tensor([int(ev["overflow"].sum()), int(ev["underflow"].sum())], dtype=torch.int64)
            return torch.from_numpy(k), torch.from_numpy(fl), cnt

        lo16, hi16 = _shard.block(9, world, rank)
        c16 = (torch.arange(lo16, hi16, dtype=torch.int16)[:, None] * 1000 - 4000).repeat(1, 3)
        g16 = _shard.gather_rows(c16, _shard.row_cuts(9, world), dist, world)
        codes, flags, cnt = _shard.sharded_matmul(compute, torch.from_numpy(A), torch.from_numpy(B), rank, world,
                                                  dist)
        t = _shard.max_over_ranks(1.5 + rank, "cpu", dist, world)
        lo, hi = _shard.block(255, world, rank, start=-127)
        rows = torch.arange(lo, hi, dtype=torch.int64)[:, None].repeat(1, 2)
        allrows = _shard.gather_rows(rows, _shard.row_cuts(255, world, -127), dist, world)
        # block-cyclic pieces gathered one at a time land in global row order
        full = torch.empty(24, 3, dtype=torch.int16)
        pieces = _shard.cyclic_pieces(24, world, 3, rank)
        works = [_shard.gather_piece(full, torch.arange(lo, hi, dtype=torch.int16)[:, None].repeat(1, 3), j, dist,
                                     world, async_op=True) for j, (lo, hi) in enumerate(pieces)]
        for w in works:
            w.wait()
        if rank == 0:
            np.save(out, {"g16": g16.numpy(), "codes": codes.numpy(), "flags": flags.numpy(), "cnt": cnt.numpy(), "t": t,
                          "rows": allrows.numpy(), "cyclic": full.numpy()}, allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_sharded_matmul_and_gathers_over_gloo(tmp_path):
    import torch.multiprocessing as mp
    from oracle import sfref
    out = str(tmp_path / "r.npy")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    r = np.load(out, allow_pickle=True).item()
    rng = np.random.default_rng(7)
    A = rng.integers(-32767, 32768, (2, 37, 23))
    B = rng.integers(-32767, 32768, (2, 23, 11))
    k, ev = sfref.matmul_chain(16, A, B)
    np.testing.assert_array_equal(r["codes"], k)
    np.testing.assert_array_equal(r["flags"], ev["overflow"].astype(np.uint8) | (ev["underflow"].astype(np.uint8) << 1))
    assert r["cnt"].tolist() == [int(ev["overflow"].sum()), int(ev["underflow"].sum())]
    assert r["t"] == 2.5
    np.testing.assert_array_equal(r["rows"][:, 0], np.arange(-127, 128))
    assert r["g16"].dtype == np.int16
    np.testing.assert_array_equal(r["g16"], (np.arange(9)[:, None] * 1000 - 4000).repeat(3, 1))
    np.testing.assert_array_equal(r["cyclic"], np.arange(24)[:, None].repeat(3, 1))


def test_row_cuts_cover_every_row():
    from superfloat.python_b200 import _shard
    for n in (0, 1, 7, 65535):
        for world in (1, 2, 3, 8):
            c = _shard.row_cuts(n, world, -5)
            assert c[0] == -5 and c[-1] == n - 5 and all(b >= a for a, b in zip(c, c[1:]))
            assert max(b - a for a, b in zip(c, c[1:])) - min(b - a for a, b in zip(c, c[1:])) <= 1
