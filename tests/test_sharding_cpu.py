"""Token-axis sharding on CPU ranks (gloo, world_size 2 and 3).

Runs the host logic of ``switchyard.sharding`` -- the contiguous token
partition and the fixed-order dw exchange -- across real ``torch.distributed``
processes. The per-rank dw partial comes from the oracle (this is a CPU test:
no kernel runs), so what is checked is the plumbing: the partition covers
every token exactly once, every rank ends with the bitwise-same dw, and that
dw equals the oracle's full-batch gradient. A rank that fails makes the others
fail within the process-group timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
N, B, T, D = 5, 2, 13, 24


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(7)
    v = rng.standard_normal((N, B, T, D))
    w = rng.standard_normal(D) / np.sqrt(D)
    g = rng.standard_normal((B, T, D))
    return v, w, g


def _worker(rank, world, port, outdir, fail_rank):
    for p in (ROOT / "blackwell-switchyard_b200", ROOT):
        sys.path.insert(0, str(p))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        from oracle import attnres_oracle as O
        from switchyard.sharding import exchange_dw, token_range

        if rank == fail_rank:
            raise RuntimeError("injected failure on this rank")
        v, w, g = _inputs()
        bt = B * T
        lo, hi = token_range(bt, world, rank)
        vf = v.reshape(N, bt, D)[:, lo:hi]
        gf = g.reshape(bt, D)[lo:hi]
        _, dw_local = O.backward(vf[:, None], w, gf[None])
        total = exchange_dw(torch.from_numpy(dw_local).float(), None)
        np.save(Path(outdir) / f"rank{rank}.npy", total.numpy())
        np.save(Path(outdir) / f"range{rank}.npy", np.array([lo, hi]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(world, tmp_path, fail_rank=-1):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            p.join()
    return [p.exitcode for p in procs]


def test_token_range_partitions_the_axis():
    from switchyard.sharding import token_range

    for bt in (0, 1, 7, 26, 4096, 4097):
        for world in (1, 2, 3, 8):
            ranges = [token_range(bt, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == bt
            for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        token_range(10, 0, 0)


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_dw_exchange_matches_full_batch(world, tmp_path):
    codes = _run(world, tmp_path)
    assert codes == [0] * world
    from oracle import attnres_oracle as O

    v, w, g = _inputs()
    _, dw_full = O.backward(v, w, g)
    got = [np.load(tmp_path / f"rank{r}.npy") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(got[0], got[r]), "ranks disagree on dw"
    np.testing.assert_allclose(got[0], dw_full, rtol=2e-5, atol=2e-6)
    covered = sorted(tuple(np.load(tmp_path / f"range{r}.npy")) for r in range(world))
    assert covered[0][0] == 0 and covered[-1][1] == B * T


def test_a_failing_rank_does_not_hang_the_others(tmp_path):
    codes = _run(2, tmp_path, fail_rank=1)
    assert codes[1] != 0
    assert codes[0] != 0  # its collective fails (peer gone / timeout) instead of hanging
