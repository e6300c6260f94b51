"""Token-axis sharding on two or more GPUs (NCCL process group, one process per
GPU): the peer-memory dw exchange (``sy_dw_exchange``) against the collective
fallback and the float64 oracle.

Each rank holds its contiguous token range of the same inputs; after forward +
backward every rank must hold the bitwise-same ``dw`` (and, for the batched
training op with four queries, the same ``dq``), equal bitwise between the
peer-memory path and the all-gather path (both add the ranks in rank order),
stable over repeated steps (the exchange alternates its two slots), and within
the bf16 rounding floor of the oracle's full-batch gradient. Skipped with fewer
than two GPUs.
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
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
N, B, T, D = 9, 1, 512, 2048


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    for p in (ROOT / "blackwell-switchyard_b200", ROOT):
        sys.path.insert(0, str(p))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        from switchyard import _native, sharding
        from switchyard.sharding import (
            block_attn_res_batched_sharded,
            block_attn_res_sharded,
            token_range,
        )

        g = torch.Generator().manual_seed(11)
        v = torch.randn(N, B, T, D, generator=g).to(torch.bfloat16)
        w = (torch.randn(D, generator=g) / D**0.5).to(torch.bfloat16)
        dout = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
        lo, hi = token_range(B * T, world, rank)
        v_loc = v.reshape(N, B * T, D)[:, lo:hi].reshape(N, 1, hi - lo, D).to(dev)
        g_loc = dout.reshape(B * T, D)[lo:hi].reshape(1, hi - lo, D).to(dev)
        w_dev = w.to(dev)

        def step():
            vv = v_loc.detach().requires_grad_(True)
            ww = w_dev.detach().requires_grad_(True)
            block_attn_res_sharded(vv, ww, 1e-6).backward(g_loc)
            return vv.grad, ww.grad

        dws = []
        for _ in range(3):  # three steps: both slots, then the first again
            dv, dw = step()
            dws.append(dw.clone())
        # the batched training op on the same shard: S = 4 queries
        qs = (torch.randn(4, D, generator=g) / D**0.5).to(torch.bfloat16)
        gq = torch.randn(4, B, T, D, generator=g).to(torch.bfloat16)
        gq_loc = gq.reshape(4, B * T, D)[:, lo:hi].reshape(4, 1, hi - lo, D).to(dev)
        q_dev = qs.to(dev)

        def bstep():
            vv = v_loc.detach().requires_grad_(True)
            qq = q_dev.detach().requires_grad_(True)
            block_attn_res_batched_sharded(vv, qq, 1e-6).backward(gq_loc)
            return qq.grad

        dqs = [bstep().clone() for _ in range(2)]
        peer_used = bool(sharding._PEER)
        os.environ["SWITCHYARD_DW_EXCHANGE"] = "collective"
        dqs.append(bstep().clone())
        np.save(Path(outdir) / f"dq{rank}.npy", torch.stack(dqs).float().cpu().numpy())
        _, dw_coll = step()
        torch.cuda.synchronize()
        assert _native.device_error() == 0
        np.save(Path(outdir) / f"dw{rank}.npy", torch.stack(dws + [dw_coll]).float().cpu().numpy())
        np.save(Path(outdir) / f"peer{rank}.npy", np.array([peer_used]))
        dist.barrier()
    finally:
        sharding._PEER.clear()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_dw_exchange_matches_collective_and_oracle(world, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            p.join()
    assert [p.exitcode for p in procs] == [0] * world

    got = [np.load(tmp_path / f"dw{r}.npy") for r in range(world)]
    assert all(bool(np.load(tmp_path / f"peer{r}.npy")[0]) for r in range(world))
    for r in range(world):
        for k in range(1, 4):  # steps agree, and the collective path gives the same bits
            assert np.array_equal(got[r][0], got[r][k])
        assert np.array_equal(got[0][0], got[r][0])  # every rank the same

    sys.path.insert(0, str(ROOT))
    from oracle import attnres_oracle as O

    g = torch.Generator().manual_seed(11)
    v = torch.randn(N, B, T, D, generator=g).to(torch.bfloat16)
    w = (torch.randn(D, generator=g) / D**0.5).to(torch.bfloat16)
    dout = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    f64 = lambda t: t.to(torch.float64).numpy()  # noqa: E731
    _, dw_o = O.backward(f64(v), f64(w), f64(dout))
    assert O.rel_l2(got[0][0], dw_o) <= 1.005 * O.dtype_floor(dw_o, "bfloat16")

    # batched: dq the same on every rank, peer and collective paths bitwise
    # equal, and at the bf16 floor of the oracle's full-batch gradient
    dq = [np.load(tmp_path / f"dq{r}.npy") for r in range(world)]
    for r in range(world):
        assert np.array_equal(dq[r][0], dq[r][1]) and np.array_equal(dq[r][0], dq[r][2])
        assert np.array_equal(dq[0][0], dq[r][0])
    qs = (torch.randn(4, D, generator=g) / D**0.5).to(torch.bfloat16)
    gq = torch.randn(4, B, T, D, generator=g).to(torch.bfloat16)
    _, dq_o = O.batched_backward(f64(v), f64(qs), f64(gq))
    assert O.rel_l2(dq[0][0], dq_o) <= 1.005 * O.dtype_floor(dq_o, "bfloat16")
