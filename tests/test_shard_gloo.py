"""Row-sharded layer solve plumbing (mpq_b200.shard) on CPU: world-size-2 gloo process groups.

Each rank solves its shard of a small layer with the CPU oracle's scalar layer driver (the stand-in for
the GPU solve, which needs no change to shard), and the gathered layer must equal the shards solved one
after another in a single process.  No GPU is used."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mpq_b200.shard import gather_rows, row_shards, solve_layer_sharded


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(m, n, seed):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(m, n, generator=g) * 0.02
    X = torch.randn(4 * n, n, generator=g) * torch.exp(torch.randn(n, generator=g)).sqrt()
    H = X.T @ X / X.shape[0]
    H += torch.eye(n) * 0.01 * H.diagonal().mean()
    return W, H


def _solve_rows(W_rows, H):
    from oracle import layer as OL
    from oracle.uniform_vamp import UniformVampConfig
    if W_rows.shape[0] == 0:
        return [torch.empty(0, W_rows.shape[1], dtype=torch.uint8), torch.empty(0, W_rows.shape[1])]
    cfg = UniformVampConfig(iters=4, prior_tau=0.2, damping=0.5, polish_sweeps=1)
    out = OL.run_scalar_layer(W=W_rows.numpy(), H=H.numpy(), bits=4, group_size=32, vamp_cfg=cfg,
                              block_rows=W_rows.shape[0], module_name="shard.test")
    return [torch.from_numpy(out["q_int"]), torch.from_numpy(out["Q"])]


def _worker(rank, world, port, m, n, align, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        if rank == 0:
            W, H = _layer(m, n, 7)
        else:  # the other ranks receive W and H by broadcast
            W, H = torch.empty(m, n), torch.empty(n, n)
        q, Q = solve_layer_sharded(W, H, _solve_rows, align=align)
        torch.save({"q": q, "Q": Q}, os.path.join(outdir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_row_shards_cover_rows_in_order():
    for m, world, align in [(4096, 8, 1), (4096, 3, 128), (10, 2, 4), (3, 4, 1), (0, 2, 1), (129, 2, 128)]:
        sh = row_shards(m, world, align)
        assert len(sh) == world
        assert sh[0][0] == 0 and sh[-1][1] == m
        for (a, b), (c, d) in zip(sh, sh[1:]):
            assert b == c and a <= b
        assert all((b - a) % align == 0 for a, b in sh[:-1])
    assert row_shards(10, 2, 4) == [(0, 8), (8, 10)]
    assert row_shards(3, 4, 1) == [(0, 1), (1, 2), (2, 3), (3, 3)]
    with pytest.raises(ValueError):
        row_shards(8, 0, 1)


def test_gather_rows_single_process_is_identity():
    t = torch.arange(12).reshape(4, 3)
    assert gather_rows(t, [(0, 4)]) is t


@pytest.mark.parametrize("m,align", [(12, 1), (10, 4)])
def test_sharded_solve_matches_per_shard_solves(tmp_path, m, align):
    n, world = 64, 2
    mp.spawn(_worker, args=(world, _free_port(), m, n, align, str(tmp_path)), nprocs=world, join=True)
    W, H = _layer(m, n, 7)
    want_q, want_Q = [], []
    for a, b in row_shards(m, world, align):
        q, Q = _solve_rows(W[a:b].contiguous(), H)
        want_q.append(q)
        want_Q.append(Q)
    want_q, want_Q = torch.cat(want_q), torch.cat(want_Q)
    for rank in range(world):
        got = torch.load(tmp_path / f"rank{rank}.pt")
        assert got["q"].dtype == torch.uint8 and got["q"].shape == (m, n)
        assert torch.equal(got["q"], want_q)
        assert torch.equal(got["Q"], want_Q)
    assert np.isfinite(want_Q.numpy()).all()
