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


def _e8_layer(m, n, seed):
    from oracle import layer as OL
    W, H = _layer(m, n, seed)
    g = torch.Generator().manual_seed(seed + 1)
    SV = (torch.randint(0, 2, (n,), generator=g) * 2 - 1).numpy().astype(np.float32)
    SU = (torch.randint(0, 2, (m,), generator=g) * 2 - 1).numpy().astype(np.float32)
    Hr = OL.right_block_hadamard(np.ascontiguousarray(H.numpy().T), SV, n).T.copy()
    Hr = OL.right_block_hadamard(Hr, SV, n)
    Wr = OL.right_block_hadamard(W.numpy(), SV, n)
    Wr = OL.right_block_hadamard(np.ascontiguousarray(Wr.T), SU, m).T.copy()
    Wn = (Wr / np.sqrt((Wr.astype(np.float64) ** 2).mean())).astype(np.float32)
    return Wn, Hr.astype(np.float32)


def _e8_shard_worker(rank, world, port, m, n, block_rows, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=300))
    try:
        from oracle import e8p12 as OE
        Wn, Hr = _e8_layer(m, n, 11)
        r0, r1 = row_shards(m, world, block_rows)[rank]
        out = OE.refine_codebook(Wr=Wn[r0:r1], Hr=Hr, cb=OE.E8P12_codebook(),
                                 cfg=OE.E8P12VampConfig(iters=8, prior_tau=0.25, polish_sweeps=2),
                                 block_rows=block_rows)
        hat = gather_rows(torch.from_numpy(np.ascontiguousarray(out["hatWr"])), row_shards(m, world, block_rows))
        torch.save(hat, os.path.join(outdir, f"hat{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_e8p12_restart_per_shard_matches_the_serial_chain_on_proxy_loss(tmp_path):
    """Row sharding over N ranks restarts the obs-precision chain in every shard (each shard's first block starts
    from its own RTN warm start) instead of carrying it from the previous shard's last block.  The layer's proxy
    loss tr((W - Q) H (W - Q)^T) of the sharded solve must stay within 0.5 % of the serial chain's."""
    from oracle import e8p12 as OE
    from oracle import layer as OL
    m, n, br, world = 64, 256, 16, 2
    mp.spawn(_e8_shard_worker, args=(world, _free_port(), m, n, br, str(tmp_path)), nprocs=world, join=True)
    Wn, Hr = _e8_layer(m, n, 11)
    serial = OE.refine_codebook(Wr=Wn, Hr=Hr, cb=OE.E8P12_codebook(),
                                cfg=OE.E8P12VampConfig(iters=8, prior_tau=0.25, polish_sweeps=2), block_rows=br)
    want = OL.proxy_loss(Wn, serial["hatWr"], Hr)
    hats = [torch.load(tmp_path / f"hat{r}.pt").numpy() for r in range(world)]
    np.testing.assert_array_equal(hats[0], hats[1])
    got = OL.proxy_loss(Wn, hats[0], Hr)
    print(f"proxy loss: sharded {got:.4f}, serial chain {want:.4f} ({(got - want) / want:+.2e})")
    assert abs(got - want) <= 0.005 * want, (got, want)


def _store_exchange(n, slots):
    """EigenExchange's protocol (ownership, slots, ready keys, acknowledgements) over a host transport: the slot
    contents travel through the key-value store instead of peer memory (there is no GPU here)."""
    from mpq_b200.exchange import EigenExchange

    class X(EigenExchange):
        def _open_transport(self):
            self._ptr = 1
            self.writes = []

        def _write_slot(self, slot, eig):
            lam, V, floor = eig
            buf = torch.cat([lam, V.reshape(-1), torch.tensor([floor], dtype=torch.float32)])
            self.writes.append(slot)
            self._set(f"{self.prefix}/slot/{self.rank}/{slot}", buf.numpy().tobytes())

        def _read_slot(self, owner, slot):
            raw = self._get(f"{self.prefix}/slot/{owner}/{slot}")
            self.recv.copy_(torch.from_numpy(np.frombuffer(raw, dtype=np.float32).copy()))

        def _close_transport(self):
            dist.barrier()
            self._ptr = 0

    return X(n, torch.device("cpu"), slots=slots, timeout_s=60.0)


def _xchg_worker(rank, world, port, n, layers, outdir):
    import threading
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        x = _store_exchange(n, slots=2)

        def eig_of(k):
            g = torch.Generator().manual_seed(1000 + k)
            return torch.rand(n, generator=g), torch.randn(n, n, generator=g), 1e-6 * (k + 1)

        # the owner publishes from its own thread, ahead of the readers, as the set-up pipeline does
        errors = []

        def publisher():
            try:
                for k in range(rank, layers, world):
                    x.publish(k, eig_of(k))
            except Exception as e:  # surfaced by the main thread
                errors.append(e)

        th = threading.Thread(target=publisher)
        th.start()
        got = {}
        for k in range(layers):
            if k % world == rank:
                continue
            lam, V, floor = x.fetch(k)
            got[k] = (lam.clone(), V.clone(), floor)
        th.join()
        if errors:
            raise errors[0]
        x.close()
        torch.save({"got": got, "writes": x.writes}, os.path.join(outdir, f"x{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_eigen_exchange_protocol_round_robin(tmp_path):
    """Every reader receives every layer it does not own, bit for bit, while owners reuse two slots per rank (a
    slot is rewritten only after the layer in it was acknowledged by every reader)."""
    n, world, layers = 8, 3, 13
    mp.spawn(_xchg_worker, args=(world, _free_port(), n, layers, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        out = torch.load(tmp_path / f"x{r}.pt")
        assert sorted(out["got"]) == [k for k in range(layers) if k % world != r]
        for k, (lam, V, floor) in out["got"].items():
            g = torch.Generator().manual_seed(1000 + k)
            assert torch.equal(lam, torch.rand(n, generator=g))
            assert torch.equal(V, torch.randn(n, n, generator=g))
            assert abs(floor - 1e-6 * (k + 1)) <= 1e-12
        assert out["writes"] == [(k // world) % 2 for k in range(r, layers, world)]
