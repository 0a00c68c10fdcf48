"""Peer-memory exchange of layer eigendecompositions between two GPUs (mpq_b200.exchange): two processes, one
per GPU, NCCL process group; skipped with fewer than two visible GPUs."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _eig_of(k, n, dev):
    g = torch.Generator().manual_seed(2000 + k)
    return torch.rand(n, generator=g).to(dev), torch.randn(n, n, generator=g).to(dev), 1e-6 * (k + 1)


def _worker(rank, world, port, n, layers, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from mpq_b200.exchange import EigenExchange
        from mpq_b200.pipeline import SetupPipeline
        x = EigenExchange(n, dev, timeout_s=60.0)
        got = {}
        with SetupPipeline(dev) as pipe:
            def setup(k):
                e = _eig_of(k, n, dev)
                x.publish(k, e)
                return e
            for k in range(rank, layers, world):
                pipe.submit(k, setup, k)
            for k in range(layers):
                if k % world == rank:
                    pipe.get(k)
                    continue
                lam, V, floor = x.fetch(k)
                got[k] = (lam.cpu().clone(), V.cpu().clone(), floor)
        x.close()
        torch.save(got, os.path.join(outdir, f"g{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_eigen_exchange_over_peer_memory(tmp_path):
    n, world, layers = 64, 2, 9
    mp.spawn(_worker, args=(world, _free_port(), n, layers, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        got = torch.load(tmp_path / f"g{r}.pt")
        assert sorted(got) == [k for k in range(layers) if k % world != r]
        for k, (lam, V, floor) in got.items():
            lw, Vw, fw = _eig_of(k, n, "cpu")
            assert torch.equal(lam, lw) and torch.equal(V, Vw)
            assert abs(floor - fw) <= 1e-12
