"""The row-block partition of a GEMM over GPUs with the gather fused into the GEMM kernels.

Rank r's epilogue stores its rows straight into the root's [M, N] buffer (over NVLink when the
root is another GPU). A rank's block is the same product, with the same kernel schedule, as the
single-GPU GEMM of that block, so the gathered C must equal those products stacked, bit for bit;
against the GEMM of the whole matrix (a different schedule: the stream-K tail may split other
tiles) it agrees within the 3xTF32 bound. On a one-GPU box the ranks share cuda:0 (the row
offsets, the per-rank descriptors and the ordering are still exercised); the cross-GPU cases run
where the box has two GPUs.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from mensurflow_b200 import sharded

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu


def _operands(m, n, k, device, seed=3):
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(device)
    b = torch.randn(n, k, generator=g).to(device)
    c = torch.randn(m, n, generator=g).to(device)
    bias = (torch.rand(n, generator=g) - 0.5).to(device)
    return a, b, c, bias


@pytest.mark.parametrize("precision", ["3xtf32", "1xtf32"])
def test_row_blocks_gathered_on_one_gpu_equal_the_single_product(cuda, precision):
    m, n, k = 757, 520, 300
    a, b, c, bias = _operands(m, n, k, cuda)
    bounds = [0, 300, 557, m]  # uneven blocks, one not a multiple of the 256-row tile
    blocks = [a[bounds[i]:bounds[i + 1]] for i in range(3)]
    cb = [c[bounds[i]:bounds[i + 1]] for i in range(3)]
    want = torch.cat([mf.gemm(blocks[i], b, 0.5, cb[i], 1.0, False, True, bias=bias,
                              activation="gelu", precision=precision) for i in range(3)], 0)
    whole = mf.gemm(a, b, 0.5, c, 1.0, False, True, bias=bias, activation="gelu",
                    precision=precision)
    for gather in (True, False):
        got = sharded.gemm_row_blocks(blocks, [b] * 3, 0.5, cb, 1.0, True, bias=[bias] * 3,
                                      activation="gelu", precision=precision, gather=gather)
        torch.cuda.synchronize()
        if not gather:
            got = torch.cat(got, 0)
        assert got.shape == (m, n)
        assert torch.equal(got, want), f"gather={gather}"
    rel = 1e-5 if precision == "3xtf32" else 2e-3
    mag = 0.5 * (a.abs() @ b.abs().t()) + c.abs() + bias.abs()
    assert bool(((got - whole).abs() <= rel * 1.2 * mag + 1e-6).all())
    assert mf.device_status() == 0


@pytest.mark.parametrize("precision", ["3xtf32", "1xtf32"])
def test_declared_peer_output_equals_the_tma_store_path(cuda, precision):
    """mfk_gemm_peer_f32 (C declared another GPU's memory: plain 128-byte row stores and a
    system-scope fence, never a tensor map) writes the same bits as mfk_gemm_f32 (TMA stores) —
    only the store path differs. On one GPU the "peer" buffer is local memory, where the
    declared path is valid too; rows and columns not multiples of the tile, and a row stride
    wider than N, check the edges."""
    m, n, k = 333, 300, 257
    a, b, c, bias = _operands(m, n, k, cuda, seed=11)
    want = mf.gemm(a, b, 0.5, c, 1.0, False, True, bias=bias, activation="relu",
                   precision=precision)
    ld = n + 12
    buf = torch.full((m, ld), float("nan"), device=cuda)
    sharded.gemm_into_peer(a, b, 0.5, c, 1.0, True, buf.data_ptr(), ld, bias=bias,
                           activation="relu", precision=precision, peer_memory=True)
    torch.cuda.synchronize()
    assert torch.equal(buf[:, :n], want)
    assert bool(torch.isnan(buf[:, n:]).all()), "the declared path wrote past N"
    assert mf.device_status() == 0


def test_row_blocks_argument_errors(cuda):
    a = torch.zeros(4, 8, device=cuda)
    with pytest.raises(ValueError):
        sharded.gemm_row_blocks([a, a], [torch.zeros(8, 5, device=cuda)])
    with pytest.raises(ValueError):
        sharded.gemm_row_blocks([a], [torch.zeros(7, 5, device=cuda)])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("root", [0, 1])
def test_row_blocks_gathered_across_two_gpus(cuda, root):
    """Rank 1 (or 0) writes its rows into the other GPU's buffer over NVLink."""
    m, n, k = 1024, 768, 512
    a, b, c, bias = _operands(m, n, k, cuda, seed=9)
    want = torch.cat([mf.gemm(a[:600], b, 1.0, c[:600], 0.5, False, True, bias=bias),
                      mf.gemm(a[600:], b, 1.0, c[600:], 0.5, False, True, bias=bias)], 0).cpu()
    d1 = torch.device("cuda", 1)
    blocks = [a[:600], a[600:].to(d1)]
    reps = [b, b.to(d1)]
    cb = [c[:600], c[600:].to(d1)]
    biases = [bias, bias.to(d1)]
    got = sharded.gemm_row_blocks(blocks, reps, 1.0, cb, 0.5, True, bias=biases, root=root)
    assert got.device == blocks[root].device
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    assert torch.equal(got.cpu(), want)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _peer_worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import mensurflow_b200 as mf
        from mensurflow_b200 import sharded

        m, n, k = 1000, 640, 384
        a, b, c, bias = _operands(m, n, k, dev, seed=21)
        start, stop = sharded.block_range(m, world, rank)
        peer = sharded.PeerRowGather(m, n, dev, root=0)
        ok = True
        for step in range(2):  # the mapped buffer is reused across steps
            alpha = 0.5 + step
            full = sharded.sharded_gemm(a[start:stop], b, m, alpha, c[start:stop], 1.0, True,
                                        bias=bias, gather="peer", peer=peer)
            if rank == 0:
                want = torch.cat([mf.gemm(a[s0:s1], b, alpha, c[s0:s1], 1.0, False, True,
                                          bias=bias)
                                  for s0, s1 in (sharded.block_range(m, world, r)
                                                 for r in range(world))], 0)
                ok = ok and torch.equal(full, want)
            else:
                ok = ok and full is None
        peer.close()
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_gather_one_process_per_gpu(cuda):
    """Two processes (NCCL for the handle exchange and the step barrier only): rank 1's GEMM
    writes into rank 0's buffer through a CUDA IPC mapping; rank 0 then holds the full C."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = dict(q.get(timeout=5) for _ in procs)
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}
