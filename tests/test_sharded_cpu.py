"""Multi-rank host logic of the sharded GEMM on CPU: world_size 2 with the gloo backend, each
rank computing its row block with the oracle (the CPU stand-in for the per-GPU kernel); the
gathered result must equal the single-process product bit for bit."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_gemm(a, b, alpha, c, beta, transpose_a, transpose_b, bias=None, activation=None):
    from oracle import oracle as O

    out = O.gemm(a.numpy(), b.numpy(), alpha, None if c is None else c.numpy(), beta,
                 transpose_a, transpose_b, bias=None if bias is None else bias.numpy(),
                 act=activation)
    return torch.from_numpy(out)


def oracle_batched(a, b, alpha, c, beta, transpose_a, transpose_b):
    from oracle import oracle as O

    outs = [O.gemm(a[i].numpy(), b[i].numpy(), alpha, None, 0.0, transpose_a, transpose_b)
            for i in range(a.shape[0])]
    return torch.from_numpy(np.stack(outs)) if outs else torch.empty(0)


def _worker(rank, world, port, m, n, k, q):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mensurflow_b200 import sharded

        g = torch.Generator().manual_seed(7)
        a = torch.randn(m, k, generator=g)
        b = torch.randn(n, k, generator=g)
        c = torch.randn(m, n, generator=g)
        bias = torch.rand(n, generator=g) - 0.5
        a_local = sharded.local_rows(a, world, rank)
        c_local = sharded.local_rows(c, world, rank)
        full = sharded.sharded_gemm(a_local, b, m, 0.5, c_local, 1.0, True, bias=bias,
                                    gather=True, gemm_fn=oracle_gemm)
        want = oracle_gemm(a, b, 0.5, c, 1.0, False, True, bias=bias)
        ok2d = torch.equal(full, want)
        qb = torch.randn(5, 6, 7, generator=g)
        kb = torch.randn(5, 8, 7, generator=g)
        outb = sharded.sharded_gemm_batched(sharded.local_rows(qb, world, rank),
                                            sharded.local_rows(kb, world, rank), 5, 0.25, True,
                                            gather=True, gemm_fn=oracle_batched)
        okb = torch.equal(outb, oracle_batched(qb, kb, 0.25, None, 0.0, False, True))
        q.put((rank, ok2d, okb, tuple(full.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m", [64, 67])  # even and uneven row blocks
def test_sharded_gemm_two_ranks(m):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, m, 40, 33, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = sorted(q.get(timeout=10) for _ in procs)
    for p in procs:
        assert p.exitcode == 0
    for rank, ok2d, okb, shape in results:
        assert shape == (m, 40)
        assert ok2d, f"rank {rank}: gathered row blocks differ from the whole product"
        assert okb, f"rank {rank}: gathered batch differs"


def test_block_range_covers_rows_once():
    from mensurflow_b200.sharded import block_range

    for total in (0, 1, 7, 8, 32768):
        for world in (1, 2, 3, 4, 8):
            rows = []
            for r in range(world):
                s, e = block_range(total, world, r)
                assert 0 <= s <= e <= total
                rows.extend(range(s, e))
            assert rows == list(range(total))
    with pytest.raises(ValueError):
        block_range(10, 2, 2)


def _failing_worker(rank, world, port, q):
    """Rank 1 holds the wrong number of rows: sharded_gemm rejects it on the host (ValueError)
    and the rank leaves without joining the gather. Rank 0 reaches the gather, whose peer is
    gone: the collective must end with an error within the process group's short timeout rather
    than wait for ever."""
    import datetime
    import time

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    from mensurflow_b200 import sharded

    m, n, k = 64, 16, 8
    a = torch.randn(m, k)
    b = torch.randn(n, k)
    a_local = sharded.local_rows(a, world, rank)
    if rank == 1:
        try:
            sharded.sharded_gemm(a_local[:-1], b, m, transpose_b=True, gather=True,
                                 gemm_fn=oracle_gemm)
            q.put((rank, "no error"))
        except ValueError:
            q.put((rank, "ValueError"))
        q.close()
        q.join_thread()
        os._exit(0)  # leaves without the collective
    t0 = time.time()
    try:
        sharded.sharded_gemm(a_local, b, m, transpose_b=True, gather=True, gemm_fn=oracle_gemm)
        q.put((rank, "no error"))
    except Exception as e:  # the collective's failure (timeout or closed connection)
        q.put((rank, f"error after {time.time() - t0:.1f} s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_a_rank_that_leaves_makes_the_gather_fail_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank is still waiting in the gather"
    results = dict(q.get(timeout=10) for _ in procs)
    assert results[1] == "ValueError"
    assert results[0].startswith("error after"), results[0]


class _SharedRows:
    """CPU stand-in for PeerRowGather: the root's buffer is shared memory every rank writes its
    rows into; row_ptr() hands out the row index in place of a device address."""

    def __init__(self, buffer, root, rank):
        self.rows, self.cols = buffer.shape
        self.root = root
        self.rank = rank
        self.shared = buffer
        self.buffer = buffer if rank == root else None

    def row_ptr(self, row):
        return row


def _reuse_worker(rank, world, port, buffer, q):
    sys.path.insert(0, ROOT)
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mensurflow_b200 import sharded

        peer = _SharedRows(buffer, 0, rank)

        def rows_into_shared(a, b, alpha, c, beta, transpose_b, row0, ldc, *, bias=None,
                             activation=None, precision=None, peer_memory=None):
            # the root writes its own buffer; every other rank declares the buffer peer memory
            assert peer_memory == (rank != 0)
            peer.shared[row0:row0 + a.shape[0]] = oracle_gemm(a, b, alpha, c, beta, False,
                                                              transpose_b)

        sharded.gemm_into_peer = rows_into_shared
        m, n, k = 48, 24, 16
        g = torch.Generator().manual_seed(5)
        a, b, c = torch.randn(m, k, generator=g), torch.randn(k, n, generator=g), torch.zeros(m, n)
        start, stop = sharded.block_range(m, world, rank)
        ok = True
        for step in range(3):
            full = sharded.sharded_gemm(a[start:stop], b, m, 1.0 + step, c[start:stop], 0.0,
                                        gather="peer", peer=peer)
            if rank == 0:
                time.sleep(0.5)  # a slow reader: the other rank must not start the next step
                ok = ok and torch.equal(full, oracle_gemm(a, b, 1.0 + step, None, 0.0, False,
                                                          False))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_peer_gather_buffer_not_overwritten_while_the_root_reads():
    """gather='peer' reuses the root's buffer from call to call: a rank must not write its next
    rows while the root is still reading the previous C (the barrier before the GEMMs). The
    root here reads slowly after each call; the other rank would overwrite its rows at once."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    buffer = torch.zeros(48, 24).share_memory_()
    procs = [ctx.Process(target=_reuse_worker, args=(r, 2, port, buffer, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = dict(q.get(timeout=10) for _ in procs)
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}
