"""Sharding of the GEMM path over GPUs.

The path has no reduction across ranks: a 2-D GEMM splits by row blocks of A and C (B and the
bias replicated), a batched GEMM by the batch index, a gemv by rows of A. Each rank computes its
own slice with the single-GPU kernels; nothing crosses NVLink on the data path unless the caller
wants C gathered on one device. Then each rank's GEMM epilogue stores its rows straight into the
root's [M, N] buffer over NVLink — the gather is part of the GEMM kernels, with no extra kernel or
collective (the blocks are contiguous rows, so the gathered buffer needs no repacking):

* one process driving several GPUs: `gemm_row_blocks` (the C ABI's mfk_sharded_gemm_f32);
* one process per GPU (torch.distributed): `PeerRowGather`, which maps the root's buffer into
  every rank through CUDA IPC handles, and `sharded_gemm(..., gather="peer")`.

`gather_rows` is the NCCL alternative (`all_gather_into_tensor`: every rank receives C), kept as
the baseline the fused gather is measured against.
"""
from __future__ import annotations

import ctypes
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


def block_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [start, stop) of `rank`: equal blocks of ceil(total / world), the last one short."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    per = -(-total // world)
    start = min(total, rank * per)
    return start, min(total, start + per)


def local_rows(x: torch.Tensor, world: int, rank: int, dim: int = 0) -> torch.Tensor:
    """This rank's block of `x` along `dim` (a view, no copy)."""
    start, stop = block_range(x.shape[dim], world, rank)
    return x.narrow(dim, start, stop - start)


def gather_rows(local: torch.Tensor, total: int, group=None) -> torch.Tensor:
    """All-gathers every rank's row block (rows of block_range) into one [total, ...] tensor.
    Blocks are padded to the common block size for the collective and trimmed after it."""
    world = dist.get_world_size(group)
    per = -(-total // world)
    if local.shape[0] < per:
        pad = torch.zeros((per - local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        send = torch.cat([local, pad], 0)
    else:
        send = local.contiguous()
    out = torch.empty((per * world,) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    dist.all_gather_into_tensor(out, send, group=group)
    return out[:total]


def gemm_row_blocks(a_blocks: Sequence[torch.Tensor], b: Sequence[torch.Tensor],
                    alpha: float = 1.0, c_blocks: Optional[Sequence[torch.Tensor]] = None,
                    beta: float = 0.0, transpose_b: bool = False, *,
                    bias: Optional[Sequence[torch.Tensor]] = None,
                    activation: Optional[str] = None, precision: Optional[str] = None,
                    gather: bool = True, root: int = 0):
    """One process, several GPUs: rank r multiplies a_blocks[r] (rows of A on its GPU) by its
    replica b[r] (and adds beta * c_blocks[r] + bias[r]). With `gather` the row blocks are written
    by the GEMM kernels straight into one [sum of rows, N] tensor on a_blocks[root]'s GPU, which
    is returned; the root's current stream is ordered after every rank. Without it the per-rank
    C blocks are returned as a list. Every rank runs on its GPU's current stream."""
    from . import _lib
    from .ops import _gemm_desc, _kernel_for

    nranks = len(a_blocks)
    if nranks == 0 or len(b) != nranks:
        raise ValueError("gemm_row_blocks: one A block and one B replica per rank")
    if c_blocks is not None and len(c_blocks) != nranks:
        raise ValueError("gemm_row_blocks: one C block per rank")
    for t in a_blocks:
        _kernel_for("gemm_row_blocks", t)
    n = b[0].shape[0] if transpose_b else b[0].shape[1]
    devices = [t.device for t in a_blocks]
    outs: List[torch.Tensor] = []
    descs = (_lib.GemmDesc * nranks)()
    m_total = 0
    for r in range(nranks):
        a, br = a_blocks[r], b[r]
        if br.device != devices[r]:
            raise ValueError(f"gemm_row_blocks: B replica {r} is not on rank {r}'s device")
        right = br.t() if transpose_b else br
        if a.shape[1] != right.shape[0] or right.shape[1] != n:
            raise ValueError("gemm_row_blocks: operand shapes differ between ranks")
        out = torch.empty((a.shape[0], n), dtype=torch.float32, device=devices[r]) \
            if not gather else torch.empty((1, n), dtype=torch.float32, device=devices[r])
        c_in = None if c_blocks is None or beta == 0.0 else c_blocks[r]
        bias_r = None if bias is None else bias[r].contiguous()
        descs[r] = _gemm_desc(a, right, out, alpha, c_in, beta if c_in is not None else 0.0,
                              bias_r, activation, precision)
        descs[r].m = a.shape[0]
        outs.append(out)
        m_total += a.shape[0]
    gathered = None
    if gather:
        gathered = torch.empty((m_total, n), dtype=torch.float32, device=devices[root])
    dev_idx = (ctypes.c_int32 * nranks)(*[d.index for d in devices])
    streams = (ctypes.c_void_p * nranks)(*[torch.cuda.current_stream(d).cuda_stream
                                           for d in devices])
    _lib.check(_lib.lib().mfk_sharded_gemm_f32(
        descs, nranks, dev_idx, streams, 1 if gather else 0, root,
        gathered.data_ptr() if gather else None, n), "gemm_row_blocks")
    return gathered if gather else outs


class PeerRowGather:
    """One process per GPU: a [rows, cols] fp32 buffer on the root rank that every rank's GEMM
    writes its row block into directly, over NVLink. The root allocates the buffer; its CUDA IPC
    handle goes to every rank once (a collective over `group`), and the other ranks map it. The
    buffer is reused across steps; close() unmaps it (collective)."""

    def __init__(self, rows: int, cols: int, device: torch.device, root: int = 0, group=None):
        from . import _lib

        self.group = group
        self.root = root
        self.rows, self.cols = rows, cols
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.buffer = None
        self._base = None
        if self.rank == root:
            self.buffer = torch.empty((rows, cols), dtype=torch.float32, device=device)
            handle = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
            offset = ctypes.c_int64(0)
            _lib.check(_lib.lib().mfk_ipc_get_handle(self.buffer.data_ptr(), handle,
                                                     ctypes.byref(offset)), "PeerRowGather")
            payload = [bytes(handle), offset.value]
        else:
            payload = [None, None]
        dist.broadcast_object_list(payload, src=dist.get_global_rank(group, root)
                                   if group is not None else root, group=group)
        if self.rank == root:
            self.ptr = self.buffer.data_ptr()
        else:
            handle = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(payload[0])
            base = ctypes.c_void_p(0)
            with torch.cuda.device(device):
                _lib.check(_lib.lib().mfk_ipc_open_handle(handle, ctypes.byref(base)),
                           "PeerRowGather")
            self._base = base.value
            self.ptr = base.value + payload[1]

    def row_ptr(self, row: int) -> int:
        """Device address (valid on this rank's GPU) of row `row` of the root's buffer."""
        return self.ptr + 4 * row * self.cols

    def close(self) -> None:
        from . import _lib

        dist.barrier(group=self.group)
        if self._base is not None:
            _lib.check(_lib.lib().mfk_ipc_close_handle(ctypes.c_void_p(self._base)),
                       "PeerRowGather.close")
            self._base = None


def sharded_gemm(a_local: torch.Tensor, b: torch.Tensor, m_total: int, alpha: float = 1.0,
                 c_local: Optional[torch.Tensor] = None, beta: float = 0.0,
                 transpose_b: bool = False, *, bias: Optional[torch.Tensor] = None,
                 activation: Optional[str] = None, gather=False, group=None,
                 peer: Optional[PeerRowGather] = None, precision: Optional[str] = None,
                 gemm_fn: Optional[Callable] = None) -> Optional[torch.Tensor]:
    """C[rows of this rank] = act(alpha * A_local op(B) + beta * C_local + bias).

    gather=False: returns this rank's rows. gather=True or "nccl": every rank receives the whole
    [m_total, N] C through NCCL's all-gather. gather="peer": this rank's GEMM writes its rows into
    `peer.buffer` on the root over NVLink (no collective on the data path); after a barrier on the
    current streams the root holds C — the root gets the buffer back, the others None. The buffer
    is reused by the next call: a barrier before the GEMMs keeps every rank from writing into it
    until the root's current stream has finished the work queued before the call (reading the
    previous C, for one); read it on another stream only after synchronising with that one.

    `gemm_fn` defaults to the B200 kernel (mensurflow_b200.ops.gemm); it is a parameter so the
    host logic can be exercised with CPU ranks."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    start, stop = block_range(m_total, world, rank)
    if a_local.shape[0] != stop - start:
        raise ValueError(f"sharded_gemm: rank {rank} holds {a_local.shape[0]} rows of A, its "
                         f"block is {stop - start}")
    if gather == "peer":
        if peer is None or peer.rows != m_total:
            raise ValueError("sharded_gemm: gather='peer' needs the PeerRowGather of C")
        # the root is done with the previous contents once every rank has reached this call
        flag = torch.zeros(1, device=a_local.device)
        dist.all_reduce(flag, group=group)
        gemm_into_peer(a_local, b, alpha, c_local, beta, transpose_b, peer.row_ptr(start),
                       peer.cols, bias=bias, activation=activation, precision=precision,
                       peer_memory=peer.rank != peer.root)
        # every rank's rows have landed once every rank's GEMM has finished
        dist.all_reduce(flag, group=group)
        return peer.buffer if rank == peer.root else None
    if gemm_fn is None:
        from .ops import gemm as gemm_fn
    c = gemm_fn(a_local, b, alpha, c_local, beta, False, transpose_b, bias=bias,
                activation=activation)
    if gather and world > 1:
        return gather_rows(c, m_total, group)
    return c


def gemm_into_peer(a: torch.Tensor, b: torch.Tensor, alpha: float, c: Optional[torch.Tensor],
                   beta: float, transpose_b: bool, out_ptr: int, ldc: int, *,
                   bias: Optional[torch.Tensor] = None, activation: Optional[str] = None,
                   precision: Optional[str] = None, peer_memory: bool = True) -> None:
    """The GEMM with its output rows at a raw device address (a peer GPU's buffer mapped on this
    GPU): row i of C at out_ptr + 4 * i * ldc. Queued on the current stream. With `peer_memory`
    (the default) the output is declared another GPU's memory (mfk_gemm_peer_f32: plain stores
    and a system-scope fence, no tensor map over it); the root, writing into its own buffer,
    passes peer_memory=False."""
    from . import _lib
    from .ops import _gemm_desc, _kernel_for, _stream

    _kernel_for("gemm", a)
    right = b.t() if transpose_b else b
    n = right.shape[1]
    stub = torch.empty((1, n), dtype=torch.float32, device=a.device)
    c_in = c if beta != 0.0 else None
    d = _gemm_desc(a, right, stub, alpha, c_in, beta if c_in is not None else 0.0,
                   None if bias is None else bias.contiguous(), activation, precision)
    d.m = a.shape[0]
    d.c = out_ptr
    d.ldc = ldc
    fn = _lib.lib().mfk_gemm_peer_f32 if peer_memory else _lib.lib().mfk_gemm_f32
    _lib.check(fn(ctypes.byref(d), _stream()), "gemm")


def sharded_gemm_batched(a_local: torch.Tensor, b_local: torch.Tensor, batch_total: int,
                         alpha: float = 1.0, transpose_b: bool = False, *, gather: bool = False,
                         group=None, gemm_fn: Optional[Callable] = None) -> torch.Tensor:
    """The batched GEMM split by the (flattened) batch index: each rank multiplies its matrices."""
    if gemm_fn is None:
        from .ops import gemm_strided_batched as gemm_fn
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    out = gemm_fn(a_local, b_local, alpha, None, 0.0, False, transpose_b)
    if gather and world > 1:
        return gather_rows(out, batch_total, group)
    return out
