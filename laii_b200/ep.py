"""Expert parallelism for the lfm2moe MoE FFN: one process per GPU, experts
sharded across the ranks, tokens data-parallel.

Each rank holds the full router (replicated) and a contiguous shard of
E/G experts (``shard_of``).  One layer step on a rank's own T tokens:

  1. route locally -- RMSNorm + Q8_K + router + top-K (``ops.route``):
     idx[T, K] global expert ids, w[T, K] weights, q8[T] block_q8_K rows;
  2. dispatch: every (t, k) assignment's Q8_K row goes to the rank owning
     expert idx[t, k] (all-to-all #1 of rows, with their expert ids);
  3. the received rows run through the local experts (``ops.experts``):
     y unweighted, one row per assignment;
  4. combine traffic: y goes back to the home rank (all-to-all #2) and is put
     back in (t, k) order;
  5. combine at home in the reference's k order (``ops.combine``),
     x[t] = fma(w[t, k], y[t, k], x[t]) (tools/lfm2_moe_checkpoint.c:266-269),
     so the result equals the single-GPU layer bit for bit.

Two ways to run it:
  * ``ep_forward`` with a comm object: the exchanges are
    ``torch.distributed.all_to_all_single`` (NCCL over NVLink between GPUs;
    gloo for the host-side tests) and the compute is the CUDA library's
    ``lfm_gpu_moe_ep_*`` entry points (``GpuOps``).  The split sizes come to
    the host every layer.
  * ``p2p_connect`` + ``GpuMoE.ep_p2p_forward``: the whole layer step in the
    library, the exchanges done by its own kernels through CUDA IPC mappings
    of every rank's exchange arena (peer loads and stores over NVLink), with
    no host synchronisation; torch.distributed only carries the IPC handles
    once at setup.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch

Q8K_BYTES = 292


def shard_of(E: int, world: int, rank: int) -> Tuple[int, int]:
    """(first, count) of rank's contiguous expert shard; the first E % world ranks get one more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    base, rem = divmod(E, world)
    first = rank * base + min(rank, rem)
    return first, base + (1 if rank < rem else 0)


def shard_bounds(E: int, world: int) -> List[int]:
    """first expert of every rank, then E."""
    return [shard_of(E, world, r)[0] for r in range(world)] + [E]


def owner_of(ids: torch.Tensor, E: int, world: int) -> torch.Tensor:
    """Owning rank of each global expert id (int64 tensor on ids.device)."""
    bounds = torch.tensor(shard_bounds(E, world)[1:-1], dtype=torch.int64, device=ids.device)
    return torch.bucketize(ids.to(torch.int64), bounds, right=True)


class LocalComm:
    """World of one: every row stays home."""

    world = 1
    rank = 0

    def exchange(self, send: torch.Tensor, send_counts: Sequence[int],
                 recv_counts: Optional[Sequence[int]] = None) -> Tuple[torch.Tensor, List[int]]:
        return send, list(send_counts)


class TorchComm:
    """all_to_all_single over a torch.distributed group (rows of variable counts per peer)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def exchange(self, send: torch.Tensor, send_counts: Sequence[int],
                 recv_counts: Optional[Sequence[int]] = None) -> Tuple[torch.Tensor, List[int]]:
        send_counts = [int(c) for c in send_counts]
        if recv_counts is None:
            sc = torch.tensor(send_counts, dtype=torch.int64, device=send.device)
            rc = torch.empty_like(sc)
            self.dist.all_to_all_single(rc, sc, group=self.group)
            recv_counts = rc.tolist()
        recv_counts = [int(c) for c in recv_counts]
        recv = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        self.dist.all_to_all_single(recv, send.contiguous(), output_split_sizes=recv_counts,
                                    input_split_sizes=send_counts, group=self.group)
        return recv, recv_counts


def ep_forward(ops, comm, layer: int, x: torch.Tensor, E: int, K: int) -> torch.Tensor:
    """x[T, D] += MoE(x) for this rank's tokens, in place, experts spread over comm's ranks."""
    T = x.shape[0]
    idx, w, q8 = ops.route(layer, x)
    flat = idx.reshape(-1).to(torch.int64)
    owner = owner_of(flat, E, comm.world)
    order = torch.argsort(owner, stable=True)          # assignments grouped by destination rank
    send_counts = torch.bincount(owner, minlength=comm.world).tolist()
    send_q8 = q8.index_select(0, order // K)            # the token's Q8_K row, once per assignment
    send_ids = flat.index_select(0, order).to(torch.int32)
    recv_q8, recv_counts = comm.exchange(send_q8, send_counts)
    recv_ids, _ = comm.exchange(send_ids, send_counts, recv_counts)
    y_recv = ops.experts(layer, recv_q8, recv_ids)
    y_back, _ = comm.exchange(y_recv, recv_counts, send_counts)
    y = torch.empty_like(y_back)
    y[order] = y_back                                   # (t, k) order again
    ops.combine(layer, x, w, y.reshape(T * K, -1))
    return x


class GpuOps:
    """The CUDA library's expert-parallel calls on a GpuMoE handle, on torch's current stream."""

    MAX_ROWS = 65535

    def __init__(self, moe, D: int, K: int):
        self.moe = moe
        self.D = D
        self.K = K
        self.launches = 0  # CUDA kernels launched by the library through these calls

    def _count(self):
        self.launches += self.moe.last_stats()["kernels_launched"]

    def _stream(self) -> int:
        return torch.cuda.current_stream().cuda_stream

    def route(self, layer: int, x: torch.Tensor):
        T = x.shape[0]
        dev = x.device
        idx = torch.empty((T, self.K), dtype=torch.int32, device=dev)
        w = torch.empty((T, self.K), dtype=torch.float32, device=dev)
        q8 = torch.empty((T, self.D // 256 * Q8K_BYTES), dtype=torch.uint8, device=dev)
        self.moe.ep_route(layer, x.data_ptr(), T, idx.data_ptr(), w.data_ptr(), q8.data_ptr(), self._stream())
        self._count()
        return idx, w, q8

    def experts(self, layer: int, q8: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        n = q8.shape[0]
        y = torch.empty((n, self.D), dtype=torch.float32, device=q8.device)
        q8 = q8.contiguous()
        ids = ids.contiguous()
        for a in range(0, n, self.MAX_ROWS):
            m = min(self.MAX_ROWS, n - a)
            self.moe.ep_experts(layer, q8[a:].data_ptr(), m, ids[a:].data_ptr(), y[a:].data_ptr(), self._stream())
            self._count()
        return y

    def combine(self, layer: int, x: torch.Tensor, w: torch.Tensor, y: torch.Tensor) -> None:
        self.moe.ep_combine(layer, x.data_ptr(), x.shape[0], w.contiguous().data_ptr(), y.contiguous().data_ptr(),
                            self._stream())
        self._count()


def p2p_connect(moe, max_tokens: int, D: int, E: int, K: int, I: int, group=None, wait_ms: int = 0):
    """Attach moe's exchange arena for up to max_tokens tokens per rank and map
    every other rank's (one process per GPU, torch.distributed initialised;
    without it, a world of one).  Returns (rank, world).  Collective: every
    rank calls it, then ``moe.ep_p2p_forward`` for the same layers in order."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        world, rank = dist.get_world_size(group), dist.get_rank(group)
    else:
        world, rank = 1, 0
    handle = moe.ep_p2p_attach(rank, world, max_tokens, D, E, K, I, wait_ms)
    if world == 1:
        moe.ep_p2p_connect([handle])
        return rank, world
    handles: List[Optional[bytes]] = [None] * world
    dist.all_gather_object(handles, handle, group=group)
    moe.ep_p2p_connect(handles)
    dist.barrier(group=group)  # no rank writes into an arena before its owner has mapped every peer
    return rank, world
