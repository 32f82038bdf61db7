"""Multi-GPU decode: one process per GPU, torch.distributed (NCCL over NVLink)
for the plumbing.

Two ways the hot path spreads over the GPUs of one box:

* Batched decode (independent sequences): each rank owns whole sequences and
  decodes them with no collective on the data path. `lpt_partition` balances a
  fixed set of sequences over ranks by KV bytes (strong scaling); the benchmark
  gives every rank its own set (weak scaling).

* Split-KV decode (long contexts): every rank holds the same contiguous slice
  of every sequence's positions (`position_slice`), the new token landing on the
  last rank. `SplitKVDecode.step` computes this rank's partial (o, m, l) per
  (sequence, query head), gathers all ranks' partials with one all-gather, and
  merges them with the log-sum-exp combine in ascending rank order, so every
  rank gets the same bits. `PeerSplitKV` does the same exchange inside the
  attention kernel (peer stores and flags over NVLink, b2a_attention_decode_split):
  one launch per step and no library collective; `SplitKVDecode` with NCCL is
  the baseline it replaces.

The compute and the gather are pluggable so the orchestration can be tested
with the gloo backend on CPU; by default they are the CUDA kernels of
libb2a.so and torch.distributed's NCCL all-gather.
"""
from __future__ import annotations

import ctypes
import heapq
from typing import Callable, Sequence


def position_slice(total: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the positions 0..total-1 that `rank` holds: contiguous ceil-divided slices."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    per = (total + world - 1) // world
    lo = min(total, rank * per)
    hi = min(total, lo + per)
    return lo, hi


def lpt_partition(weights: Sequence[int], world: int) -> list[list[int]]:
    """Greedy longest-processing-time assignment of items (sequence indices) to
    `world` bins by weight (KV positions): heaviest first onto the lightest bin.
    Deterministic: ties go to the lower rank."""
    order = sorted(range(len(weights)), key=lambda i: (-weights[i], i))
    heap = [(0, r) for r in range(world)]
    bins: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        bins[r].append(i)
        heapq.heappush(heap, (load + int(weights[i]), r))
    return [sorted(b) for b in bins]


class SplitKVDecode:
    """One split-KV decode step across the ranks of a process group.

    partial_fn(q, k_new, v_new, positions, out_partial) -> None
        writes this rank's [batch, heads, head_dim + 4] partial; k_new/v_new are
        given only on the rank that holds the new token (the last one).
    gather_fn(local) -> stacked [world, ...] partials in rank order.
    combine_fn(stacked, out) -> None
        merges the world partials into out [batch, heads, head_dim].
    """

    def __init__(self, rank: int, world: int, partial_fn: Callable, gather_fn: Callable, combine_fn: Callable):
        self.rank, self.world = rank, world
        self.partial_fn, self.gather_fn, self.combine_fn = partial_fn, gather_fn, combine_fn

    @property
    def holds_new_token(self) -> bool:
        return self.rank == self.world - 1

    def step(self, q, k_new, v_new, positions, local_partial, out):
        self.partial_fn(q, k_new if self.holds_new_token else None, v_new if self.holds_new_token else None,
                        positions, local_partial)
        stacked = self.gather_fn(local_partial)
        self.combine_fn(stacked, out)
        return out


def nccl_gather_fn(group=None):
    """All-gather of a CUDA tensor into a new [world, *shape] tensor (NCCL)."""
    import torch
    import torch.distributed as dist

    def gather(local):
        world = dist.get_world_size(group)
        flat = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                           device=local.device)
        dist.all_gather_into_tensor(flat, local.contiguous(), group=group)
        return flat.view((world,) + tuple(local.shape))

    return gather


def cuda_split_kv(ctx, cache, rope, layer: int, num_heads: int, rank: int, world: int, group=None,
                  dtype: str | None = None, num_layers: int = 1) -> SplitKVDecode:
    """SplitKVDecode wired to libb2a's partial and combine kernels and NCCL, over
    layers [layer, layer + num_layers) per step (partials [batch, layers, heads, 68])."""
    from . import attention as A

    head_dim = cache.config.headDim

    def partial_fn(q, k_new, v_new, positions, out_partial):
        A.decodePartial(ctx, cache, rope, layer, q, k_new, v_new, positions, out_partial, num_heads, dtype=dtype,
                        numLayers=num_layers)

    def combine_fn(stacked, out):
        rows = stacked.shape[1] * num_layers   # (sequence, layer) rows
        A.lseCombine(ctx, stacked, world, rows, num_heads, head_dim, out)

    return SplitKVDecode(rank, world, partial_fn, nccl_gather_fn(group), combine_fn)


class NcclComm:
    """An NCCL communicator made through libnccl.so.2 itself (ctypes), for the
    one-call NCCL split-KV decode (b2a_split_kv_decode_nccl): one rank makes
    `unique_id()`, the others receive it over any channel, and every rank opens
    NcclComm(uid, world, rank) with its GPU current. `single()` makes a
    communicator of one rank. The library loaded is the process's own
    libnccl.so.2 (torch's, once torch has loaded it)."""

    ID_BYTES = 128

    class _Id(ctypes.Structure):
        _fields_ = [("internal", ctypes.c_char * 128)]

    @staticmethod
    def _lib():
        return ctypes.CDLL("libnccl.so.2")

    @classmethod
    def unique_id(cls) -> bytes:
        uid = cls._Id()
        r = cls._lib().ncclGetUniqueId(ctypes.byref(uid))
        if r != 0:
            raise RuntimeError(f"ncclGetUniqueId failed ({r})")
        return ctypes.string_at(ctypes.addressof(uid), cls.ID_BYTES)

    def __init__(self, uid: bytes | None, world: int, rank: int, _comm=None):
        self.world, self.rank = world, rank
        self._handle = ctypes.c_void_p()
        if _comm is not None:
            self._handle = _comm
            return
        if uid is None or len(uid) != self.ID_BYTES:
            raise ValueError("an NCCL unique id of 128 bytes")
        u = self._Id()
        ctypes.memmove(ctypes.addressof(u), uid, self.ID_BYTES)
        r = self._lib().ncclCommInitRank(ctypes.byref(self._handle), world, u, rank)
        if r != 0:
            raise RuntimeError(f"ncclCommInitRank failed ({r})")

    @classmethod
    def single(cls, device: int = 0) -> "NcclComm":
        comm = ctypes.c_void_p()
        devs = (ctypes.c_int * 1)(device)
        r = cls._lib().ncclCommInitAll(ctypes.byref(comm), 1, devs)
        if r != 0:
            raise RuntimeError(f"ncclCommInitAll failed ({r})")
        return cls(None, 1, 0, _comm=comm)

    @property
    def value(self) -> int:
        return self._handle.value

    def close(self) -> None:
        if self._handle.value:
            self._lib().ncclCommDestroy(self._handle)
            self._handle = ctypes.c_void_p()


class NcclSplitKV:
    """Split-KV decode with the all-gather over NCCL in one library call per step
    (b2a_split_kv_decode_nccl): the C-ABI form of `cuda_split_kv`, for hosts that
    hold an NCCL communicator but no torch.distributed process group."""

    def __init__(self, ctx, cache, rope, layer: int, num_heads: int, comm: NcclComm, num_layers: int = 1,
                 dtype: str | None = None):
        self.ctx, self.cache, self.rope, self.layer = ctx, cache, rope, layer
        self.num_heads, self.comm, self.num_layers, self.dtype = num_heads, comm, num_layers, dtype

    def step(self, q, k_new, v_new, positions, out):
        from . import attention as A
        A.decodeSplitNccl(self.ctx, self.cache, self.rope, self.layer, q, k_new, v_new, positions, self.comm,
                          self.comm.world, self.comm.rank, out, self.num_heads, dtype=self.dtype,
                          numLayers=self.num_layers)
        return out


def gather_handles(handle: bytes, world: int, group=None) -> bytes:
    """Every rank's exchange handle in rank order: one all-gather of a byte tensor
    (a CUDA tensor under NCCL, a CPU tensor under gloo)."""
    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
        else torch.device("cpu")
    local = torch.tensor(list(handle), dtype=torch.uint8, device=dev)
    flat = torch.empty(world * len(handle), dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(flat, local, group=group)
    return bytes(flat.cpu().tolist())


def _all_ranks_ok(ok: bool, group=None) -> bool:
    """True on every rank iff ok is true on every rank (an all-reduce of a flag)."""
    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
        else torch.device("cpu")
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(t.item())


class PeerSplitKV:
    """Split-KV decode whose cross-rank exchange runs inside the attention kernel.

    Construction is collective: every rank makes its exchange, the handles are
    all-gathered once, and each rank maps the others' buffers. step() is one
    launch per rank; every rank must call it the same number of times."""

    def __init__(self, ctx, cache, rope, layer: int, num_heads: int, rank: int, world: int, group=None,
                 dtype: str | None = None, num_layers: int = 1):
        from .runtime import Exchange

        self.ctx, self.cache, self.rope, self.layer = ctx, cache, rope, layer
        self.num_heads, self.rank, self.world, self.dtype = num_heads, rank, world, dtype
        self.num_layers = num_layers
        self.exchange = None
        err = None
        try:
            self.exchange = Exchange(ctx, world, rank, cache.batch, num_heads, cache.config.numKVHeads, num_layers)
            handle = self.exchange.handle_bytes()
        except Exception as e:   # every rank must still reach the collectives below
            err, handle = e, bytes(64)
        if not _all_ranks_ok(err is None, group):
            raise RuntimeError(f"creating the exchange failed on some rank: {err}") from err
        handles = gather_handles(handle, world, group)
        try:
            self.exchange.open(handles)
        except Exception as e:
            err = e
        if not _all_ranks_ok(err is None, group):
            raise RuntimeError(f"opening the peers' exchange buffers failed on some rank: {err}") from err

    @property
    def holds_new_token(self) -> bool:
        return self.rank == self.world - 1

    def step(self, q, k_new, v_new, positions, out):
        from . import attention as A

        A.decodeSplit(self.ctx, self.cache, self.rope, self.layer, q, k_new if self.holds_new_token else None,
                      v_new if self.holds_new_token else None, positions, self.exchange, out, self.num_heads,
                      dtype=self.dtype, numLayers=self.num_layers)
        return out

    def close(self) -> None:
        if self.exchange is not None:
            self.exchange.close()
