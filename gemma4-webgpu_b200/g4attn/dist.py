"""Multi-GPU partitioning of the decode path (new capability: the reference has one WebGPU device).

Two partitionings, both one process per GPU:

* Batched decode -- independent sequences are assigned to ranks by longest-processing-time
  (LPT) bin packing on their KV bytes; every rank runs the paged decode on its own sequences.
  No collective touches the data path.
* Long-context decode -- one sequence's KV positions are split evenly along the length; each
  rank computes a split-KV partial (m | l | o) over its slice with ``g4a_decode_attn_partial``,
  the partials (8 * (head_dim + 2) floats per rank) are all-gathered over NCCL with
  ``torch.distributed``, and every rank runs the log-sum-exp merge kernel ``g4a_lse_merge``.

Collective plumbing: either torch.distributed (NCCL on GPUs, gloo for the CPU tests), or the
library's own communicator through its C ABI (``g4a_dist_init`` / ``g4a_decode_attn_splitkv`` /
``g4a_dist_allgather_host``: ``CabiSplitKVDecoder`` and ``CabiPeerSplitKVDecoder``), which needs
no torch.distributed at all -- the path a TypeScript / N-API host uses.  The numeric work stays
in libg4attn.so either way.
"""
from __future__ import annotations

import heapq

import numpy as np


def lpt_shard(costs, n_ranks: int) -> list[list[int]]:
    """Assign items (by index) to n_ranks bins, largest cost first to the least-loaded bin.
    Deterministic: ties go to the lower rank; each bin's items are returned sorted."""
    costs = np.asarray(costs, dtype=np.int64)
    order = sorted(range(len(costs)), key=lambda i: (-int(costs[i]), i))
    heap = [(0, r) for r in range(n_ranks)]
    heapq.heapify(heap)
    bins: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in order:
        load, r = heapq.heappop(heap)
        bins[r].append(i)
        heapq.heappush(heap, (load + int(costs[i]), r))
    return [sorted(b) for b in bins]


def decode_cost_bytes(lengths, window: int = 0, head_dim: int = 256, num_kv_heads: int = 1) -> np.ndarray:
    """KV bytes one decode layer-call reads per sequence (visible K and V rows, f16)."""
    L = np.asarray(lengths, dtype=np.int64)
    vis = np.minimum(L, window) if window else L
    return 2 * vis * num_kv_heads * head_dim * 2


def splitkv_ranges(kv_len: int, n_ranks: int, align: int = 32) -> list[tuple[int, int]]:
    """Even split of positions [0, kv_len) into n_ranks contiguous ranges (boundaries rounded down
    to `align` positions so every rank's slice starts on a whole stage)."""
    bounds = [0]
    for r in range(1, n_ranks):
        b = (kv_len * r // n_ranks) // align * align
        bounds.append(max(b, bounds[-1]))
    bounds.append(kv_len)
    return [(bounds[r], bounds[r + 1]) for r in range(n_ranks)]


def partial_floats(num_q_heads: int, head_dim: int) -> int:
    return num_q_heads * (head_dim + 2)


def merge_partials_host(parts: np.ndarray, num_q_heads: int, head_dim: int) -> np.ndarray:
    """Host restatement of the LSE merge for checking gathered partials (base-2 maxima).
    parts: [n, num_q_heads * (head_dim + 2)] laid out m | l | o."""
    parts = np.asarray(parts, dtype=np.float64).reshape(len(parts), -1)
    m = parts[:, :num_q_heads]
    l_ = parts[:, num_q_heads:2 * num_q_heads]
    o = parts[:, 2 * num_q_heads:].reshape(len(parts), num_q_heads, head_dim)
    M = m.max(axis=0)
    with np.errstate(invalid="ignore"):
        w = np.where(np.isfinite(m), np.exp2(m - M), 0.0)
    L = (w * l_).sum(axis=0)
    O = (w[:, :, None] * o).sum(axis=0)
    out = np.where(L[:, None] > 0, O / np.where(L[:, None] > 0, L[:, None], 1.0), 0.0)
    return out.astype(np.float32)


class SplitKVDecoder:
    """Long-context decode of one sequence split along KV length over a process group.

    Each rank holds K/V rows for positions [begin, end) of its slice (``splitkv_ranges``).
    ``step`` computes the rank's partial, all-gathers every rank's partial and merges them;
    every rank ends with the full attention output.
    """

    def __init__(self, ctx, group=None, num_q_heads: int = 8, head_dim: int = 256):
        import torch
        import torch.distributed as dist

        self.ctx = ctx
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nqh = num_q_heads
        self.hd = head_dim
        n = partial_floats(num_q_heads, head_dim)
        dev = torch.device("cuda", ctx.device)
        self.part = torch.empty(n, dtype=torch.float32, device=dev)
        self.gathered = torch.empty(self.world * n, dtype=torch.float32, device=dev)

    def partial(self, q, k_slice, v_slice, *, begin, end, kv_len_total, scale=1.0, sliding_window=0,
                num_kv_heads=1):
        self.ctx.decode_attn_partial(q, k_slice, v_slice, self.part, num_q_heads=self.nqh, num_kv_heads=num_kv_heads,
                                     head_dim=self.hd, kv_begin=begin, kv_end=end, kv_len_total=kv_len_total,
                                     scale=scale, sliding_window=sliding_window)
        return self.part

    def gather_and_merge(self, out):
        import torch.distributed as dist

        dist.all_gather_into_tensor(self.gathered, self.part, group=self.group)
        self.ctx.lse_merge(self.gathered, self.world, out, num_q_heads=self.nqh, head_dim=self.hd)
        return out

    def step(self, q, k_slice, v_slice, out, *, begin, end, kv_len_total, scale=1.0, sliding_window=0):
        self.partial(q, k_slice, v_slice, begin=begin, end=end, kv_len_total=kv_len_total, scale=scale,
                     sliding_window=sliding_window)
        return self.gather_and_merge(out)


class PeerSplitKVDecoder:
    """Long-context decode of one sequence split along KV length, with the partials exchanged
    over NVLink peer memory by the library's exchange kernel instead of a collective.

    Every rank allocates one exchange buffer (``g4a_exchange_buffer_bytes``), exports it as a
    CUDA IPC handle, and opens the other ranks' handles; the 64-byte handles travel once over
    the process group (any backend).  ``step`` computes this rank's partial and calls
    ``splitkv_exchange_merge``, which pushes it into every rank's buffer, waits for all of them
    and merges; every rank ends with the full attention output.  All ranks must call ``step``
    the same number of times; ``close`` (collective) releases the buffers after a barrier.
    """

    def __init__(self, ctx, group=None, num_q_heads: int = 8, head_dim: int = 256):
        import torch
        import torch.distributed as dist

        from ._lib import load

        self.ctx = ctx
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nqh = num_q_heads
        self.hd = head_dim
        self.seq = 0
        self._setup(load, num_q_heads, head_dim)

    def _allgather_bytes(self, data: bytes) -> list[bytes]:
        import torch
        import torch.distributed as dist

        t = torch.tensor(list(data), dtype=torch.uint8)
        if dist.get_backend(self.group) == "nccl":
            t = t.cuda(self.ctx.device)
        out = [torch.zeros_like(t) for _ in range(self.world)]
        dist.all_gather(out, t, group=self.group)
        return [bytes(x.cpu().tolist()) for x in out]

    def _barrier(self) -> None:
        import torch.distributed as dist

        dist.barrier(group=self.group)

    def _setup(self, load, num_q_heads: int, head_dim: int) -> None:
        import torch

        ctx = self.ctx
        nbytes = int(load().g4a_exchange_buffer_bytes(self.world, num_q_heads, head_dim))
        self.own = ctx.alloc(nbytes)
        ctx.memset(self.own, 0, nbytes)
        ctx.sync()
        handles = self._allgather_bytes(ctx.ipc_handle(self.own))
        self.opened = []
        self.buffers = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.buffers.append(self.own)
            else:
                p = ctx.ipc_open(h)
                self.opened.append(p)
                self.buffers.append(p)
        self._barrier()
        dev = torch.device("cuda", ctx.device)
        self.part = torch.empty(partial_floats(num_q_heads, head_dim), dtype=torch.float32, device=dev)

    def step(self, q, k_slice, v_slice, out, *, begin, end, kv_len_total, scale=1.0, sliding_window=0,
             num_kv_heads=1):
        self.ctx.decode_attn_partial(q, k_slice, v_slice, self.part, num_q_heads=self.nqh, num_kv_heads=num_kv_heads,
                                     head_dim=self.hd, kv_begin=begin, kv_end=end, kv_len_total=kv_len_total,
                                     scale=scale, sliding_window=sliding_window)
        self.seq += 1
        self.ctx.splitkv_exchange_merge(self.part, self.buffers, self.rank, self.seq, out, num_q_heads=self.nqh,
                                        head_dim=self.hd)
        return out

    def close(self) -> None:
        self.ctx.sync()
        self._barrier()  # nobody writes into a buffer after this point
        for p in self.opened:
            self.ctx.ipc_close(p)
        self.opened = []
        self._barrier()
        if self.own:
            self.ctx.free(self.own)
            self.own = 0


class CabiPeerSplitKVDecoder(PeerSplitKVDecoder):
    """``PeerSplitKVDecoder`` bootstrapped over the context's own communicator (``ctx.dist_init``
    done by the caller): the IPC handles travel with ``g4a_dist_allgather_host`` and the barriers
    are one-byte all-gathers, so no torch.distributed is involved."""

    def __init__(self, ctx, num_q_heads: int = 8, head_dim: int = 256, timeout_ms: int = 60000):
        from ._lib import load

        self.ctx = ctx
        self.group = None
        self.rank, self.world = ctx.dist_info()
        if self.world < 1:
            raise ValueError("the context has no communicator: call ctx.dist_init first")
        self.nqh = num_q_heads
        self.hd = head_dim
        self.seq = 0
        self.timeout_ms = timeout_ms
        self._setup(load, num_q_heads, head_dim)

    def _allgather_bytes(self, data: bytes) -> list[bytes]:
        return self.ctx.dist_allgather_host(data, self.timeout_ms)

    def _barrier(self) -> None:
        self.ctx.dist_allgather_host(b"\x01", self.timeout_ms)


class CabiSplitKVDecoder:
    """Long-context split-KV decode through the C ABI alone: ``g4a_decode_attn_splitkv`` computes
    the partial of this rank's slice, all-gathers the partials over the context's NCCL
    communicator (``ctx.dist_init``, non-blocking with deadlines) and merges them."""

    def __init__(self, ctx, num_q_heads: int = 8, head_dim: int = 256, timeout_ms: int = 60000):
        import torch

        self.ctx = ctx
        self.rank, self.world = ctx.dist_info()
        if self.world < 1:
            raise ValueError("the context has no communicator: call ctx.dist_init first")
        self.nqh = num_q_heads
        self.hd = head_dim
        self.timeout_ms = timeout_ms
        dev = torch.device("cuda", ctx.device)
        self.parts_all = torch.empty(self.world * partial_floats(num_q_heads, head_dim), dtype=torch.float32,
                                     device=dev)

    def step(self, q, k_slice, v_slice, out, *, begin, end, kv_len_total, scale=1.0, sliding_window=0):
        self.ctx.decode_attn_splitkv(q, k_slice, v_slice, self.parts_all, out, num_q_heads=self.nqh, num_kv_heads=1,
                                     head_dim=self.hd, kv_begin=begin, kv_end=end, kv_len_total=kv_len_total,
                                     scale=scale, sliding_window=sliding_window, timeout_ms=self.timeout_ms)
        return out
