"""Multi-GPU layer for the INT8 decode path (one process per GPU, torch.distributed).

The reference has no distributed code; this layer adds the two ways the
north-star spec splits decode across the GPUs of one node:

* Batch x head shards (configurations 2, 4, 5): every rank owns whole
  sequences in its own HBM and decodes them with no communication.
  `batch_shard` gives contiguous equal shards; `lpt_assign` balances ragged
  batches by tokens (longest-processing-time greedy).
* Sequence split (configuration 3, very long contexts): rank g owns tokens
  [g*S/N, (g+1)*S/N) of every head. Each rank decodes its shard into partial
  (m, l, o) records (KVD_FLAG_PARTIAL_OUT), the records of all ranks are
  all-gathered over NVLink (NCCL), and every rank merges them with the
  log-sum-exp combine kernel. Only B*Hq*(D+4) floats per rank cross NVLink.

The local decode and the combine are the library's CUDA kernels; tests may
inject host stand-ins to exercise the orchestration on CPU with gloo ranks.
"""
from __future__ import annotations

import heapq
from typing import Callable, Sequence

import kvdecode as kvd


def batch_shard(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous shard [lo, hi) of `batch` sequences for `rank` (sizes differ by at most 1)."""
    lo = (rank * batch) // world
    hi = ((rank + 1) * batch) // world
    return lo, hi


def seq_shard(seq_len: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Contiguous token range [lo, hi) of rank `rank`; boundaries rounded to `align` tokens."""
    def cut(g: int) -> int:
        x = (g * seq_len) // world
        return min(seq_len, ((x + align - 1) // align) * align) if 0 < g < world else x

    return cut(rank), cut(rank + 1)


def lpt_assign(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Sequences -> ranks, balancing the summed lengths (greedy, longest first)."""
    order = sorted(range(len(lengths)), key=lambda b: -int(lengths[b]))
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for b in order:
        load, r = heapq.heappop(heap)
        out[r].append(b)
        heapq.heappush(heap, (load + int(lengths[b]), r))
    for r in range(world):
        out[r].sort()
    return out


class SeqSplitDecode:
    """Sequence-split decode across the ranks of a process group.

    Call with this rank's token shard of the cache (K/V [B, Hkv, shard, D],
    scales [B, Hkv, shard]) and the full query [B, Hq, D]; returns the combined
    output [B, Hq, D] on every rank. Buffers are allocated once, so a step
    allocates nothing and can be timed or captured (NCCL calls inside a CUDA
    graph need the graph released before destroy_process_group)."""

    def __init__(self, batch: int, q_heads: int, head_dim: int, device, group=None,
                 local_decode: Callable | None = None, combine: Callable | None = None):
        import torch
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        rows = batch * q_heads
        self.shape = (batch, q_heads, head_dim)
        self.records = torch.empty((batch, q_heads, head_dim + 4), dtype=torch.float32, device=device)
        self.gathered = torch.empty((self.world, rows, head_dim + 4), dtype=torch.float32, device=device)
        self.local_decode = local_decode or self._decode_records
        self.combine = combine or (lambda parts, out: kvd.combine(parts, out=out))
        self.workspace = None

    def _decode_records(self, q, K, V, ks, vs, records, seq_lens=None):
        import torch

        if self.workspace is None:
            desc = kvd.make_desc(q, K, ks, records, seq_lens, partial=True)
            self.workspace = torch.empty(max(kvd.workspace_size(desc), 1), dtype=torch.uint8, device=q.device)
        kvd.decode(q, K, V, ks, vs, out=records, seq_lens=seq_lens, partial=True, workspace=self.workspace)

    def __call__(self, q, K, V, ks, vs, out=None, seq_lens=None):
        import torch

        if out is None:
            out = torch.empty(self.shape, dtype=torch.float32, device=q.device)
        self.local_decode(q, K, V, ks, vs, self.records, seq_lens)
        self.dist.all_gather_into_tensor(self.gathered.view(-1), self.records.view(-1), group=self.group)
        self.combine(self.gathered, out.view(-1, self.shape[2]))
        return out
