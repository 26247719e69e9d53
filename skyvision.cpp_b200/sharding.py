"""Multi-GPU placement of the KV-cache path.

The reference is single-GPU (every backend brings up ``ggml_backend_cuda_init(0)``,
src/core/engine/backend.cpp:84-94); its only parallelism is batching several
sequences into one cache (src/models/videochat3/vc3_batch.inc:98-183).  Two
placements follow from that structure:

* **sessions**: independent sessions shard across GPUs with no exchange --
  ``session_shards`` balances them by total context (longest first);
* **kv heads**: one long session shards by KV head -- rank g owns kv heads
  ``kv_head_range(NKV, g, G)`` and the query heads that read them (GQA maps
  query head h to kv head h // (NH/NKV), so a contiguous block of kv heads
  owns a contiguous block of query heads), keeps only those heads' K/V, and the
  per-layer head outputs are all-gathered (``HeadShardedDecode``).

Only the gather is a collective; the attention itself never crosses GPUs.
"""
from __future__ import annotations

import numpy as np


def session_shards(lengths, n_ranks: int) -> list[list[int]]:
    """Longest-first greedy assignment of sessions to ranks by total context."""
    lengths = np.asarray(lengths)
    order = np.argsort(-lengths, kind="stable")
    loads = [0] * n_ranks
    shards: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in order:
        g = int(np.argmin(loads))
        shards[g].append(int(i))
        loads[g] += int(lengths[i])
    return shards


def kv_head_range(n_kv_head: int, rank: int, world: int) -> tuple[int, int]:
    """KV heads [lo, hi) owned by `rank`; requires world to divide n_kv_head."""
    if n_kv_head % world:
        raise ValueError(f"{world} ranks cannot split {n_kv_head} kv heads evenly")
    per = n_kv_head // world
    return rank * per, (rank + 1) * per


def q_head_range(n_head: int, n_kv_head: int, rank: int, world: int) -> tuple[int, int]:
    lo, hi = kv_head_range(n_kv_head, rank, world)
    g = n_head // n_kv_head
    return lo * g, hi * g


class HeadShardedDecode:
    """Decode attention of one session sharded by KV head.

    attend(layer, q_local, k_local, v_local) -> local f32 [T, NH/G, HD] (the rank's heads);
    step_layer() runs it and all-gathers the head outputs into `out_full` [T, NH, HD]
    (torch.distributed: NCCL over NVLink on GPUs, gloo on CPU)."""

    def __init__(self, n_head: int, n_kv_head: int, head_dim: int, rank: int, world: int, group=None):
        self.NH, self.NKV, self.HD = n_head, n_kv_head, head_dim
        self.rank, self.world, self.group = rank, world, group
        self.kv_lo, self.kv_hi = kv_head_range(n_kv_head, rank, world)
        self.q_lo, self.q_hi = q_head_range(n_head, n_kv_head, rank, world)

    def local_heads(self, q_full, k_full, v_full):
        """Slice a full [T, NH, HD] query and [T, NKV*HD] K/V rows down to this rank's heads."""
        HD = self.HD
        return (q_full[:, self.q_lo:self.q_hi],
                k_full[:, self.kv_lo * HD:self.kv_hi * HD],
                v_full[:, self.kv_lo * HD:self.kv_hi * HD])

    def gather(self, local_out, out_full):
        """local_out [T, NH/G, HD] -> out_full [T, NH, HD] in head order."""
        import torch
        import torch.distributed as dist
        if self.world == 1:
            out_full.copy_(local_out)
            return out_full
        T = local_out.shape[0]
        if T == 1 and dist.get_backend(self.group) == "nccl":
            # [G][1][NH/G][HD] is already [1][NH][HD] in memory
            dist.all_gather_into_tensor(out_full.view(self.world, -1), local_out.reshape(-1), group=self.group)
            return out_full
        parts = [torch.empty_like(local_out) for _ in range(self.world)]
        dist.all_gather(parts, local_out.contiguous(), group=self.group)
        out_full.copy_(torch.cat(parts, dim=1))
        return out_full

    def step_layer(self, attend, layer, q_full, k_full, v_full, out_full):
        ql, kl, vl = self.local_heads(q_full, k_full, v_full)
        local = attend(layer, ql.contiguous(), kl.contiguous(), vl.contiguous())
        return self.gather(local, out_full)
