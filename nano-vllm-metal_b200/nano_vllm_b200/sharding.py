"""KV-head-group partitioning of the attention hot path across GPUs.

Attention is independent per (sequence, kv head) and GQA q heads sit under their
kv head, so each rank owns a contiguous group of kv heads, their page pools
(``[P, Hkv/G, page_size, D]`` with the same page ids on every rank, so block tables
and context lengths are replicated) and the matching q heads.  When there are more
ranks than kv heads (e.g. 4 kv heads on 8 GPUs) each kv head is further split by
batch.  No collective is needed on the data path: every rank writes a disjoint
slice of the output.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    kv_lo: int
    kv_hi: int
    q_lo: int
    q_hi: int
    b_lo: int
    b_hi: int

    @property
    def num_kv_heads(self) -> int:
        return self.kv_hi - self.kv_lo

    @property
    def num_q_heads(self) -> int:
        return self.q_hi - self.q_lo

    @property
    def batch(self) -> int:
        return self.b_hi - self.b_lo


def kv_head_shard(rank: int, world: int, Hq: int, Hkv: int, B: int) -> Shard:
    """The slice of (kv heads, q heads, batch) that `rank` of `world` computes."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if Hq % Hkv != 0:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    g = Hq // Hkv
    if world <= Hkv:
        if Hkv % world != 0:
            raise ValueError(f"{Hkv} kv heads cannot be split evenly over {world} ranks")
        per = Hkv // world
        lo = rank * per
        return Shard(lo, lo + per, lo * g, (lo + per) * g, 0, B)
    if world % Hkv != 0:
        raise ValueError(f"{world} ranks cannot share {Hkv} kv heads evenly")
    splits = world // Hkv
    kv = rank // splits
    part = rank % splits
    chunk = (B + splits - 1) // splits
    b_lo = min(B, part * chunk)
    b_hi = min(B, b_lo + chunk)
    return Shard(kv, kv + 1, kv * g, (kv + 1) * g, b_lo, b_hi)
