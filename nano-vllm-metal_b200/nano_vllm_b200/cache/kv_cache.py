"""Batch-level KV cache over paged request caches (names of ``src/nano_vllm_metal/cache/kv_cache.py``).

Only the paged path is provided.  ``BatchingKvCache.update_and_fetch_paged`` (the
reference's ``kv_cache.py:113-173``) gives every active request the same page ids,
``-1``-padded block-table row and ``context_lens`` entry (its offset after the append;
0 for an empty slot) as the reference, and writes the new K/V of the whole batch with
one scatter-write launch.  The reference's dense batching path (``update_and_fetch``
concatenating per-request tensors behind an additive mask, and ``TinyKvFullCache``)
is not part of the attention hot path and is not provided: ``update_and_fetch`` on the
batch raises ``NotImplementedError``.
"""

from __future__ import annotations

import torch

__all__ = ["TinyKvCache", "BatchingKvCache"]


class TinyKvCache:
    """Interface the model's attention layers call on a per-layer cache.

    A subclass that stores pages implements ``update_and_fetch_paged`` (returns a
    ``PagedKvMetadata``); ``update_and_fetch`` returns dense ``(keys, values, length,
    mask)`` for callers that want the gathered tensors.  ``rewind`` drops tokens from
    the end, ``release`` drops everything.
    """

    def update_and_fetch(self, key, value, mask_length=None, mask=None):
        raise NotImplementedError(f"{type(self).__name__} has no dense update_and_fetch")

    def update_and_fetch_paged(self, key, value, mask_length=None, mask=None):
        raise NotImplementedError(f"{type(self).__name__} does not support paged attention")

    def rewind(self, n: int):
        raise NotImplementedError(f"{type(self).__name__} does not support rewind")

    def release(self):
        return None


class BatchingKvCache(TinyKvCache):
    """Fixed slots of per-request paged caches that share one page pool.

    Slot ``i`` holds a request cache or ``None``.  A batch step passes ``[slots, H, S,
    D]`` keys/values; every active slot appends its ``S`` tokens.
    """

    def __init__(self, max_active_requests: int, max_seq_len: int):
        self.max_active_requests = max_active_requests
        self.max_seq_len = max_seq_len
        self.kv_caches: list[TinyKvCache | None] = [None] * max_active_requests
        self.HD: tuple[int, int] | None = None  # (kv heads, head dim), fixed by the first step

    def _shape(self, keys: torch.Tensor, values: torch.Tensor) -> tuple[int, int, int, int]:
        if keys.shape != values.shape:
            raise ValueError(f"keys {tuple(keys.shape)} and values {tuple(values.shape)} differ")
        slots, heads, new_tokens, dim = keys.shape
        if slots != self.max_active_requests:
            raise ValueError(f"batch has {slots} slots, the cache {self.max_active_requests}")
        if new_tokens > self.max_seq_len:
            raise ValueError(f"{new_tokens} new tokens exceed max_seq_len {self.max_seq_len}")
        if self.HD is None:
            self.HD = (heads, dim)
        elif self.HD != (heads, dim):
            raise ValueError(f"expect (heads, dim) {self.HD} but got {(heads, dim)}")
        return slots, heads, new_tokens, dim

    def update_and_fetch(self, keys, values, mask_length=None, mask=None):
        raise NotImplementedError("BatchingKvCache serves paged attention only; call update_and_fetch_paged")

    def update_and_fetch_paged(self, keys, values, mask_length=None, mask=None):
        from .paged import PagedKvMetadata, TinyKvPagedCache, write_slots

        slots, heads, new_tokens, dim = self._shape(keys, values)
        active = [(i, c) for i, c in enumerate(self.kv_caches) if c is not None]
        if not active:
            raise ValueError("Cannot build paged metadata without active requests")
        pool = active[0][1].pool if isinstance(active[0][1], TinyKvPagedCache) else None
        for _, c in active:
            if not isinstance(c, TinyKvPagedCache):
                raise ValueError("BatchingKvCache contains a non-paged request cache")
            if c.pool is not pool:
                raise ValueError("Paged batch caches must share one page pool")
        # page bookkeeping for every request first (in slot order: the page ids of the
        # reference's sequential loop), then one scatter-write for the whole batch
        slot_of_token = torch.full((slots, new_tokens), -1, dtype=torch.int64)
        for i, c in active:
            slot_of_token[i] = torch.tensor(c.plan_append(new_tokens), dtype=torch.int64)
        dev = keys.device
        pool._ensure_page_storage(keys[:1])
        tok_major = lambda x: x.permute(0, 2, 1, 3).reshape(slots * new_tokens, heads, dim)  # noqa: E731
        write_slots(tok_major(keys), tok_major(values), slot_of_token.view(-1).to(dev), pool.key_pages,
                    pool.value_pages, pool.key_scales, pool.value_scales)
        width = max(c.num_pages for _, c in active)
        table = torch.full((slots, width), -1, dtype=torch.int32)
        lens = torch.zeros(slots, dtype=torch.int32)
        for i, c in active:
            table[i, :c.num_pages] = torch.tensor(c.page_ids, dtype=torch.int32)
            lens[i] = c.offset
        return PagedKvMetadata(key_pages=pool.key_pages, value_pages=pool.value_pages, block_table=table.to(dev),
                               context_lens=lens.to(dev), page_size=pool.page_size, key_scales=pool.key_scales,
                               value_scales=pool.value_scales, mask=mask)

    def add_request(self, prefilled: TinyKvCache, id: int):
        if id >= self.max_active_requests:
            raise ValueError(f"Request id {id} is out of range")
        self.kv_caches[id] = prefilled

    def remove_request(self, id: int):
        cache = self.kv_caches[id]
        if cache is None:
            raise ValueError(f"Request id {id} is not in the cache")
        cache.release()
        self.kv_caches[id] = None
