"""KV cache interfaces mirroring ``src/nano_vllm_metal/cache/kv_cache.py``.

``BatchingKvCache.update_and_fetch_paged`` (reference ``kv_cache.py:113-173``) keeps
the reference's per-request bookkeeping (same page ids, same ``-1``-padded block
table, ``context_lens`` = each request's offset, 0 for empty slots) but writes the
new K/V of every request with a single scatter-write kernel launch instead of one
MLX slice-assign per page per request.  The dense path (``update_and_fetch``,
``TinyKvFullCache``) is plain torch, kept for callers and tests.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Optional

import torch

__all__ = ["TinyKvCache", "BatchingKvCache", "TinyKvFullCache"]


class TinyKvCache(ABC):
    @abstractmethod
    def update_and_fetch(self, key, value, mask_length=None, mask=None):
        """Append key/value; return (keys, values, sequence length, mask)."""

    def release(self):
        return None

    def update_and_fetch_paged(self, key, value, mask_length=None, mask=None):
        raise NotImplementedError("This KV cache does not support paged attention")

    def rewind(self, n: int):
        raise NotImplementedError("This KV cache does not support rewind")


class BatchingKvCache(TinyKvCache):
    def __init__(self, max_active_requests: int, max_seq_len: int):
        self.max_active_requests = max_active_requests
        self.max_seq_len = max_seq_len
        self.kv_caches: list[TinyKvCache | None] = [None] * max_active_requests
        self.HD = None

    def _check(self, keys, values):
        B, H, S, D = keys.shape
        assert keys.shape == values.shape
        assert S <= self.max_seq_len
        assert B == self.max_active_requests
        if self.HD is None:
            self.HD = (H, D)
        else:
            assert self.HD == (H, D), f"expect {self.HD} but got {(H, D)}"
        return B, H, S, D

    def update_and_fetch(self, keys, values, mask_length=None, mask=None):
        from ..layers.attention import causal_mask

        B, H, S, D = self._check(keys, values)
        data = []
        for b in range(B):
            cache = self.kv_caches[b]
            if cache is None:
                data.append(None)
                continue
            k, v, seq_len, row_mask = cache.update_and_fetch(keys[b:b + 1], values[b:b + 1], mask=mask)
            data.append((k[0], v[0], seq_len, row_mask))
        seq_len = max((d[2] if d is not None else 0 for d in data), default=0)
        bk = torch.zeros((B, H, seq_len, D), dtype=keys.dtype, device=keys.device)
        bv = torch.zeros((B, H, seq_len, D), dtype=values.dtype, device=values.device)
        if mask_length is None:
            mask_length = S
        masks = torch.full((B, mask_length, seq_len), float("-inf"), dtype=keys.dtype, device=keys.device)
        for b, d in enumerate(data):
            if d is None:
                continue
            k, v, row_len, row_mask = d
            start = seq_len - row_len
            bk[b, :, start:seq_len, :] = k
            bv[b, :, start:seq_len, :] = v
            if row_mask is None or (isinstance(row_mask, str) and row_mask == "causal"):
                masks[b, :, start:seq_len] = causal_mask(mask_length, row_len, keys.dtype, keys.device)
            elif isinstance(row_mask, torch.Tensor):
                masks[b, :, start:seq_len] = row_mask
            else:
                raise NotImplementedError
        return bk, bv, None, masks.reshape(B, 1, mask_length, seq_len)

    def update_and_fetch_paged(self, keys, values, mask_length=None, mask=None):
        from .paged import PagedKvMetadata, TinyKvPagedCache, write_slots

        B, H, S, D = self._check(keys, values)
        pool = None
        context_lens, slot_rows = [], []
        max_pages = 0
        for b in range(B):
            cache = self.kv_caches[b]
            if cache is None:
                context_lens.append(0)
                continue
            if not isinstance(cache, TinyKvPagedCache):
                raise ValueError("BatchingKvCache contains a non-paged request cache")
            if pool is None:
                pool = cache.pool
            elif pool is not cache.pool:
                raise ValueError("Paged batch caches must share one page pool")
            slots = cache.plan_append(S)
            slot_rows.append((b, slots))
            context_lens.append(cache.offset)
            max_pages = max(max_pages, cache.num_pages)
        if pool is None:
            raise ValueError("Cannot build paged metadata without active requests")
        dev = keys.device
        # One scatter-write for every active request: token (b, s) -> slot.
        all_slots = torch.full((B, S), -1, dtype=torch.int64)
        for b, slots in slot_rows:
            all_slots[b] = torch.tensor(slots, dtype=torch.int64)
        pool._ensure_page_storage(keys[:1])
        kt = keys.permute(0, 2, 1, 3).reshape(B * S, H, D)
        vt = values.permute(0, 2, 1, 3).reshape(B * S, H, D)
        write_slots(kt, vt, all_slots.reshape(-1).to(dev), pool.key_pages, pool.value_pages, pool.key_scales,
                    pool.value_scales)
        rows = []
        for cache in self.kv_caches:
            if cache is None:
                rows.append([-1] * max_pages)
            else:
                rows.append(cache.page_ids + [-1] * (max_pages - cache.num_pages))
        return PagedKvMetadata(
            key_pages=pool.key_pages, value_pages=pool.value_pages,
            block_table=torch.tensor(rows, dtype=torch.int32).reshape(B, max_pages).to(dev),
            context_lens=torch.tensor(context_lens, dtype=torch.int32).to(dev),
            page_size=pool.page_size, key_scales=pool.key_scales, value_scales=pool.value_scales, mask=mask)

    def add_request(self, prefilled: TinyKvCache, id: int):
        if id >= self.max_active_requests:
            raise ValueError(f"Request id {id} is out of range")
        if isinstance(prefilled, TinyKvFullCache) and prefilled.key_values is not None:
            k, _ = prefilled.key_values
            B, H, _, D = k.shape
            assert B == 1
            if self.HD is None:
                self.HD = (H, D)
            else:
                assert self.HD == (H, D)
        self.kv_caches[id] = prefilled

    def remove_request(self, id: int):
        if self.kv_caches[id] is None:
            raise ValueError(f"Request id {id} is not in the cache")
        self.kv_caches[id].release()
        self.kv_caches[id] = None


class TinyKvFullCache(TinyKvCache):
    def __init__(self):
        self.key_values = None
        self.offset = 0

    def update_and_fetch(self, key, value, mask_length=None, mask=None):
        assert key.shape == value.shape
        B, H, S, D = key.shape
        if self.key_values is None:
            assert self.offset == 0
            self.key_values = (key, value)
            self.offset = S
            return key, value, self.offset, mask
        pk, pv = self.key_values
        assert pk.shape == (B, H, self.offset, D)
        nk = torch.cat([pk, key], dim=2)
        nv_ = torch.cat([pv, value], dim=2)
        self.key_values = (nk, nv_)
        self.offset += S
        return nk, nv_, self.offset, mask

    def rewind(self, n: int):
        assert 0 <= n <= self.offset
        self.offset -= n
        if self.offset == 0:
            self.key_values = None
            return
        self.key_values = (self.key_values[0][:, :, :self.offset], self.key_values[1][:, :, :self.offset])
