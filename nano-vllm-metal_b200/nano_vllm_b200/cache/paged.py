"""Paged KV cache on device memory, mirroring ``src/nano_vllm_metal/cache/paged.py``.

* ``TinyKvPagedPool`` (reference ``paged.py:21-210``): page storage is a device
  tensor ``[capacity, H, page_size, D]`` (int8 + scales ``[capacity, H, page_size, 1]``
  for ``kv_bits=8``).  The free list, reference counts, page-id order and capacity
  growth policy are the reference's, so page ids and pool shapes match it exactly.
  ``reserve_pages`` optionally pre-allocates HBM for that many pages so growth
  becomes a view change instead of a reallocate + copy.
* Writes go through one ``nvm_reshape_and_cache`` launch per append (all pages of
  the chunk at once), in place; int8 quantisation happens in that kernel.
* The reference's ``PrefixCache`` (``paged.py:213-397``) is host bookkeeping that
  touches a pool only through ``page_size``, ``incref``, ``free_page`` and
  ``ref_counts`` and a request cache only through ``offset``, ``num_pages``,
  ``page_ids`` and ``page_lens``; it runs unchanged over these classes.
  ``DevicePageTable.attach`` is its attach step for a whole batch on the device.
* ``TinyKvPagedCache`` (``paged.py:399-559``): per-request page list, append,
  block table, context length, rewind and release.
* ``DevicePageTable``: batch metadata (block table, context lengths, free stack,
  refcounts) kept on the device and extended by ``nvm_paged_append`` without a
  host round trip.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .. import _native as nv
from .kv_cache import TinyKvCache

__all__ = ["PagedKvMetadata", "TinyKvPagedPool", "TinyKvPagedCache", "DevicePageTable",
           "write_slots"]


@dataclass
class PagedKvMetadata:
    key_pages: torch.Tensor
    value_pages: torch.Tensor
    block_table: torch.Tensor
    context_lens: torch.Tensor
    page_size: int
    key_scales: torch.Tensor | None = None
    value_scales: torch.Tensor | None = None
    mask: torch.Tensor | str | None = None


def write_slots(key: torch.Tensor, value: torch.Tensor, slots: torch.Tensor, key_pages: torch.Tensor,
                value_pages: torch.Tensor, key_scales: torch.Tensor | None = None,
                value_scales: torch.Tensor | None = None) -> None:
    """Scatter ``key``/``value`` rows into pages: token t of head h goes to slot[t].

    ``key``/``value`` are ``[T, H, D]`` views (any token/head strides, D contiguous),
    e.g. ``k[0].transpose(0, 1)`` of a ``[1, H, S, D]`` chunk.  ``slots[t]`` is
    ``page_id * page_size + offset`` (< 0 skips the token).
    """
    T, H, D = key.shape
    P, Hp, ps, Dp = key_pages.shape
    assert Hp == H and Dp == D and value.shape == key.shape
    dev = nv.require_cuda("write_page_slice", key, value, slots, key_pages, value_pages, key_scales, value_scales)
    if key.stride(2) != 1:
        key = key.contiguous()
    if value.stride(2) != 1:
        value = value.contiguous()
    if value.stride() != key.stride():
        key, value = key.contiguous(), value.contiguous()
    slots = slots.to(torch.int64).contiguous()
    sdt = nv.dtype_code(key_scales.dtype) if key_scales is not None else nv.NVM_F16
    with torch.cuda.device(dev):
        nv.check(nv.lib().nvm_reshape_and_cache(
            key.data_ptr(), value.data_ptr(), nv.dtype_code(key.dtype), key.stride(0), key.stride(1),
            key_pages.data_ptr(), value_pages.data_ptr(), nv.dtype_code(key_pages.dtype), nv.ptr(key_scales),
            nv.ptr(value_scales), sdt, slots.data_ptr(), T, H, D, P, ps, nv.stream_ptr(dev)))


class TinyKvPagedPool:
    """Model-local physical storage for paged KV (one pool per layer in the model)."""

    def __init__(self, page_size: int = 128, kv_bits: int | None = None, device: torch.device | str | None = None,
                 reserve_pages: int | None = None):
        assert page_size > 0
        if kv_bits is not None and kv_bits != 8:
            raise ValueError("TinyKvPagedPool currently supports only int8 KV")
        self.page_size = page_size
        self.kv_bits = kv_bits
        self.device = torch.device(device) if device is not None else None
        self.reserve_pages = reserve_pages
        self.key_pages: torch.Tensor | None = None
        self.value_pages: torch.Tensor | None = None
        self.key_scales: torch.Tensor | None = None
        self.value_scales: torch.Tensor | None = None
        self._store: tuple | None = None  # reserved backing tensors (k, v, ks, vs)
        self.free_page_ids: list[int] = []
        self.used_page_ids: set[int] = set()
        self.num_allocated_pages = 0
        self.ref_counts: dict[int, int] = {}
        self._capacity = 0  # logical capacity per the growth policy

    @property
    def num_pages(self) -> int:
        return self.num_allocated_pages

    @property
    def num_free_pages(self) -> int:
        return len(self.free_page_ids)

    @property
    def capacity(self) -> int:
        return self._capacity

    def _check_page_chunk(self, x: torch.Tensor) -> None:
        B, H, S, D = x.shape
        assert 0 < S <= self.page_size

    def allocate_page(self) -> int:
        """Pop the most recently freed id, else mint num_pages (reference paged.py:60-70)."""
        if self.free_page_ids:
            page_id = self.free_page_ids.pop()
        else:
            page_id = self.num_pages
            self.num_allocated_pages += 1
        self.used_page_ids.add(page_id)
        self.ref_counts[page_id] = 1
        return page_id

    def incref(self, page_id: int) -> None:
        if page_id not in self.used_page_ids:
            raise ValueError(f"Page {page_id} is free")
        self.ref_counts[page_id] += 1

    def free_page(self, page_id: int) -> None:
        """Drop one reference; the id returns to the free list at zero (paged.py:197-210)."""
        if page_id not in self.used_page_ids:
            raise ValueError(f"Page {page_id} is already free")
        self.ref_counts[page_id] -= 1
        if self.ref_counts[page_id] > 0:
            return
        del self.ref_counts[page_id]
        self.used_page_ids.remove(page_id)
        self.free_page_ids.append(page_id)

    def read_page(self, page_id: int) -> tuple[torch.Tensor, torch.Tensor]:
        if self.key_pages is None or self.value_pages is None:
            raise ValueError(f"Page {page_id} has no storage")
        if page_id >= self.num_pages:
            raise ValueError(f"Page {page_id} is out of range")
        if self.kv_bits == 8:
            return (self.key_pages[page_id:page_id + 1].float() * self.key_scales[page_id:page_id + 1].float(),
                    self.value_pages[page_id:page_id + 1].float() * self.value_scales[page_id:page_id + 1].float())
        return self.key_pages[page_id:page_id + 1], self.value_pages[page_id:page_id + 1]

    # -- capacity -----------------------------------------------------------------
    def _next_capacity(self) -> int:
        """The reference's growth policy (paged.py:109-122), applied per allocation."""
        if self._capacity >= self.num_pages:
            return self._capacity
        if self.num_pages <= 16:
            return self.num_pages
        return max(self.num_pages, self._capacity * 2)

    def _ensure_page_storage(self, key: torch.Tensor) -> None:
        """Grow device storage to the logical capacity (zero pages, unit scales)."""
        B, H, _, D = key.shape
        assert B == 1
        storage_dtype = torch.int8 if self.kv_bits == 8 else key.dtype
        if self.device is None:
            self.device = key.device
        cap = self._capacity
        if self.key_pages is not None:
            assert tuple(self.key_pages.shape[1:]) == (H, self.page_size, D)
            assert self.key_pages.dtype == storage_dtype
            if self.key_pages.shape[0] == cap:
                return
        scale_dtype = key.dtype
        if self.reserve_pages is not None and cap <= self.reserve_pages:
            if self._store is None:
                R = self.reserve_pages
                k = torch.zeros((R, H, self.page_size, D), dtype=storage_dtype, device=self.device)
                v = torch.zeros_like(k)
                ks = vs = None
                if self.kv_bits == 8:
                    ks = torch.ones((R, H, self.page_size, 1), dtype=scale_dtype, device=self.device)
                    vs = torch.ones_like(ks)
                self._store = (k, v, ks, vs)
            k, v, ks, vs = self._store
            self.key_pages, self.value_pages = k[:cap], v[:cap]
            if ks is not None:
                self.key_scales, self.value_scales = ks[:cap], vs[:cap]
            return
        new_k = torch.zeros((cap, H, self.page_size, D), dtype=storage_dtype, device=self.device)
        new_v = torch.zeros_like(new_k)
        if self.key_pages is not None:
            old = self.key_pages.shape[0]
            new_k[:old] = self.key_pages
            new_v[:old] = self.value_pages
        self.key_pages, self.value_pages = new_k, new_v
        if self.kv_bits == 8:
            new_ks = torch.ones((cap, H, self.page_size, 1), dtype=scale_dtype, device=self.device)
            new_vs = torch.ones_like(new_ks)
            if self.key_scales is not None:
                old = self.key_scales.shape[0]
                new_ks[:old] = self.key_scales
                new_vs[:old] = self.value_scales
            self.key_scales, self.value_scales = new_ks, new_vs
        self._store = None

    def grow(self) -> None:
        """Advance the logical capacity after page allocations (bookkeeping only)."""
        self._capacity = self._next_capacity()

    def write_slots(self, key: torch.Tensor, value: torch.Tensor, slots: torch.Tensor) -> None:
        """key/value ``[1, H, S, D]``; slots ``[S]`` absolute slots (page*ps + offset)."""
        self._ensure_page_storage(key)
        write_slots(key[0].transpose(0, 1), value[0].transpose(0, 1), slots, self.key_pages, self.value_pages,
                    self.key_scales, self.value_scales)

    def write_page_slice(self, page_id: int, start: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Write ``key``/``value`` ``[1, H, S, D]`` into slots start..start+S of a page (paged.py:160-195)."""
        assert key.shape == value.shape
        self._check_page_chunk(key)
        if page_id not in self.used_page_ids:
            raise ValueError(f"Page {page_id} is free")
        self.grow()
        S = key.shape[2]
        assert 0 <= start <= self.page_size
        assert start + S <= self.page_size
        base = page_id * self.page_size + start
        slots = torch.arange(base, base + S, dtype=torch.int64, device=key.device)
        self.write_slots(key, value, slots)


class TinyKvPagedCache(TinyKvCache):
    """Layer-local K/V cache of one request, backed by a model-owned page pool."""

    def __init__(self, pool: TinyKvPagedPool):
        self.pool = pool
        self.page_size = pool.page_size
        self.page_ids: list[int] = []
        self.page_lens: list[int] = []
        self.offset = 0

    @property
    def num_pages(self) -> int:
        return len(self.page_ids)

    @property
    def key_values(self):
        if self.offset == 0:
            return None
        return self.gather_dense()

    def plan_append(self, S: int) -> list[int]:
        """Page bookkeeping of appending S tokens (paged.py:424-459); returns their slots.

        Fills the tail page first, then allocates fresh pages in order, growing the
        pool's capacity after every allocation exactly as the reference does.
        """
        ps = self.page_size
        slots: list[int] = []
        start = 0
        if self.page_ids and self.page_lens[-1] < ps:
            pid = self.page_ids[-1]
            page_start = self.page_lens[-1]
            take = min(ps - page_start, S)
            self.pool.grow()
            slots.extend(range(pid * ps + page_start, pid * ps + page_start + take))
            self.page_lens[-1] += take
            start += take
        while start < S:
            end = min(start + ps, S)
            pid = self.pool.allocate_page()
            self.pool.grow()
            slots.extend(range(pid * ps, pid * ps + (end - start)))
            self.page_ids.append(pid)
            self.page_lens.append(end - start)
            start = end
        self.offset += S
        return slots

    def _append_chunk(self, key: torch.Tensor, value: torch.Tensor) -> None:
        assert key.shape == value.shape
        B, H, S, D = key.shape
        assert B == 1, "Paged request cache only supports one request at a time"
        slots = self.plan_append(S)
        self.pool.write_slots(key, value, torch.tensor(slots, dtype=torch.int64).to(key.device, non_blocking=True))

    def gather_dense(self) -> tuple[torch.Tensor, torch.Tensor]:
        assert self.offset > 0
        ks, vs = [], []
        for pid, plen in zip(self.page_ids, self.page_lens):
            kpg, vpg = self.pool.read_page(pid)
            ks.append(kpg[:, :, :plen, :])
            vs.append(vpg[:, :, :plen, :])
        if len(ks) == 1:
            return ks[0], vs[0]
        return torch.cat(ks, dim=2), torch.cat(vs, dim=2)

    def update_and_fetch(self, key, value, mask_length=None, mask=None):
        assert key.shape == value.shape
        self._append_chunk(key, value)
        dk, dv = self.gather_dense()
        return dk, dv, self.offset, mask

    def block_table(self, max_pages: int | None = None) -> torch.Tensor:
        if max_pages is None:
            max_pages = self.num_pages
        assert max_pages >= self.num_pages
        row = self.page_ids + [-1] * (max_pages - self.num_pages)
        return torch.tensor([row], dtype=torch.int32).to(self.pool.device or "cuda", non_blocking=True)

    def context_lens(self) -> torch.Tensor:
        return torch.tensor([self.offset], dtype=torch.int32).to(self.pool.device or "cuda", non_blocking=True)

    def paged_metadata(self, max_pages: int | None = None, mask=None) -> PagedKvMetadata:
        assert self.pool.key_pages is not None
        assert self.pool.value_pages is not None
        return PagedKvMetadata(
            key_pages=self.pool.key_pages, value_pages=self.pool.value_pages,
            key_scales=self.pool.key_scales, value_scales=self.pool.value_scales,
            block_table=self.block_table(max_pages=max_pages), context_lens=self.context_lens(),
            page_size=self.page_size, mask=mask)

    def update_and_fetch_paged(self, key, value, mask_length=None, mask=None) -> PagedKvMetadata:
        assert key.shape == value.shape
        self._append_chunk(key, value)
        return self.paged_metadata(mask=mask)

    def rewind(self, n: int) -> None:
        assert 0 <= n <= self.offset
        new_offset = self.offset - n
        if new_offset == self.offset:
            return
        if new_offset == 0:
            self.release()
            return
        target = (new_offset + self.page_size - 1) // self.page_size
        while len(self.page_ids) > target:
            pid = self.page_ids.pop()
            self.page_lens.pop()
            self.pool.free_page(pid)
        self.page_lens[-1] = new_offset - self.page_size * (target - 1)
        self.offset = new_offset

    def release(self) -> None:
        for pid in self.page_ids:
            self.pool.free_page(pid)
        self.page_ids.clear()
        self.page_lens.clear()
        self.offset = 0


class DevicePageTable:
    """Device-resident batch metadata extended by ``nvm_paged_append``.

    Holds ``block_table [B, max_pages]`` (-1 padded), ``context_lens [B]``, a LIFO
    ``free_stack`` with ``free_top``, ``num_pages`` (ids minted so far) and per-page
    ``refcount`` for a pool of ``capacity`` pages.  ``append(new_tokens)`` extends
    every request at once on the device and returns the slot of each new token, in
    request order -- the ids and slots the reference's sequential ``_append_chunk``
    loop would produce (``kv_cache.py:134-151``, ``paged.py:424-459``).
    """

    def __init__(self, batch: int, max_pages: int, page_size: int, capacity: int, device="cuda"):
        self.device = torch.device(device)
        self.B, self.max_pages, self.page_size, self.capacity = batch, max_pages, page_size, capacity
        i32 = dict(dtype=torch.int32, device=self.device)
        self.block_table = torch.full((batch, max_pages), -1, **i32)
        self.context_lens = torch.zeros(batch, **i32)
        self.free_stack = torch.zeros(max(capacity, 1), **i32)
        self.free_top = torch.zeros(1, **i32)
        self.num_pages = torch.zeros(1, **i32)
        self.refcount = torch.zeros(max(capacity, 1), **i32)
        self.last_call = torch.full((max(capacity, 1),), -1, **i32)  # rewind scratch, kept at -1
        self.status = torch.zeros(1, **i32)

    def append(self, new_tokens: torch.Tensor, slot_mapping: torch.Tensor | None = None) -> torch.Tensor:
        """new_tokens ``[B]`` int32 on the device; returns int64 slots ``[sum(new_tokens)]``.

        ``slot_mapping`` (optional) is a preallocated int64 buffer at least that long;
        without it the host needs the total, so the call synchronises once.
        """
        nt = new_tokens.to(device=self.device, dtype=torch.int32).contiguous()
        if slot_mapping is None:
            slot_mapping = torch.empty(int(nt.sum().item()), dtype=torch.int64, device=self.device)
        with torch.cuda.device(self.device):
            nv.check(nv.lib().nvm_paged_append(
                self.block_table.data_ptr(), self.context_lens.data_ptr(), nt.data_ptr(), self.free_stack.data_ptr(),
                self.free_top.data_ptr(), self.num_pages.data_ptr(), self.refcount.data_ptr(),
                slot_mapping.data_ptr(), slot_mapping.numel(), self.status.data_ptr(), self.B, self.max_pages,
                self.page_size,
                self.capacity, nv.stream_ptr(self.device)))
        return slot_mapping

    def rewind(self, n_tokens: torch.Tensor) -> None:
        """Drop ``n_tokens[b]`` tokens from the end of every request at once on the device:
        the reference's ``TinyKvPagedCache.rewind`` for b = 0..B-1 in order
        (``paged.py:530-550``; dropping a request's whole length is ``release``,
        ``paged.py:552-559``).  Pages past the new lengths lose a reference and return to
        the free stack, in the reference's order, when their count reaches zero."""
        n = n_tokens.to(device=self.device, dtype=torch.int32).contiguous()
        with torch.cuda.device(self.device):
            nv.check(nv.lib().nvm_paged_rewind(
                self.block_table.data_ptr(), self.context_lens.data_ptr(), n.data_ptr(), self.free_stack.data_ptr(),
                self.free_top.data_ptr(), self.refcount.data_ptr(), self.last_call.data_ptr(),
                self.status.data_ptr(), self.B, self.max_pages, self.page_size, self.capacity,
                nv.stream_ptr(self.device)))

    def release(self, mask: torch.Tensor | None = None) -> None:
        """Release requests (all, or those where ``mask`` is true): rewind by their length."""
        n = self.context_lens.clone()
        if mask is not None:
            n = torch.where(mask.to(device=self.device, dtype=torch.bool), n, torch.zeros_like(n))
        self.rewind(n)

    def apply_verify(self, result) -> None:
        """After a batched speculative verify step (``spec_verify.verify_accept``): drop
        each request's rejected suffix (``result.rewind``) and release the requests that
        finished, in one batched rewind on the device -- the reference's per-request
        ``rewind`` (``engine/generate.py:147-153``, ``paged.py:530-550``) and the release
        of finished requests."""
        fin = result.finished.to(device=self.device, dtype=torch.bool)
        self.rewind(torch.where(fin, self.context_lens, result.rewind.to(device=self.device, dtype=torch.int32)))

    def attach(self, pages: torch.Tensor, count: torch.Tensor) -> None:
        """``PrefixCache.attach`` on the device (``paged.py:305-328``): fresh request b
        takes the shared full pages ``pages[b, :count[b]]`` (each gains a reference) and
        starts at length ``count[b] * page_size``."""
        pg = pages.to(device=self.device, dtype=torch.int32).contiguous()
        ct = count.to(device=self.device, dtype=torch.int32).contiguous()
        if pg.dim() != 2 or pg.shape[0] != self.B or ct.numel() != self.B:
            raise ValueError("attach: pages must be [B, max_prefix] and count [B]")
        with torch.cuda.device(self.device):
            nv.check(nv.lib().nvm_paged_attach(
                self.block_table.data_ptr(), self.context_lens.data_ptr(), pg.data_ptr(), ct.data_ptr(),
                self.refcount.data_ptr(), self.status.data_ptr(), self.B, self.max_pages, self.page_size,
                pg.shape[1], self.capacity, nv.stream_ptr(self.device)))

    def free_list(self) -> list[int]:
        """The free stack bottom to top (the next page taken is the last entry)."""
        return self.free_stack[: int(self.free_top.item())].tolist()

    def check_status(self) -> None:
        st = int(self.status.item())
        if st != 0:
            raise RuntimeError(f"page table: device call failed (status {st}: out of pages, block-table row full, "
                               "or an invalid rewind / attach)")
