"""Attention operators with the reference's signatures, running on libnvm_attn.

Mirrors ``src/nano_vllm_metal/layers/attention.py`` of nano-vllm-metal:

* ``paged_attention`` (reference ``attention.py:154-230``): same arguments, same
  mask rules (None or "causal"; an array mask raises NotImplementedError), same
  default scale ``1/sqrt(D)``, same fp32 ``[B, Hq, L, D]`` result.  int8 pages with
  ``key_scales`` / ``value_scales`` are dequantised inside the kernel for every L
  (the reference dequantises the whole pool for L > 1, ``attention.py:204-215``).
* ``flash_attention`` (reference ``attention.py:103-151``): dense attention with
  GQA and an optional additive mask; "causal" never materialises a mask tensor.
* ``causal_mask`` / ``scaled_dot_product_attention_grouped`` (``attention.py:59-100``):
  plain-torch dense references, used by tests and callers that want them.

Extensions (keyword-only, defaults keep the reference behaviour): ``out_dtype``
lets the model receive bf16/fp16 directly instead of casting the fp32 result.
Query tensors are read in their own dtype (fp32, fp16 or bf16); the reference's
``query.astype(float32)`` is exact for 16-bit queries, so it is skipped.
"""

from __future__ import annotations

import torch

from .. import _native as nv

__all__ = [
    "causal_mask",
    "scaled_dot_product_attention_grouped",
    "flash_attention",
    "paged_attention",
]


def causal_mask(L: int, S: int, dtype: torch.dtype = torch.float32, device=None) -> torch.Tensor:
    """0 where key s <= l + (S - L), -inf elsewhere (reference attention.py:59-61)."""
    allowed = torch.ones((L, S), dtype=torch.bool, device=device).tril(diagonal=S - L)
    zero = torch.zeros((), dtype=dtype, device=device)
    ninf = torch.full((), float("-inf"), dtype=dtype, device=device)
    return torch.where(allowed, zero, ninf)


def scaled_dot_product_attention_grouped(query, key, value, scale=None, mask=None):
    """Dense grouped-query SDPA with plain torch ops (reference attention.py:64-100)."""
    expected_shape = query.shape
    Hq, L, D = query.shape[-3:]
    Hkv, S, _ = key.shape[-3:]
    batch = query.shape[:-3]
    assert Hq % Hkv == 0
    rep = Hq // Hkv
    q = query.reshape(*batch, 1, Hkv, rep, L, D)
    k = key.reshape(*batch, 1, Hkv, 1, S, D)
    v = value.reshape(*batch, 1, Hkv, 1, S, D)
    factor = scale if scale is not None else 1.0 / (D ** 0.5)
    scores = torch.matmul(q, k.transpose(-2, -1)) * factor
    if isinstance(mask, str):
        assert mask == "causal"
        scores = scores + causal_mask(L, S, scores.dtype, scores.device)
    elif mask is not None:
        m = torch.broadcast_to(mask, (*batch, Hq, L, S)).reshape(*batch, 1, Hkv, rep, L, S)
        scores = scores + m
    out = torch.matmul(torch.softmax(scores, dim=-1), v)
    return out.reshape(expected_shape)


def flash_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scale: float | None = None,
                    mask: torch.Tensor | str | None = None, *, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Dense flash attention (reference attention.py:103-151).

    query ``[..., Hq, L, E]``, key/value ``[B, Hkv, S, E]`` (fp32, fp16 or bf16, all
    the same dtype).  ``mask`` is None, "causal", or a float tensor broadcastable to
    ``[..., Hq, L, S]`` that is added to the scaled scores.  Returns ``[..., Hq, L, E]``
    in ``out_dtype`` (default: the query dtype, i.e. fp32 for the reference's fp32
    inputs).
    """
    factor = scale if scale is not None else 1.0 / (query.shape[-1] ** 0.5)
    *batch_shape, Hq, L, D = query.shape
    _, Hkv, S, _ = key.shape
    assert Hq % Hkv == 0
    dev = nv.require_cuda("flash_attention", query, key, value)
    if not (query.dtype == key.dtype == value.dtype):
        raise RuntimeError("flash_attention: query, key and value must have the same dtype")
    N = query.numel() // (L * D) if query.numel() else 0
    B = N // Hq
    q = query.contiguous()
    k = key.contiguous()
    v = value.contiguous()
    is_causal = isinstance(mask, str) and mask == "causal"
    if isinstance(mask, str) and mask != "causal":
        raise NotImplementedError(f"flash_attention: unknown mask {mask!r}")
    m = None
    ms = (0, 0, 0)
    if isinstance(mask, torch.Tensor):
        mb = torch.broadcast_to(mask.to(device=dev, dtype=torch.float32), (*batch_shape, Hq, L, S))
        m = mb.reshape(N, L, S)
        ms = m.stride()
    od = out_dtype or query.dtype
    out = torch.empty((*batch_shape, Hq, L, D), dtype=od, device=dev)
    L_ = nv.lib()
    with torch.cuda.device(dev):
        nv.check(L_.nvm_flash_attention(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), nv.dtype_code(q.dtype), nv.ptr(m), ms[0], ms[1], ms[2],
            out.data_ptr(), nv.dtype_code(od), B, Hq, Hkv, L, S, D, float(factor), int(is_causal),
            nv.stream_ptr(dev)))
    return out


def paged_attention(query: torch.Tensor, key_pages: torch.Tensor, value_pages: torch.Tensor,
                    block_table: torch.Tensor, context_lens: torch.Tensor, page_size: int,
                    key_scales: torch.Tensor | None = None, value_scales: torch.Tensor | None = None,
                    scale: float | None = None, mask: torch.Tensor | str | None = None, *,
                    out_dtype: torch.dtype = torch.float32, out: torch.Tensor | None = None) -> torch.Tensor:
    """Paged attention over block-paged K/V pools (reference attention.py:154-230).

    query ``[B, Hq, L, D]``; key_pages/value_pages ``[P, Hkv, page_size, D]`` (fp32,
    fp16, bf16, or int8 with ``key_scales``/``value_scales`` ``[P, Hkv, page_size, 1]``);
    block_table ``[B, max_pages]`` (-1 padded); context_lens ``[B]`` (tokens of each
    sequence, the new L included).  Returns ``[B, Hq, L, D]`` (fp32 by default).
    """
    if isinstance(mask, torch.Tensor):
        raise NotImplementedError("Paged attention only supports mask=None or causal")
    if mask is not None and mask != "causal":
        raise NotImplementedError
    factor = scale if scale is not None else 1.0 / (query.shape[-1] ** 0.5)
    B, Hq, L, D = query.shape
    P, Hkv, ps, _ = key_pages.shape
    assert Hq % Hkv == 0
    dev = nv.require_cuda("paged_attention", query, key_pages, value_pages, block_table, context_lens,
                          key_scales, value_scales)
    if key_pages.dtype != value_pages.dtype:
        raise RuntimeError("paged_attention: key_pages and value_pages must have the same dtype")
    if key_pages.shape != value_pages.shape:
        raise RuntimeError("paged_attention: key_pages and value_pages must have the same shape")
    if key_pages.shape[3] != D:
        raise RuntimeError("paged_attention: q and page tensors must have the same head dimension")
    q = query.contiguous()
    kp = key_pages.contiguous()
    vp = value_pages.contiguous()
    bt = block_table.to(torch.int32).contiguous()
    cl = context_lens.to(torch.int32).contiguous()
    if bt.dim() != 2 or cl.dim() != 1:
        raise RuntimeError("paged_attention: block_table must be 2D and context_lens must be 1D")
    if bt.shape[0] != cl.shape[0] or bt.shape[0] != B:
        raise RuntimeError("paged_attention: q batch size must match block_table batch size")
    ks = vs = None
    sdt = nv.NVM_F16
    if kp.dtype == torch.int8:
        assert key_scales is not None
        assert value_scales is not None
        ks = key_scales.contiguous()
        vs = value_scales.contiguous()
        if ks.dtype != vs.dtype:
            vs = vs.to(ks.dtype)
        sdt = nv.dtype_code(ks.dtype)
    if out is None:
        out = torch.empty((B, Hq, L, D), dtype=out_dtype, device=dev)
    L_ = nv.lib()
    kvc = nv.dtype_code(kp.dtype)
    ws_bytes = L_.nvm_paged_attention_workspace_size(B, Hq, Hkv, L, D, ps, bt.shape[1], kvc)
    ws = nv.workspace(dev, ws_bytes)
    with torch.cuda.device(dev):
        nv.check(L_.nvm_paged_attention(
            q.data_ptr(), nv.dtype_code(q.dtype), kp.data_ptr(), vp.data_ptr(), kvc, nv.ptr(ks), nv.ptr(vs), sdt,
            bt.data_ptr(), cl.data_ptr(), out.data_ptr(), nv.dtype_code(out.dtype), B, Hq, Hkv, L, D, P, ps,
            bt.shape[1], float(factor), int(mask == "causal"), nv.ptr(ws), ws_bytes, nv.stream_ptr(dev)))
    return out
