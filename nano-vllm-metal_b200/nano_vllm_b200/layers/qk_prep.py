"""Fused per-layer attention preparation on the GPU.

``qk_norm_rope_write`` does, in one kernel, what Qwen3Attention.__call__ of the
reference does between the QKV projection and the attention call
(src/nano_vllm_metal/models/qwen3.py:100-116): RMSNorm of every q and k head row
(q_norm / k_norm), RoPE of q and k at each token's position, and the paged write of
the rotated K and the raw V (int8-quantised for int8 pools), returning q in the layout
``paged_attention`` takes.
"""

from __future__ import annotations

import torch

from .. import _native as nv
from .rotary_embedding import RoPE


def _token_rows(x: torch.Tensor) -> tuple[torch.Tensor, int]:
    """[B, L, H, D] -> (tensor whose rows are read in place, elements between tokens).
    Views of a fused QKV projection ([B, L, (Hq + 2 Hkv) * D] split along the last
    axis) keep their token stride and are read without a copy."""
    B, L, H, D = x.shape
    if x.stride(3) == 1 and x.stride(2) == D and (B == 1 or x.stride(0) == L * x.stride(1)) and x.stride(1) >= H * D:
        return x, x.stride(1)
    return x.contiguous(), H * D


def qk_norm_rope_write(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm_weight: torch.Tensor,
                       k_norm_weight: torch.Tensor, rope: RoPE, positions: torch.Tensor, key_pages: torch.Tensor,
                       value_pages: torch.Tensor, slot_mapping: torch.Tensor, *, eps: float = 1e-5,
                       key_scales: torch.Tensor | None = None, value_scales: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """q [B, L, Hq, D], k/v [B, L, Hkv, D] (the projections, f16/bf16); positions [B, L]
    (request offset + index); slot_mapping [B * L] int64 (page_id * page_size + offset,
    negative = skip).  Returns q normalised and rotated, [B, Hq, L, D]; K (normalised,
    rotated) and V are written into key_pages / value_pages [P, Hkv, page_size, D]."""
    nv.require_cuda("qk_norm_rope_write", q, k, v, q_norm_weight, k_norm_weight, positions, key_pages, value_pages,
                    slot_mapping)
    if q.dim() != 4 or k.dim() != 4 or v.shape != k.shape:
        raise RuntimeError("qk_norm_rope_write: q must be [B, L, Hq, D], k and v [B, L, Hkv, D]")
    B, L, Hq, D = q.shape
    Hkv = k.shape[2]
    if k.shape[0] != B or k.shape[1] != L or k.shape[3] != D:
        raise RuntimeError("qk_norm_rope_write: q, k, v disagree on batch, length or head dim")
    if q.dtype != k.dtype or q.dtype != v.dtype or q.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("qk_norm_rope_write: q, k, v must share one dtype, float16 or bfloat16")
    if rope.dims != D:
        raise RuntimeError("qk_norm_rope_write: the RoPE tables are for a different head dim")
    T = B * L
    qc, q_st = _token_rows(q)
    kc, k_st = _token_rows(k)
    vc, v_st = _token_rows(v)
    if k_st != v_st:
        kc, vc = k.contiguous(), v.contiguous()
        k_st = v_st = Hkv * D
    wq = q_norm_weight.to(q.dtype).contiguous()
    wk = k_norm_weight.to(q.dtype).contiguous()
    pos = positions.reshape(T).to(torch.int32).contiguous()
    slots = slot_mapping.reshape(T).to(torch.int64).contiguous()
    cos = rope.cos_freqs.to(q.device).contiguous()
    sin = rope.sin_freqs.to(q.device).contiguous()
    kp, vp = key_pages, value_pages
    P, Hkv_p, ps, D_p = kp.shape
    if Hkv_p != Hkv or D_p != D or vp.shape != kp.shape:
        raise RuntimeError("qk_norm_rope_write: page pools must be [P, Hkv, page_size, D] matching k")
    if not (kp.is_contiguous() and vp.is_contiguous()):
        raise RuntimeError("qk_norm_rope_write: page pools must be contiguous (written in place)")
    if positions.numel() != T or slot_mapping.numel() != T:
        raise RuntimeError("qk_norm_rope_write: positions and slot_mapping need one entry per token")
    int8 = kp.dtype == torch.int8
    if int8:
        if key_scales is None or value_scales is None:
            raise RuntimeError("qk_norm_rope_write: int8 pages need key_scales and value_scales")
        for sc in (key_scales, value_scales):
            if tuple(sc.shape) != (P, Hkv, ps, 1) or not sc.is_contiguous() or not sc.is_floating_point():
                raise RuntimeError("qk_norm_rope_write: scales must be contiguous float [P, Hkv, page_size, 1]")
        if key_scales.dtype != value_scales.dtype:
            raise RuntimeError("qk_norm_rope_write: key and value scales must share one dtype")
    if out is None:
        out = torch.empty((B, Hq, L, D), dtype=q.dtype, device=q.device)
    elif tuple(out.shape) != (B, Hq, L, D) or out.dtype != q.dtype or not out.is_contiguous():
        raise RuntimeError("qk_norm_rope_write: out must be a contiguous [B, Hq, L, D] tensor of q's dtype")
    ks = key_scales if int8 else None
    vs = value_scales if int8 else None
    nv.check(nv.lib().nvm_qk_norm_rope_write(
        qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), nv.dtype_code(q.dtype), q_st, k_st, wq.data_ptr(),
        wk.data_ptr(), float(eps), cos.data_ptr(), sin.data_ptr(), cos.shape[0], 1 if rope.traditional else 0,
        pos.data_ptr(), out.data_ptr(), L, kp.data_ptr(), vp.data_ptr(), nv.dtype_code(kp.dtype),
        ks.data_ptr() if ks is not None else None, vs.data_ptr() if vs is not None else None,
        nv.dtype_code(ks.dtype) if ks is not None else nv.NVM_F16, slots.data_ptr(), T, Hq, Hkv, D, P, ps,
        nv.stream_ptr(q.device)))
    return out
