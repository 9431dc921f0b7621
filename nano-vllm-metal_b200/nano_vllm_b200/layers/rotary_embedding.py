"""RoPE tables and RMSNorm weights for the fused attention-preparation kernel.

``RoPE`` mirrors ``layers/rotary_embedding.py:RoPE`` of the reference (custom backend):
the same constructor arguments, and fp32 cos/sin tables built the same way —
``inv_freq[i] = base ** (-(i / half))``, ``freqs = outer(positions, inv_freq)``,
``cos(freqs)`` / ``sin(freqs)`` (rotary_embedding.py:28-44).  The tables live on the
GPU and are handed to ``qk_norm_rope_write``; ``apply`` is a plain torch restatement
of the reference's ``__call__`` (rotary_embedding.py:74-124) for tests and fallbacks
outside the hot path.
"""

from __future__ import annotations

import torch


class RoPE:
    def __init__(self, dims: int, seq_len: int, base: float = 10000, traditional: bool = False,
                 device: torch.device | str | None = None):
        if dims % 2 != 0:
            raise ValueError("dims must be even")
        self.dims = dims
        self.seq_len = seq_len
        self.base = base
        self.traditional = traditional
        self.half_dims = dims // 2
        positions = torch.arange(seq_len, dtype=torch.float32)
        dim_indices = torch.arange(self.half_dims, dtype=torch.float32)
        inv_freqs = torch.pow(torch.tensor(float(base), dtype=torch.float32), -(dim_indices / self.half_dims))
        freqs = torch.outer(positions, inv_freqs)
        dev = torch.device(device) if device is not None else torch.device("cpu")
        self.cos_freqs = torch.cos(freqs).contiguous().to(dev)
        self.sin_freqs = torch.sin(freqs).contiguous().to(dev)

    def to(self, device) -> "RoPE":
        self.cos_freqs = self.cos_freqs.to(device)
        self.sin_freqs = self.sin_freqs.to(device)
        return self

    def apply(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """x [..., L, H, D] (the reference's [B, L, H, D]) rotated at positions [..., L];
        fp32 math from x's values, result in x.dtype."""
        cos = self.cos_freqs.to(x.device)[positions.long()].unsqueeze(-2)
        sin = self.sin_freqs.to(x.device)[positions.long()].unsqueeze(-2)
        xf = x.float()
        if self.traditional:
            x1, x2 = xf[..., 0::2], xf[..., 1::2]
            out = torch.stack([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).flatten(-2)
        else:
            x1, x2 = xf[..., :self.half_dims], xf[..., self.half_dims:self.dims]
            out = torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)
        return out.to(x.dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """Torch restatement of ``mx.fast.rms_norm`` as used by layers/layernorm.py:4-14:
    x * rsqrt(mean(x^2) + eps) * weight in fp32, result in x.dtype."""
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (xf * inv * weight.float()).to(x.dtype)
