"""4-bit (W4A16, group 128) quantized matmul on the GPU.

Mirrors ``layers/linear.py:73-126`` of the reference: ``quantized_matmul(scales, biases,
group_size, bits, a, b, transpose_b)`` with ``b`` the packed weights ``[K, N / 8]``
uint32 (eight 4-bit values per word, element ``n`` in bits ``4 (n % 8)``), scales and
biases ``[K, N / 128]`` in the activation dtype, and ``a`` ``[..., N]``; the result is
``[..., K]``.  ``QuantizedWeights`` / ``quantized_linear`` keep the reference's names.
The kernel is ``nvm_w4a16_matmul`` (tensor-core contraction, fp32 accumulation).
"""

from __future__ import annotations

import torch

from .. import _native as nv


class QuantizedWeights:
    def __init__(self, scales: torch.Tensor, biases: torch.Tensor, group_size: int, bits: int, weight: torch.Tensor):
        self.scales = scales
        self.biases = biases
        self.group_size = group_size
        self.bits = bits
        self.weight = weight


def quantized_matmul(scales: torch.Tensor, biases: torch.Tensor, group_size: int, bits: int, a: torch.Tensor,
                     b: torch.Tensor, transpose_b: bool = False) -> torch.Tensor:
    op = "quantized_matmul"
    nv.require_cuda(op, scales, biases, a, b)
    if scales.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError(f"{op}: scales must be float16 or bfloat16")
    if scales.dtype != biases.dtype:
        raise RuntimeError(f"{op}: scales and biases must be the same dtype")
    if b.dtype not in (torch.int32, torch.uint32):
        raise RuntimeError(f"{op}: b must be uint32")
    if a.dtype != scales.dtype:
        raise RuntimeError(f"{op}: a must be the same dtype as scales")
    if b.dim() != 2:
        raise RuntimeError(f"{op}: b must be a 2D array")
    if bits != 4:
        raise RuntimeError(f"{op}: bits must be 4")
    if group_size != 128:
        raise RuntimeError(f"{op}: group_size must be 128")
    if not transpose_b:
        raise RuntimeError(f"{op}: b must be transposed")
    *lead, N = a.shape
    a2 = a.reshape(-1, N).contiguous()
    M, K = a2.shape[0], b.shape[0]
    if scales.shape != biases.shape:
        raise RuntimeError(f"{op}: scales and biases must have the same shape")
    if scales.shape[0] != K:
        raise RuntimeError(f"{op}: b must have the same number of rows as scales")
    if N % group_size != 0:
        raise RuntimeError(f"{op}: a columns must be divisible by group_size")
    if scales.shape[1] != N // group_size:
        raise RuntimeError(f"{op}: scales must have one column per input group")
    if b.shape[1] != N // 8:
        raise RuntimeError(f"{op}: a must have the same number of columns as b")
    bc, sc, bi = b.contiguous(), scales.contiguous(), biases.contiguous()
    out = torch.empty((M, K), dtype=a.dtype, device=a.device)
    nv.check(nv.lib().nvm_w4a16_matmul(a2.data_ptr(), nv.dtype_code(a.dtype), bc.data_ptr(), sc.data_ptr(),
                                        bi.data_ptr(), out.data_ptr(), M, N, K, group_size, bits,
                                        nv.stream_ptr(a.device)))
    return out.reshape(*lead, K)


def quantized_linear(x: torch.Tensor, w: QuantizedWeights, bias: torch.Tensor | None = None) -> torch.Tensor:
    out = quantized_matmul(w.scales, w.biases, w.group_size, w.bits, x, w.weight, True)
    if bias is not None:
        out = out + bias
    return out
