"""Batched speculative-decoding acceptance on the device.

``verify_accept`` replaces the per-request acceptance loop of the reference's
``speculative_generate`` (src/nano_vllm_metal/engine/generate.py:130-169) for a whole
batch in one kernel launch, and ``DevicePageTable.apply_verify`` turns its result into
one batched rewind of the page tables (rejected suffixes dropped, finished requests
released), so a verify step needs no host round trip.
"""

from __future__ import annotations

from typing import NamedTuple

import torch

from . import _native as nv

__all__ = ["VerifyResult", "verify_accept"]


class VerifyResult(NamedTuple):
    emitted: torch.Tensor       # [B, K1] tokens emitted this step, -1 padded
    n_emitted: torch.Tensor     # [B]
    next_token: torch.Tensor    # [B] the token the next step starts from (-1 once finished)
    rewind: torch.Tensor        # [B] tokens to drop from the target model's cache
    draft_rewind: torch.Tensor  # [B] tokens to drop from the draft model's cache
    finished: torch.Tensor      # [B] 1 when the request ended (end-of-sequence or budget)


def verify_accept(candidates: torch.Tensor, verified: torch.Tensor, eos_id: int | None = None,
                  budget: torch.Tensor | None = None, active: torch.Tensor | None = None) -> VerifyResult:
    """candidates [B, K1]: each request's last accepted token followed by its K1 - 1 draft
    tokens; verified [B, K1]: the target model's argmax at those positions.  budget [B]
    (tokens the request may still emit, < 0 = unlimited) and active [B] (0 = idle slot)
    are optional.  All on one CUDA device; the result stays there."""
    dev = nv.require_cuda("spec_verify_accept", candidates, verified, budget, active)
    if candidates.dim() != 2 or verified.shape != candidates.shape:
        raise RuntimeError("spec_verify_accept: candidates and verified must both be [B, K1]")
    B, K1 = candidates.shape
    i32 = lambda t: None if t is None else t.to(device=dev, dtype=torch.int32).contiguous()  # noqa: E731
    cand, ver, bud, act = i32(candidates), i32(verified), i32(budget), i32(active)
    for name, t in (("budget", bud), ("active", act)):
        if t is not None and t.numel() != B:
            raise RuntimeError(f"spec_verify_accept: {name} must have one entry per request")
    emitted = torch.empty(B, K1, dtype=torch.int32, device=dev)
    outs = [torch.empty(B, dtype=torch.int32, device=dev) for _ in range(5)]
    with torch.cuda.device(dev):
        nv.check(nv.lib().nvm_spec_verify_accept(
            cand.data_ptr(), ver.data_ptr(), B, K1, -1 if eos_id is None else int(eos_id), nv.ptr(bud), nv.ptr(act),
            emitted.data_ptr(), *[o.data_ptr() for o in outs], nv.stream_ptr(dev)))
    return VerifyResult(emitted, *outs)
