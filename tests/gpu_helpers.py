"""Shared helpers of the GPU parity tests: torch <-> oracle conversions and random paged problems."""

from __future__ import annotations

import numpy as np
import torch

# North-star tolerance for fp16/bf16 (and int8) attention outputs with fp32 accumulation.
TOL16 = dict(atol=2e-3, rtol=1e-2)
# Reference tolerance for fp32 (tests/utils.py:25-27 of the reference).
TOL32 = dict(atol=1e-6, rtol=1e-5)


def to_np(t: torch.Tensor) -> np.ndarray:
    """Tensor -> numpy; bf16 becomes uint16 bit patterns (the oracle's bf16 form)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def assert_close(got: torch.Tensor, ref: np.ndarray, tol: dict, msg: str = "") -> None:
    g = got.detach().float().cpu().numpy()
    np.testing.assert_allclose(g, ref, err_msg=msg, **tol)


def random_paged_problem(gen: torch.Generator, B, Hq, Hkv, L, D, ps, kv_dtype, ctx_lo, ctx_hi, holes=False,
                         empty=False, spare_pages=3, device="cuda", q_dtype=None):
    """Random pools + block tables (random page permutation), optional holes and an empty row."""
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (B,), generator=gen)
    ctx = torch.maximum(ctx, torch.full_like(ctx, L))
    if empty and B > 1:
        ctx[1] = 0
    pages = [(int(c) + ps - 1) // ps for c in ctx]
    MP = max(max(pages), 1)
    P = sum(pages) + spare_pages
    perm = torch.randperm(P, generator=gen)
    bt = torch.full((B, MP), -1, dtype=torch.int32)
    k = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[k:k + pages[b]].to(torch.int32)
        k += pages[b]
        if holes and pages[b] > 2:
            bt[b, 1] = -1
    if kv_dtype == torch.int8:
        kp = torch.randint(-127, 128, (P, Hkv, ps, D), generator=gen, dtype=torch.int8)
        vp = torch.randint(-127, 128, (P, Hkv, ps, D), generator=gen, dtype=torch.int8)
        ks = (torch.randn(P, Hkv, ps, 1, generator=gen).abs() / 127).to(torch.float16)
        vs = (torch.randn(P, Hkv, ps, 1, generator=gen).abs() / 127).to(torch.float16)
    else:
        kp = torch.randn(P, Hkv, ps, D, generator=gen).to(kv_dtype)
        vp = torch.randn(P, Hkv, ps, D, generator=gen).to(kv_dtype)
        ks = vs = None
    qd = q_dtype or (torch.float16 if kv_dtype == torch.int8 else kv_dtype)
    q = torch.randn(B, Hq, L, D, generator=gen).to(qd)
    dev = torch.device(device)
    mv = lambda t: None if t is None else t.to(dev)  # noqa: E731
    return dict(q=mv(q), kp=mv(kp), vp=mv(vp), ks=mv(ks), vs=mv(vs), bt=mv(bt), cl=mv(ctx.to(torch.int32)), ps=ps)


def oracle_paged(o, prob, mask="causal", scale=None, nthreads=8):
    q = prob["q"].float().cpu().numpy()
    kp, vp = to_np(prob["kp"]), to_np(prob["vp"])
    ks = to_np(prob["ks"]) if prob["ks"] is not None else None
    vs = to_np(prob["vs"]) if prob["vs"] is not None else None
    return o.paged_attention_ref(q, kp, vp, to_np(prob["bt"]), to_np(prob["cl"]), prob["ps"], ks, vs, scale=scale,
                                 mask=mask, kv_is_bf16=prob["kp"].dtype == torch.bfloat16, nthreads=nthreads)
