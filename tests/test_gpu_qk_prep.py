"""GPU parity of the fused q/k RMSNorm + RoPE + paged K/V write (nvm_qk_norm_rope_write).

Compared bit for bit with oracle_qk_norm_rope_write (the oracle sums the squares of a
row in the kernel's lane order, so every rounding point is the same), on the same
fp32 RoPE tables.  Shapes follow the Qwen3 models of the reference's benchmarks
(16/8 heads for 0.6B, 32/8 for 4B, d 128; d 64 as the smaller supported head dim).
"""

import os

import numpy as np
import pytest
import torch

from gpu_helpers import to_np
from nano_vllm_b200 import _native as nv
from nano_vllm_b200 import paged_attention
from nano_vllm_b200.layers.qk_prep import qk_norm_rope_write
from nano_vllm_b200.layers.rotary_embedding import RoPE

pytestmark = pytest.mark.gpu

CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2, torch.int8: 3}
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _bf16(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


@pytest.mark.parametrize("name", ["qkprep_bf16", "qkprep_i8_trad"])
def test_golden_qk_prep(cuda, name):
    """The committed fixtures (tests/golden/make_golden.py), bit for bit."""
    d = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    T, Hq, D = d["q"].shape
    Hkv = d["k"].shape[1]
    P, ps, i8 = int(d["P"]), int(d["ps"]), int(d["kv_code"]) == 3
    rope = RoPE(D, d["cos"].shape[0], 1000000, bool(int(d["trad"])), device=cuda)
    rope.cos_freqs = torch.from_numpy(d["cos"]).to(cuda)
    rope.sin_freqs = torch.from_numpy(d["sin"]).to(cuda)
    kv_dtype = torch.int8 if i8 else torch.bfloat16
    kp = torch.zeros(P, Hkv, ps, D, dtype=kv_dtype, device=cuda)
    vp = torch.zeros_like(kp)
    ks = torch.zeros(P, Hkv, ps, 1, dtype=torch.bfloat16, device=cuda) if i8 else None
    vs = None if ks is None else torch.zeros_like(ks)
    out = qk_norm_rope_write(_bf16(d["q"], cuda).reshape(1, T, Hq, D), _bf16(d["k"], cuda).reshape(1, T, Hkv, D),
                             _bf16(d["v"], cuda).reshape(1, T, Hkv, D), _bf16(d["wq"], cuda), _bf16(d["wk"], cuda),
                             rope, torch.from_numpy(d["pos"]).to(cuda).reshape(1, T), kp, vp,
                             torch.from_numpy(d["slots"]).to(cuda), eps=float(d["eps"]), key_scales=ks,
                             value_scales=vs)
    assert nv.device_error(cuda) == 0
    np.testing.assert_array_equal(to_np(out.permute(0, 2, 1, 3).reshape(T, Hq, D)), d["out_q"])
    np.testing.assert_array_equal(to_np(kp), d["out_kp"])
    np.testing.assert_array_equal(to_np(vp), d["out_vp"])
    if i8:
        np.testing.assert_array_equal(to_np(ks), d["out_ks"])
        np.testing.assert_array_equal(to_np(vs), d["out_vs"])


def _problem(seed, B, L, Hq, Hkv, D, dtype, kv_dtype, P, ps, offsets, skip_every=0):
    gen = torch.Generator().manual_seed(seed)
    T = B * L
    q = (torch.randn(B, L, Hq, D, generator=gen) * torch.rand(B, L, Hq, 1, generator=gen) * 8).to(dtype)
    k = (torch.randn(B, L, Hkv, D, generator=gen) * 3).to(dtype)
    v = torch.randn(B, L, Hkv, D, generator=gen).to(dtype)
    wq = torch.empty(D).uniform_(0.5, 1.5, generator=gen).to(dtype)
    wk = torch.empty(D).uniform_(0.5, 1.5, generator=gen).to(dtype)
    pos = torch.stack([torch.arange(o, o + L) for o in offsets]).to(torch.int32)
    slots = torch.randperm(P * ps, generator=gen)[:T].to(torch.int64)
    if skip_every:
        slots[::skip_every] = -1
    if kv_dtype == torch.int8:
        kp = torch.randint(-127, 128, (P, Hkv, ps, D), generator=gen, dtype=torch.int8)
        ks = torch.rand(P, Hkv, ps, 1, generator=gen).to(dtype)
    else:
        kp = torch.randn(P, Hkv, ps, D, generator=gen).to(kv_dtype)
        ks = None
    vp = kp.clone()
    vs = None if ks is None else ks.clone()
    return dict(q=q, k=k, v=v, wq=wq, wk=wk, pos=pos, slots=slots, kp=kp, vp=vp, ks=ks, vs=vs)


def _oracle(oracle, pr, rope, dtype, kv_dtype, eps):
    B, L, Hq, D = pr["q"].shape
    Hkv = pr["k"].shape[2]
    T = B * L
    kp, vp = to_np(pr["kp"]).copy(), to_np(pr["vp"]).copy()
    ks = None if pr["ks"] is None else to_np(pr["ks"]).copy()
    vs = None if pr["vs"] is None else to_np(pr["vs"]).copy()
    q_out, err = oracle.qk_norm_rope_write_ref(
        to_np(pr["q"]).reshape(T, Hq, D), to_np(pr["k"]).reshape(T, Hkv, D), to_np(pr["v"]).reshape(T, Hkv, D),
        CODE[dtype], to_np(pr["wq"]), to_np(pr["wk"]), eps, rope.cos_freqs.cpu().numpy(),
        rope.sin_freqs.cpu().numpy(), rope.traditional, pr["pos"].reshape(T).numpy(), kp, vp, CODE[kv_dtype], ks, vs,
        CODE[dtype], pr["slots"].numpy())
    return q_out, err, kp, vp, ks, vs


def _run_gpu(pr, rope, eps, cuda):
    g = {n: (None if t is None else t.to(cuda)) for n, t in pr.items()}
    out = qk_norm_rope_write(g["q"], g["k"], g["v"], g["wq"], g["wk"], rope, g["pos"], g["kp"], g["vp"], g["slots"],
                             eps=eps, key_scales=g["ks"], value_scales=g["vs"])
    torch.cuda.synchronize()
    return out, g


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("traditional", [False, True], ids=["halves", "traditional"])
@pytest.mark.parametrize("kv", ["same", "int8"])
def test_bit_exact(cuda, oracle, dtype, D, traditional, kv):
    kv_dtype = torch.int8 if kv == "int8" else dtype
    B, L, Hq, Hkv, P, ps, eps = 3, 5, 16, 8, 7, 16, 1e-6
    rope = RoPE(D, 4096, 1000000, traditional, device=cuda)
    pr = _problem(D + traditional, B, L, Hq, Hkv, D, dtype, kv_dtype, P, ps, [0, 100, 4090], skip_every=4)
    out, g = _run_gpu(pr, rope, eps, cuda)
    assert nv.device_error(cuda) == 0
    q_ref, err, kp, vp, ks, vs = _oracle(oracle, pr, rope, dtype, kv_dtype, eps)
    assert err == 0
    got_q = to_np(out.permute(0, 2, 1, 3).reshape(B * L, Hq, D))
    np.testing.assert_array_equal(got_q, q_ref)
    np.testing.assert_array_equal(to_np(g["kp"]), kp)
    np.testing.assert_array_equal(to_np(g["vp"]), vp)
    if kv == "int8":
        np.testing.assert_array_equal(to_np(g["ks"]), ks)
        np.testing.assert_array_equal(to_np(g["vs"]), vs)


def test_fused_projection_views(cuda, oracle):
    """q/k/v as views of one [B, L, (Hq + 2 Hkv) * D] projection are read in place."""
    B, L, Hq, Hkv, D, P, ps, eps = 2, 7, 32, 8, 128, 4, 16, 1e-6
    dtype = torch.bfloat16
    rope = RoPE(D, 64, 1000000, device=cuda)
    pr = _problem(3, B, L, Hq, Hkv, D, dtype, dtype, P, ps, [3, 40])
    qkv = torch.cat([pr["q"].reshape(B, L, -1), pr["k"].reshape(B, L, -1), pr["v"].reshape(B, L, -1)], -1).to(cuda)
    q = qkv[..., :Hq * D].view(B, L, Hq, D)
    k = qkv[..., Hq * D:(Hq + Hkv) * D].view(B, L, Hkv, D)
    v = qkv[..., (Hq + Hkv) * D:].view(B, L, Hkv, D)
    kp, vp = pr["kp"].to(cuda), pr["vp"].to(cuda)
    out = qk_norm_rope_write(q, k, v, pr["wq"].to(cuda), pr["wk"].to(cuda), rope, pr["pos"].to(cuda), kp, vp,
                             pr["slots"].to(cuda), eps=eps)
    q_ref, err, kp_ref, vp_ref, _, _ = _oracle(oracle, pr, rope, dtype, dtype, eps)
    assert err == 0 and nv.device_error(cuda) == 0
    np.testing.assert_array_equal(to_np(out.permute(0, 2, 1, 3).reshape(B * L, Hq, D)), q_ref)
    np.testing.assert_array_equal(to_np(kp), kp_ref)
    np.testing.assert_array_equal(to_np(vp), vp_ref)


@pytest.mark.parametrize("T", [1, 31, 257])
def test_ragged_token_counts(cuda, oracle, T):
    """Row counts that leave the last warp and block partly empty."""
    dtype, D, Hq, Hkv, P, ps, eps = torch.bfloat16, 128, 16, 8, 40, 16, 1e-6
    rope = RoPE(D, 512, 1000000, device=cuda)
    pr = _problem(T, 1, T, Hq, Hkv, D, dtype, dtype, P, ps, [0], skip_every=5)
    out, g = _run_gpu(pr, rope, eps, cuda)
    q_ref, err, kp, vp, _, _ = _oracle(oracle, pr, rope, dtype, dtype, eps)
    assert err == 0 and nv.device_error(cuda) == 0
    np.testing.assert_array_equal(to_np(out.permute(0, 2, 1, 3).reshape(T, Hq, D)), q_ref)
    np.testing.assert_array_equal(to_np(g["kp"]), kp)
    np.testing.assert_array_equal(to_np(g["vp"]), vp)


def test_grid_stride_loop(cuda, oracle):
    """More tokens than resident warps: warps loop over tokens."""
    dtype, D, Hq, Hkv, ps, eps = torch.float16, 64, 4, 2, 16, 1e-6
    T = 9000
    P = (T + ps - 1) // ps + 3
    rope = RoPE(D, 8, 10000, device=cuda)
    pr = _problem(77, 1, T, Hq, Hkv, D, dtype, torch.int8, P, ps, [0], skip_every=13)
    pr["pos"] = (torch.arange(T, dtype=torch.int32) % 8).reshape(1, T)
    out, g = _run_gpu(pr, rope, eps, cuda)
    q_ref, err, kp, vp, ks, vs = _oracle(oracle, pr, rope, dtype, torch.int8, eps)
    assert err == 0 and nv.device_error(cuda) == 0
    np.testing.assert_array_equal(to_np(out.permute(0, 2, 1, 3).reshape(T, Hq, D)), q_ref)
    np.testing.assert_array_equal(to_np(g["kp"]), kp)
    np.testing.assert_array_equal(to_np(g["vp"]), vp)
    np.testing.assert_array_equal(to_np(g["ks"]), ks)
    np.testing.assert_array_equal(to_np(g["vs"]), vs)


def test_out_of_range_position_reports_error(cuda, oracle):
    """A position past the table is skipped and reported through the device error word
    (code 7); the other rows are still written."""
    dtype, D, Hq, Hkv, P, ps, eps = torch.bfloat16, 128, 16, 8, 4, 16, 1e-6
    rope = RoPE(D, 16, 1000000, device=cuda)
    pr = _problem(9, 2, 3, Hq, Hkv, D, dtype, dtype, P, ps, [0, 14])  # positions 14, 15, 16
    nv.device_error(cuda)  # clear
    out, g = _run_gpu(pr, rope, eps, cuda)
    assert nv.device_error(cuda) == 7
    q_ref, err, kp, vp, _, _ = _oracle(oracle, pr, rope, dtype, dtype, eps)
    assert err == 1
    got = to_np(out.permute(0, 2, 1, 3).reshape(6, Hq, D))
    np.testing.assert_array_equal(got[:5], q_ref[:5])
    np.testing.assert_array_equal(to_np(g["vp"]), vp)  # V rows need no position


def test_argument_errors(cuda):
    rope = RoPE(128, 16, device=cuda)
    q = torch.zeros(1, 1, 4, 128, dtype=torch.float32, device=cuda)
    kp = torch.zeros(1, 2, 16, 128, dtype=torch.float32, device=cuda)
    w = torch.ones(128, device=cuda)
    pos = torch.zeros(1, 1, dtype=torch.int32, device=cuda)
    sl = torch.zeros(1, dtype=torch.int64, device=cuda)
    with pytest.raises(RuntimeError, match="float16 or bfloat16"):
        qk_norm_rope_write(q, q[:, :, :2], q[:, :, :2], w, w, rope, pos, kp, kp.clone(), sl)
    qb, kb = q.bfloat16(), torch.zeros(1, 2, 16, 128, dtype=torch.int8, device=cuda)
    with pytest.raises(RuntimeError, match="scales"):
        qk_norm_rope_write(qb, qb[:, :, :2], qb[:, :, :2], w, w, rope, pos, kb, kb.clone(), sl)


@pytest.mark.parametrize("kv", ["bf16", "int8"])
def test_feeds_paged_decode(cuda, oracle, kv):
    """The fused step followed by paged_attention gives the oracle pipeline's output:
    a decode step of 4 sequences whose earlier K/V were written by the same kernel."""
    from gpu_helpers import TOL16

    dtype, D, Hq, Hkv, ps, eps = torch.bfloat16, 128, 16, 8, 16, 1e-6
    kv_dtype = torch.int8 if kv == "int8" else dtype
    B, ctx = 4, [37, 64, 1, 100]
    MP = max((c + ps - 1) // ps for c in ctx)
    P = B * MP
    rope = RoPE(D, 256, 1000000, device=cuda)
    gen = torch.Generator().manual_seed(21)
    kp = torch.zeros(P, Hkv, ps, D, dtype=kv_dtype, device=cuda)
    vp = torch.zeros_like(kp)
    ks = torch.ones(P, Hkv, ps, 1, dtype=dtype, device=cuda) if kv == "int8" else None
    vs = None if ks is None else ks.clone()
    bt = torch.arange(P, dtype=torch.int32).reshape(B, MP)
    wq = torch.empty(D).uniform_(0.5, 1.5, generator=gen).to(dtype).to(cuda)
    wk = torch.empty(D).uniform_(0.5, 1.5, generator=gen).to(dtype).to(cuda)
    # prefill: every token of every sequence but the last, one call per sequence
    for b in range(B):
        n = ctx[b] - 1
        if n == 0:
            continue
        qq = torch.randn(1, n, Hq, D, generator=gen).to(dtype).to(cuda)
        kk = torch.randn(1, n, Hkv, D, generator=gen).to(dtype).to(cuda)
        vv = torch.randn(1, n, Hkv, D, generator=gen).to(dtype).to(cuda)
        pos = torch.arange(n, dtype=torch.int32, device=cuda).reshape(1, n)
        t = torch.arange(n)
        slots = (bt[b, t // ps].long() * ps + t % ps).to(cuda)
        qk_norm_rope_write(qq, kk, vv, wq, wk, rope, pos, kp, vp, slots, eps=eps, key_scales=ks, value_scales=vs)
    # decode step: one token per sequence at position ctx - 1
    qd = torch.randn(B, 1, Hq, D, generator=gen).to(dtype).to(cuda)
    kd = torch.randn(B, 1, Hkv, D, generator=gen).to(dtype).to(cuda)
    vd = torch.randn(B, 1, Hkv, D, generator=gen).to(dtype).to(cuda)
    pos = torch.tensor([[c - 1] for c in ctx], dtype=torch.int32, device=cuda)
    slots = torch.tensor([int(bt[b, (c - 1) // ps]) * ps + (c - 1) % ps for b, c in enumerate(ctx)],
                         dtype=torch.int64, device=cuda)
    kp0, vp0 = kp.clone(), vp.clone()
    ks0 = None if ks is None else ks.clone()
    vs0 = None if vs is None else vs.clone()
    q_rot = qk_norm_rope_write(qd, kd, vd, wq, wk, rope, pos, kp, vp, slots, eps=eps, key_scales=ks, value_scales=vs)
    cl = torch.tensor(ctx, dtype=torch.int32, device=cuda)
    got = paged_attention(q_rot, kp, vp, bt.to(cuda), cl, ps, key_scales=ks, value_scales=vs)
    assert nv.device_error(cuda) == 0
    # oracle pipeline: the fused step on the pre-decode pools, then the paged oracle
    kpn, vpn = to_np(kp0).copy(), to_np(vp0).copy()
    ksn = None if ks0 is None else to_np(ks0).copy()
    vsn = None if vs0 is None else to_np(vs0).copy()
    q_ref, err = oracle.qk_norm_rope_write_ref(
        to_np(qd).reshape(B, Hq, D), to_np(kd).reshape(B, Hkv, D), to_np(vd).reshape(B, Hkv, D), CODE[dtype],
        to_np(wq), to_np(wk), eps, rope.cos_freqs.cpu().numpy(), rope.sin_freqs.cpu().numpy(), False,
        pos.cpu().numpy().reshape(B), kpn, vpn, CODE[kv_dtype], ksn, vsn, CODE[dtype], slots.cpu().numpy())
    assert err == 0
    np.testing.assert_array_equal(to_np(kp), kpn)
    np.testing.assert_array_equal(to_np(vp), vpn)
    q32 = oracle.to_f32(q_ref, CODE[dtype]).reshape(B, Hq, 1, D)
    bt_np, cl_np = bt.numpy(), np.array(ctx, np.int32)
    if kv == "int8":
        ref = oracle.paged_attention_ref(q32, kpn, vpn, bt_np, cl_np, ps, key_scales=ksn, value_scales=vsn,
                                         scales_are_bf16=True)
    else:
        ref = oracle.paged_attention_ref(q32, kpn, vpn, bt_np, cl_np, ps, kv_is_bf16=True)
    np.testing.assert_allclose(got.float().cpu().numpy(), ref, **TOL16)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_int8_v_rounding_ties(cuda, oracle, dtype):
    """V rows are quantised as given: rows whose x / s are exact half-integers must round
    half to even exactly as the oracle's IEEE x / s does."""
    B, L, Hq, Hkv, D, P, ps, eps = 1, 8, 16, 8, 128, 4, 16, 1e-6
    rope = RoPE(D, 4096, 1000000, False, device=cuda)
    pr = _problem(3, B, L, Hq, Hkv, D, dtype, torch.int8, P, ps, [7])
    gen = torch.Generator().manual_seed(5)
    vals = torch.tensor([254.0 / 256] + [(2 * k + 1) / 256 for k in range(127)], dtype=torch.float64)
    sign = torch.where(torch.rand(B, L, Hkv, D, generator=gen) < 0.5, -1.0, 1.0).double()
    pr["v"] = (vals * sign).to(dtype)
    out, g = _run_gpu(pr, rope, eps, cuda)
    _, err, kp, vp, ks, vs = _oracle(oracle, pr, rope, dtype, torch.int8, eps)
    assert err == 0
    np.testing.assert_array_equal(to_np(g["vp"]), vp)
    np.testing.assert_array_equal(to_np(g["vs"]), vs)
    np.testing.assert_array_equal(to_np(g["kp"]), kp)
