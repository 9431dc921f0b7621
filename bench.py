"""Benchmark of the B200 attention hot path (decode KV GB/s, prefill TFLOPS).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N ...

Headline workload (``config.workload``): BASELINE config 3, paged decode with prefix
sharing, Qwen3-4B attention shape (32 q / 8 kv heads, d=128, bf16 pages, page 16),
batch 256, context lengths uniform in [4096, 32768], the first 1024 tokens of each
16-sequence group on shared physical pages, the other pages randomly permuted.  A
step is one ``paged_attention`` call over the whole batch (inputs resident in HBM,
19 GB of K/V, far larger than L2, so no flush is needed between steps).  With N
GPUs every rank owns Hkv/N kv heads and their pools (KV-head sharding, no
collective in the timed region); ``value`` = logical K/V+Q/O+metadata bytes of all
ranks / max-over-ranks time (strong scaling: the job is fixed as N grows).

Secondary lines (N=1 only) time configs 1, 4, 5 (decode GB/s), 2a / 2b (prefill
TFLOPS) and the fused q/k-norm + RoPE + K/V write at the 2a token count (GB/s) one
launch at a time with an L2 flush between launches, the per-decode-step batch metadata
path (host wall time, device tables vs per-request host bookkeeping) and the W4A16
matmul at Qwen3-4B's MLP shapes (GB/s).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nano-vllm-metal_b200"))
sys.path.insert(0, ROOT)

HBM_FALLBACK_GBS = 6650.0
BF16_FALLBACK_TFLOPS = 1590.0


# ---------------------------------------------------------------------------
# workloads (all synthetic, seeded)
# ---------------------------------------------------------------------------

def decode_config(name: str) -> dict:
    if name == "c1":
        return dict(B=16, Hq=16, Hkv=8, L=1, D=128, ps=16, dtype=torch.float16, ctx=("uniform", 128, 1024),
                    share=None, model="Qwen3-0.6B")
    if name == "c3":
        return dict(B=256, Hq=32, Hkv=8, L=1, D=128, ps=16, dtype=torch.bfloat16, ctx=("uniform", 4096, 32768),
                    share=(16, 1024), model="Qwen3-4B")
    if name == "c4":
        return dict(B=64, Hq=64, Hkv=8, L=1, D=128, ps=16, dtype=torch.int8, ctx=("uniform", 8192, 32768),
                    share=None, model="Qwen3-32B")
    if name == "c5":
        return dict(B=128, Hq=32, Hkv=4, L=5, D=128, ps=16, dtype=torch.bfloat16,
                    ctx=("lognormal", math.log(2048), 1.0, 256, 16384), share=None, model="Qwen3-30B-A3B")
    raise ValueError(name)


def sample_context_lens(cfg: dict, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    spec = cfg["ctx"]
    if spec[0] == "uniform":
        return rng.integers(spec[1], spec[2] + 1, size=cfg["B"]).astype(np.int64)
    mu, sigma, lo, hi = spec[1:]
    return np.clip(np.rint(rng.lognormal(mu, sigma, size=cfg["B"])), lo, hi).astype(np.int64)


def block_tables(cfg: dict, ctx: np.ndarray, seed: int):
    """Block tables over a pool of (unique pages + 64 spare), randomly permuted.

    With ``share=(group, tokens)`` the first tokens/page_size pages of every group of
    `group` sequences are the same physical pages (refcounted shared prefix).
    """
    rng = np.random.default_rng(seed + 1)
    ps, B = cfg["ps"], cfg["B"]
    n_pages = (ctx + ps - 1) // ps
    MP = int(n_pages.max())
    shared = 0
    if cfg["share"] is not None:
        group, tokens = cfg["share"]
        shared = tokens // ps
        n_groups = (B + group - 1) // group
        P = n_groups * shared + int((n_pages - shared).sum()) + 64
    else:
        P = int(n_pages.sum()) + 64
    perm = rng.permutation(P).astype(np.int32)
    bt = np.full((B, MP), -1, dtype=np.int32)
    k = 0
    if shared:
        group = cfg["share"][0]
        for g0 in range(0, B, group):
            pref = perm[k:k + shared]
            k += shared
            for b in range(g0, min(B, g0 + group)):
                bt[b, :shared] = pref
    for b in range(B):
        rest = int(n_pages[b]) - shared
        bt[b, shared:shared + rest] = perm[k:k + rest]
        k += rest
    return bt, P


def decode_bytes(cfg: dict, ctx: np.ndarray, n_kv: int, n_q: int, out_bytes: int = 4) -> dict:
    """Algorithmic bytes of one decode call (logical K/V per kv head, Q, O, metadata)."""
    D, ps, L = cfg["D"], cfg["ps"], cfg["L"]
    if cfg["dtype"] == torch.int8:
        kv = int(ctx.sum()) * n_kv * (D * 2 * 1 + 2 * 2)  # int8 K+V + fp16 K/V scales per token
        qb = 2
    else:
        e = 2
        kv = int(ctx.sum()) * n_kv * D * 2 * e
        qb = e
    q = len(ctx) * n_q * L * D * qb
    o = len(ctx) * n_q * L * D * out_bytes
    meta = int(((ctx + ps - 1) // ps).sum()) * 4 + 4 * len(ctx)
    return dict(kv=kv, q=q, o=o, meta=meta, total=kv + q + o + meta)


def build_decode(cfg: dict, rank: int, world: int, device, seed: int = 0):
    from nano_vllm_b200.sharding import kv_head_shard

    ctx = sample_context_lens(cfg, seed)
    bt, P = block_tables(cfg, ctx, seed)
    sh = kv_head_shard(rank, world, cfg["Hq"], cfg["Hkv"], cfg["B"])
    b_lo, b_hi = sh.b_lo, sh.b_hi
    gen = torch.Generator(device=device)
    gen.manual_seed(seed * 1000 + rank)
    shape = (P, sh.num_kv_heads, cfg["ps"], cfg["D"])
    if cfg["dtype"] == torch.int8:
        kp = torch.randint(-127, 128, shape, generator=gen, device=device, dtype=torch.int8)
        vp = torch.randint(-127, 128, shape, generator=gen, device=device, dtype=torch.int8)
        ks = (torch.randn(shape[:3] + (1,), generator=gen, device=device).abs_() / 127).to(torch.float16)
        vs = (torch.randn(shape[:3] + (1,), generator=gen, device=device).abs_() / 127).to(torch.float16)
        qd = torch.float16
    else:
        kp = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(cfg["dtype"])
        vp = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(cfg["dtype"])
        ks = vs = None
        qd = cfg["dtype"]
    Bl = b_hi - b_lo
    q = torch.randn((Bl, sh.num_q_heads, cfg["L"], cfg["D"]), generator=gen, device=device).to(qd)
    bt_t = torch.from_numpy(bt[b_lo:b_hi]).to(device)
    cl_t = torch.from_numpy(ctx[b_lo:b_hi].astype(np.int32)).to(device)
    nbytes = decode_bytes(cfg, ctx[b_lo:b_hi], sh.num_kv_heads, sh.num_q_heads)
    return dict(q=q, kp=kp, vp=vp, ks=ks, vs=vs, bt=bt_t, cl=cl_t, ps=cfg["ps"], ctx=ctx, bt_np=bt, P=P,
                shard=sh, bytes=nbytes)


# ---------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------

def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return dict(hbm=float(d["hbm_gbs"]), bf16=float(d["bf16_tflops"]),
                    bf16_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), src="measured")
    return dict(hbm=HBM_FALLBACK_GBS, bf16=BF16_FALLBACK_TFLOPS, bf16_sustained=1400.0, src="fallback")


def ncu_traffic(key: str):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get(key)
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples taken while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = f"/tmp/nvm_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.remove(self.path)
        loaded = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


def flush_l2(buf: torch.Tensor):
    # Read (not write) > L2 (126 MB): evicts the previous launch's lines without
    # leaving dirty lines whose write-back would be charged to the next launch.
    buf.view(torch.int32).sum(dtype=torch.int32)


def time_launches(fn, iters: int, warmup: int, flush_buf=None) -> list[float]:
    """Per-launch device ms with CUDA events on the current stream (L2 flushed between)."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        if flush_buf is not None:
            flush_l2(flush_buf)
        # keep the GPU busy (~200 us) while the host queues the start event and the
        # launch, so host-side delays never show up as idle time inside the events
        torch.cuda._sleep(400_000)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e))
    return times


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_decode_step(w):
    from nano_vllm_b200 import paged_attention

    return paged_attention(w["q"], w["kp"], w["vp"], w["bt"], w["cl"], w["ps"], w["ks"], w["vs"], mask="causal")


def e2e_decode(w, steps: int, warmup: int):
    """Same step through the public API from pinned host buffers, with every step's H2D
    copy of its inputs and D2H copy of its result inside the timed region.  As a serving
    loop would, the copies run on two side streams and overlap the neighbouring steps'
    compute (inputs and outputs double-buffered, ordered by events)."""
    from nano_vllm_b200 import paged_attention

    q_h = w["q"].cpu().pin_memory()
    bt_h = w["bt"].cpu().pin_memory()
    cl_h = w["cl"].cpu().pin_memory()
    out_h = [torch.empty(w["q"].shape, dtype=torch.float32).pin_memory() for _ in range(2)]
    dev = w["q"].device
    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    q_d = [torch.empty_like(w["q"]) for _ in range(2)]
    bt_d = [torch.empty_like(w["bt"]) for _ in range(2)]
    cl_d = [torch.empty_like(w["cl"]) for _ in range(2)]
    out_d = [torch.empty(w["q"].shape, dtype=torch.float32, device=dev) for _ in range(2)]
    ev = lambda: torch.cuda.Event()  # noqa: E731
    h2d_done = [ev() for _ in range(2)]
    comp_done = [ev() for _ in range(2)]
    d2h_done = [ev() for _ in range(2)]
    for e_ in comp_done + d2h_done:
        e_.record(comp)

    def step(i):
        sl = i & 1
        with torch.cuda.stream(up):
            up.wait_event(comp_done[sl])  # step i-2 has finished reading this slot
            q_d[sl].copy_(q_h, non_blocking=True)
            bt_d[sl].copy_(bt_h, non_blocking=True)
            cl_d[sl].copy_(cl_h, non_blocking=True)
            h2d_done[sl].record(up)
        comp.wait_event(h2d_done[sl])
        comp.wait_event(d2h_done[sl])  # step i-2's result has left this output slot
        paged_attention(q_d[sl], w["kp"], w["vp"], bt_d[sl], cl_d[sl], w["ps"], w["ks"], w["vs"], mask="causal",
                        out=out_d[sl])
        comp_done[sl].record(comp)
        with torch.cuda.stream(down):
            down.wait_event(comp_done[sl])
            out_h[sl].copy_(out_d[sl], non_blocking=True)
            d2h_done[sl].record(down)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(comp)
    up.wait_stream(comp)
    for i in range(steps):
        step(i)
    comp.wait_stream(down)
    e.record(comp)
    e.synchronize()
    ms = s.elapsed_time(e) / steps
    h2d = q_h.numel() * q_h.element_size() + bt_h.numel() * 4 + cl_h.numel() * 4
    d2h = out_h[0].numel() * 4
    return ms, h2d, d2h


def cpu_baseline_decode(cfg: dict, w: dict | None, target_s: float = 10.0):
    """The oracle (reference eval_cpu restated) on a bounded sample of the same workload.

    Sequences are drawn from the workload's context-length distribution; their K/V
    pages (same dtype and distribution as the GPU run) are generated once on the
    host for the longest sampled context and reused, so generation stays outside the
    timed calls.
    """
    # OpenMP worker threads must sleep, not spin, once the sample is done: spinning
    # threads on every core delay the host's kernel launches in the GPU timings after it
    os.environ.setdefault("OMP_WAIT_POLICY", "PASSIVE")
    from oracle import oracle as o

    nthreads = o.max_threads()
    ctx_all = w["ctx"] if w is not None else sample_context_lens(cfg, 0)
    rng = np.random.default_rng(99)
    D, H, Hq, ps, L = cfg["D"], cfg["Hkv"], cfg["Hq"], cfg["ps"], cfg["L"]
    picks = rng.integers(0, cfg["B"], size=cfg["B"])
    npg_max = int((ctx_all.max() + ps - 1) // ps)
    if cfg["dtype"] == torch.int8:
        kp = rng.integers(-127, 128, (npg_max, H, ps, D), dtype=np.int8)
        vp = rng.integers(-127, 128, (npg_max, H, ps, D), dtype=np.int8)
        ks = (np.abs(rng.standard_normal((npg_max, H, ps, 1))) / 127).astype(np.float16)
        vs = (np.abs(rng.standard_normal((npg_max, H, ps, 1))) / 127).astype(np.float16)
        bf16 = False
    else:
        kp = rng.standard_normal((npg_max, H, ps, D), dtype=np.float32)
        vp = rng.standard_normal((npg_max, H, ps, D), dtype=np.float32)
        bf16 = cfg["dtype"] == torch.bfloat16
        kp = o.f32_to_bf16_bits(kp) if bf16 else kp.astype(np.float16)
        vp = o.f32_to_bf16_bits(vp) if bf16 else vp.astype(np.float16)
        ks = vs = None
    total_time, total_bytes, used = 0.0, 0, 0
    for b in picks:
        ctx = ctx_all[b:b + 1].astype(np.int32)
        npg = int((ctx[0] + ps - 1) // ps)
        bt = np.arange(npg, dtype=np.int32)[None]
        q = rng.standard_normal((1, Hq, L, D)).astype(np.float32)
        t0 = time.perf_counter()
        o.paged_attention_ref(q, kp[:npg], vp[:npg], bt, ctx, ps, None if ks is None else ks[:npg],
                              None if vs is None else vs[:npg], mask="causal", kv_is_bf16=bf16, nthreads=nthreads)
        total_time += time.perf_counter() - t0
        total_bytes += decode_bytes(cfg, ctx.astype(np.int64), H, Hq)["total"]
        used += 1
        if total_time > target_s:
            break
    return dict(value=total_bytes / total_time / 1e9, unit="GB/s", cores=nthreads, kind="port",
                sample=f"{used} sequences (all {Hq} q heads each) of {cfg.get('name', '')}, oracle restatement "
                       f"of PagedAttention::eval_cpu with OpenMP over query rows, {total_time:.1f}s",
                seconds=total_time)


def secondary_results(peaks: dict, device) -> list[dict]:
    from nano_vllm_b200 import flash_attention, paged_attention

    res = []
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for name in ["c1", "c4", "c5"]:
        cfg = decode_config(name)
        w = build_decode(cfg, 0, 1, device)
        ms = statistics.median(time_launches(lambda: run_decode_step(w), 20, 3, flush))
        gbs = w["bytes"]["total"] / (ms * 1e-3) / 1e9
        res.append(dict(workload=f"config{name[1]} decode {cfg['model']}", metric="decode-attn KV GB/s",
                        value=round(gbs, 1), unit="GB/s", ms=round(ms, 4),
                        roofline_frac=round(gbs / peaks["hbm"], 4), l2="flushed"))
        del w
        torch.cuda.empty_cache()
    # 2a: dense causal prefill, 4 x 2048, 32/8 heads, bf16
    gen = torch.Generator(device=device)
    gen.manual_seed(5)
    B, Hq, Hkv, L, D = 4, 32, 8, 2048, 128
    q = torch.randn(B, Hq, L, D, generator=gen, device=device).bfloat16()
    k = torch.randn(B, Hkv, L, D, generator=gen, device=device).bfloat16()
    v = torch.randn(B, Hkv, L, D, generator=gen, device=device).bfloat16()
    flops = 4 * D * Hq * B * (L * (L + 1) // 2)
    ms = statistics.median(time_launches(lambda: flash_attention(q, k, v, mask="causal", out_dtype=torch.bfloat16),
                                         10, 3, flush))
    tf = flops / (ms * 1e-3) / 1e12
    res.append(dict(workload="config2a dense causal prefill Qwen3-4B 4x2048", metric="prefill attn TFLOPS",
                    value=round(tf, 1), unit="TFLOP/s", ms=round(ms, 4), roofline_frac=round(tf / peaks["bf16"], 4)))
    # 2b: chunked prefill, 512-token chunk against c tokens of paged context
    for c in [0, 1024, 4096]:
        cfg = dict(B=4, Hq=32, Hkv=8, L=512, D=128, ps=16, dtype=torch.bfloat16, ctx=("uniform", c + 512, c + 512),
                   share=None)
        w = build_decode(cfg, 0, 1, device)
        flops = 4 * D * Hq * 4 * sum(c + r + 1 for r in range(512))
        ms = statistics.median(time_launches(lambda: run_decode_step(w), 10, 3, flush))
        tf = flops / (ms * 1e-3) / 1e12
        res.append(dict(workload=f"config2b chunked prefill 512 vs {c} paged", metric="prefill attn TFLOPS",
                        value=round(tf, 1), unit="TFLOP/s", ms=round(ms, 4),
                        roofline_frac=round(tf / peaks["bf16"], 4)))
        del w
    res.extend(qk_prep_results(peaks, device, flush))
    res.append(metadata_results(device))
    res.append(decode_step_results(device))
    res.extend(w4a16_results(peaks, device, flush))
    return res


def w4a16_results(peaks: dict, device, flush, shapes=(("gate_up", 2 * 9728, 2560), ("down", 2560, 9728)),
                  ms_rows=(1, 8), iters: int = 20, warmup: int = 3) -> list[dict]:
    """Secondary lines: W4A16 (4-bit, group 128) matmul at Qwen3-4B's decode shapes
    (gate+up projection K = 2 x 9728, N = 2560; down projection K = 2560, N = 9728),
    M = 1 and 8 activation rows, bf16; GB/s of weights + scales + biases + activations."""
    from nano_vllm_b200.layers.linear import quantized_matmul

    res = []
    gen = torch.Generator(device=device)
    gen.manual_seed(11)
    for name, K, N in shapes:
        w = torch.randint(-2 ** 31, 2 ** 31 - 1, (K, N // 8), generator=gen, dtype=torch.int64,
                          device=device).to(torch.int32)
        s = (torch.rand(K, N // 128, generator=gen, device=device) * 0.02).bfloat16()
        b = (torch.rand(K, N // 128, generator=gen, device=device) * -0.1).bfloat16()
        for M in ms_rows:
            a = torch.randn(M, N, generator=gen, device=device).bfloat16()
            nbytes = K * N // 2 + 2 * K * (N // 128) * 2 + M * N * 2 + M * K * 2
            ms = statistics.median(time_launches(lambda: quantized_matmul(s, b, 128, 4, a, w, True), iters, warmup,
                                                 flush))
            gbs = nbytes / (ms * 1e-3) / 1e9
            res.append(dict(workload=f"W4A16 matmul {name} Qwen3-4B (K={K}, N={N}), M={M}, bf16",
                            metric="w4a16 GB/s", value=round(gbs, 1), unit="GB/s", ms=round(ms, 4), bytes=nbytes,
                            roofline_frac=round(gbs / peaks["hbm"], 4), l2="flushed"))
        del w, s, b
    return res


def decode_step_results(device, layers: int = 36, B: int = 64, ctx: int = 1024, steps: int = 20) -> dict:
    """Secondary line: the attention path of one decode step of a Qwen3-4B-shaped model
    (36 layers, 32 q / 8 kv heads, d 128, bf16, page 16), B requests of ctx tokens, host
    wall time per step: DevicePageTable.append once, then per layer the fused q/k norm +
    RoPE + K/V write and paged attention, with the metadata on the device throughout --
    launched eagerly, and as one CUDA graph replayed per step."""
    from nano_vllm_b200 import DevicePageTable, paged_attention
    from nano_vllm_b200.layers.qk_prep import qk_norm_rope_write
    from nano_vllm_b200.layers.rotary_embedding import RoPE

    Hq, Hkv, D, ps = 32, 8, 128, 16
    gen = torch.Generator(device=device)
    gen.manual_seed(17)
    mp = (ctx + 3 * (steps + 4) + ps - 1) // ps + 1
    cap = B * mp + 16
    table = DevicePageTable(B, mp, ps, cap, device=device)
    table.append(torch.full((B,), ctx, dtype=torch.int32, device=device))
    table.check_status()
    pools = [(torch.randn(cap, Hkv, ps, D, generator=gen, device=device).bfloat16(),
              torch.randn(cap, Hkv, ps, D, generator=gen, device=device).bfloat16()) for _ in range(layers)]
    qkv = torch.randn(layers, B, 1, (Hq + 2 * Hkv) * D, generator=gen, device=device).bfloat16()
    wq = (torch.rand(D, generator=gen, device=device) + 0.5).bfloat16()
    wk = (torch.rand(D, generator=gen, device=device) + 0.5).bfloat16()
    rope = RoPE(D, 40960, 1000000, device=device)
    ones = torch.ones(B, dtype=torch.int32, device=device)
    slots = torch.empty(B, dtype=torch.int64, device=device)

    def step():
        table.append(ones, slot_mapping=slots)
        pos = (table.context_lens - 1).view(B, 1)
        for li in range(layers):
            x = qkv[li]
            q = x[..., :Hq * D].view(B, 1, Hq, D)
            k = x[..., Hq * D:(Hq + Hkv) * D].view(B, 1, Hkv, D)
            v = x[..., (Hq + Hkv) * D:].view(B, 1, Hkv, D)
            kp, vp = pools[li]
            qr = qk_norm_rope_write(q, k, v, wq, wk, rope, pos, kp, vp, slots, eps=1e-6)
            paged_attention(qr, kp, vp, table.block_table, table.context_lens, ps, out_dtype=torch.bfloat16)

    def eager():
        step()
        torch.cuda.synchronize()

    for _ in range(3):
        eager()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()

    def replay():
        graph.replay()
        torch.cuda.synchronize()

    out = {}
    for name, fn in (("eager", eager), ("graph", replay)):
        fn()
        t0 = time.perf_counter()
        for _ in range(steps):
            fn()
        out[name] = (time.perf_counter() - t0) / steps * 1e6
    table.check_status()
    del graph, pools, qkv
    torch.cuda.empty_cache()
    return dict(workload=f"decode-step attention path, {layers} layers, B={B}, ctx {ctx}, Qwen3-4B heads, bf16: "
                         f"device append + per layer fused prep + paged attention",
                metric="host wall us per decode step", value=round(out["graph"], 1), unit="us",
                eager_us=round(out["eager"], 1), higher_is_better=False)


def metadata_results(device, B: int = 256, ctx: int = 1024, steps: int = 20) -> dict:
    """Secondary line: one decode step's batch metadata + K/V write for B requests of ctx
    tokens (1 new token each, Qwen3-4B kv heads 8, d 128, bf16, page 16), host wall time
    per step (synchronised).  Host path: the reference-shaped per-request bookkeeping
    (BatchingKvCache.update_and_fetch_paged: Python loop over requests, block-table rows
    rebuilt from lists and copied to the device).  Device path: DevicePageTable.append
    (one kernel: new pages, slots, block tables, lengths) + the same scatter-write."""
    from nano_vllm_b200 import BatchingKvCache, DevicePageTable, TinyKvPagedCache, TinyKvPagedPool, write_slots

    Hkv, D, ps = 8, 128, 16
    gen = torch.Generator(device=device)
    gen.manual_seed(3)
    k1 = torch.randn(B, Hkv, 1, D, generator=gen, device=device).bfloat16()
    v1 = torch.randn(B, Hkv, 1, D, generator=gen, device=device).bfloat16()
    # host path state
    pool = TinyKvPagedPool(page_size=ps, device=device)
    batch = BatchingKvCache(B, ctx + steps + 8)
    for b in range(B):
        c = TinyKvPagedCache(pool)
        c.plan_append(ctx)
        batch.add_request(c, b)
    pool._ensure_page_storage(k1[:1])
    torch.cuda.synchronize()

    def host_step():
        batch.update_and_fetch_paged(k1, v1)
        torch.cuda.synchronize()

    # device path state (same pool shape); room for the eager and the graph runs
    mp = (ctx + 3 * (steps + 3) + 8 + ps - 1) // ps + 1
    dt = DevicePageTable(B, mp, ps, B * mp + 16, device=device)
    dt.append(torch.full((B,), ctx, dtype=torch.int32, device=device))
    dt.check_status()
    kp = torch.zeros(B * mp + 16, Hkv, ps, D, dtype=torch.bfloat16, device=device)
    vp = torch.zeros_like(kp)
    ones = torch.ones(B, dtype=torch.int32, device=device)
    slots = torch.empty(B, dtype=torch.int64, device=device)
    kt, vt = k1[:, :, 0], v1[:, :, 0]

    def device_step():
        dt.append(ones, slot_mapping=slots)
        write_slots(kt, vt, slots, kp, vp)
        torch.cuda.synchronize()

    # the device step captured once in a CUDA graph (no per-step host work at all)
    for _ in range(3):
        device_step()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        dt.append(ones, slot_mapping=slots)
        write_slots(kt, vt, slots, kp, vp)

    def graph_step():
        graph.replay()
        torch.cuda.synchronize()

    out = {}
    for name, fn in (("host", host_step), ("device", device_step), ("graph", graph_step)):
        for _ in range(3):
            fn()
        t0 = time.perf_counter()
        for _ in range(steps):
            fn()
        out[name] = (time.perf_counter() - t0) / steps * 1e6
    dt.check_status()
    del graph, kp, vp, pool, batch
    torch.cuda.empty_cache()
    return dict(workload=f"decode-step batch metadata + K/V write, B={B}, ctx {ctx}, 1 new token, kv heads 8, d 128",
                metric="host wall us per decode step", value=round(out["device"], 1), unit="us",
                host_path_us=round(out["host"], 1), graph_us=round(out["graph"], 1),
                speedup=round(out["host"] / out["device"], 1), higher_is_better=False)


def qk_prep_bytes(T: int, Hq: int, Hkv: int, D: int, kv_bytes: int, scale_bytes: int) -> int:
    """Algorithmic bytes of one fused q/k-norm + RoPE + K/V write over T tokens: read q, k,
    v rows once, write q once and K/V (+ int8 scales) once, one fp32 cos and sin row,
    the position and the slot of every token (the norm weights are 2 * D elements)."""
    per_tok = (Hq + 2 * Hkv) * D * 2 + Hq * D * 2 + 2 * Hkv * (D * kv_bytes + scale_bytes) + D * 4 + 4 + 8
    return T * per_tok + 2 * D * 2


def qk_prep_results(peaks: dict, device, flush, B: int = 4, iters: int = 20, warmup: int = 3,
                    kinds=("bf16", "int8")) -> list[dict]:
    """Secondary lines: the fused step at the config-2a token count (4 x 2048 tokens,
    Qwen3-4B heads 32 / 8, d 128, bf16) writing into bf16 and into int8 page pools."""
    from nano_vllm_b200.layers.qk_prep import qk_norm_rope_write
    from nano_vllm_b200.layers.rotary_embedding import RoPE

    res = []
    L, Hq, Hkv, D, ps = 2048, 32, 8, 128, 16
    T = B * L
    gen = torch.Generator(device=device)
    gen.manual_seed(9)
    qkv = torch.randn(B, L, (Hq + 2 * Hkv) * D, generator=gen, device=device).bfloat16()
    q = qkv[..., :Hq * D].view(B, L, Hq, D)
    k = qkv[..., Hq * D:(Hq + Hkv) * D].view(B, L, Hkv, D)
    v = qkv[..., (Hq + Hkv) * D:].view(B, L, Hkv, D)
    wq = torch.rand(D, generator=gen, device=device).bfloat16() + 0.5
    wk = torch.rand(D, generator=gen, device=device).bfloat16() + 0.5
    rope = RoPE(D, 40960, 1000000, device=device)
    pos = (torch.arange(L, device=device, dtype=torch.int32) + 512).repeat(B, 1)
    P = T // ps
    slots = torch.randperm(P * ps, generator=gen, device=device)[:T]
    out = torch.empty(B, Hq, L, D, dtype=torch.bfloat16, device=device)
    for kv in kinds:
        kv_dtype = torch.int8 if kv == "int8" else torch.bfloat16
        kp = torch.zeros(P, Hkv, ps, D, dtype=kv_dtype, device=device)
        vp = torch.zeros_like(kp)
        ks = torch.ones(P, Hkv, ps, 1, dtype=torch.bfloat16, device=device) if kv == "int8" else None
        vs = None if ks is None else ks.clone()
        nbytes = qk_prep_bytes(T, Hq, Hkv, D, 1 if kv == "int8" else 2, 2 if kv == "int8" else 0)
        ms = statistics.median(time_launches(
            lambda: qk_norm_rope_write(q, k, v, wq, wk, rope, pos, kp, vp, slots, eps=1e-6, key_scales=ks,
                                       value_scales=vs, out=out), iters, warmup, flush))
        gbs = nbytes / (ms * 1e-3) / 1e9
        res.append(dict(workload=f"qk-norm+RoPE+KV write, {T} tokens (config2a shape), {kv} pages",
                        metric="qk-prep GB/s", value=round(gbs, 1), unit="GB/s", ms=round(ms, 4),
                        bytes=nbytes, roofline_frac=round(gbs / peaks["hbm"], 4), l2="flushed"))
        del kp, vp, ks, vs
    return res


def run_qkprep(args):
    """The fused q/k-norm + RoPE + K/V write alone (bf16 pools), 4 x 2048 tokens unless
    --batch says otherwise; one JSON line."""
    from nano_vllm_b200 import _native as nv

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    peaks = measured_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    r = qk_prep_results(peaks, device, flush, B=args.batch or 4, iters=args.steps, warmup=args.warmup,
                        kinds=("bf16",))[0]
    line = {"metric": r["metric"], "value": r["value"], "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True, "dtype": "bf16",
            "config": {"workload": r["workload"], "l2": "flushed between launches"},
            "roofline": {"bound": "hbm", "achieved": r["value"], "peak": peaks["hbm"], "unit": "GB/s",
                         "frac": r["roofline_frac"], "peak_source": peaks["src"], "algorithmic_bytes": r["bytes"]},
            "device_error_word": nv.device_error(device)}
    print(json.dumps(line), flush=True)


def run_w4a16(args):
    """The W4A16 matmul alone at Qwen3-4B's gate+up projection shape (M = --batch or 1
    activation rows); one JSON line."""
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    peaks = measured_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    r = w4a16_results(peaks, device, flush, shapes=(("gate_up", 2 * 9728, 2560),), ms_rows=(args.batch or 1,),
                      iters=args.steps, warmup=args.warmup)[0]
    line = {"metric": r["metric"], "value": r["value"], "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True, "dtype": "bf16",
            "config": {"workload": r["workload"], "l2": "flushed between launches"},
            "roofline": {"bound": "hbm", "achieved": r["value"], "peak": peaks["hbm"], "unit": "GB/s",
                         "frac": r["roofline_frac"], "peak_source": peaks["src"], "algorithmic_bytes": r["bytes"]}}
    print(json.dumps(line), flush=True)


def run_prefill(args):
    """Config 2a: dense causal prefill (flash_attention), bf16, TFLOPS of visible pairs."""
    from nano_vllm_b200 import flash_attention
    from nano_vllm_b200 import _native as nv

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    peaks = measured_peaks()
    B = args.batch or 4
    Hq, Hkv, L, D = 32, 8, 2048, 128
    gen = torch.Generator(device=device)
    gen.manual_seed(5)
    q = torch.randn(B, Hq, L, D, generator=gen, device=device).bfloat16()
    k = torch.randn(B, Hkv, L, D, generator=gen, device=device).bfloat16()
    v = torch.randn(B, Hkv, L, D, generator=gen, device=device).bfloat16()
    flops = 4 * D * Hq * B * (L * (L + 1) // 2)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    times = time_launches(lambda: flash_attention(q, k, v, mask="causal", out_dtype=torch.bfloat16), args.steps,
                          args.warmup, flush)
    ms = statistics.median(times)
    tf = flops / (ms * 1e-3) / 1e12
    line = {"metric": "prefill attn TFLOPS", "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "dtype": "bf16", "config": {"workload": f"config2a dense causal prefill {B}x{L}, 32q/8kv, d128",
                                        "l2": "flushed between launches"},
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peaks["bf16"], "unit": "TFLOP/s",
                         "frac": round(tf / peaks["bf16"], 4), "peak_source": peaks["src"]},
            "device_error_word": nv.device_error(device)}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch.distributed as dist

    if args.config == "c2a":
        return run_prefill(args)
    if args.config == "qkprep":
        return run_qkprep(args)
    if args.config == "w4a16":
        return run_w4a16(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    peaks = measured_peaks()
    cfg = decode_config(args.config)
    cfg["name"] = f"config{args.config[1]}"
    if args.batch:
        cfg["B"] = args.batch
        cfg["name"] += f" (batch {args.batch})"
    w = build_decode(cfg, rank, world, device)
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        run_decode_step(w)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            evs[i][0].record(stream)
            run_decode_step(w)
            evs[i][1].record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms_total = t0.elapsed_time(t1)
    launch_ms = statistics.mean(s.elapsed_time(e) for s, e in evs)
    from nano_vllm_b200 import _native as nv

    dev_err = nv.device_error(device)
    t = torch.tensor([ms_total, float(w["bytes"]["total"]), float(dev_err)], dtype=torch.float64, device=device)
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax[0:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(tmax[1:2], op=dist.ReduceOp.SUM)
        dist.all_reduce(tmax[2:3], op=dist.ReduceOp.MAX)
        t = tmax
    ms_per_step = float(t[0]) / args.steps
    total_bytes = float(t[1])
    value = total_bytes / (ms_per_step * 1e-3) / 1e9

    # e2e through the public API with host buffers (every rank, max over ranks)
    e2e_ms, h2d, d2h = e2e_decode(w, max(3, args.steps // 2), 2)
    et = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_value = total_bytes / (float(et[0]) * 1e-3) / 1e9

    achieved = w["bytes"]["total"] / (launch_ms * 1e-3) / 1e9
    roof = dict(bound="hbm", achieved=round(achieved, 1), peak=peaks["hbm"], unit="GB/s",
                frac=round(achieved / peaks["hbm"], 4), peak_source=peaks["src"],
                kernel="paged_mma_kernel (mma.sync m16n8k16, TMA-fed)",
                algorithmic_bytes_per_launch=w["bytes"]["total"])
    tr = ncu_traffic(f"paged_mma:{args.config}:world{world}")
    roof["traffic"] = tr
    line = {
        "metric": "decode-attn KV GB/s", "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; N(0,1) K/V/Q, BASELINE config distributions)",
        "config": {"workload": f"{cfg['name']} paged decode" + (" + prefix sharing" if cfg["share"] else ""),
                   "model": cfg["model"], "batch": cfg["B"], "q_heads": cfg["Hq"], "kv_heads": cfg["Hkv"],
                   "head_dim": cfg["D"], "page_size": cfg["ps"], "context": str(cfg["ctx"]),
                   "shared_prefix_tokens": cfg["share"][1] if cfg["share"] else 0,
                   "parallelism": f"kv-head shard x{world}",
                   "l2": "inputs larger than L2" if w["bytes"]["kv"] > (256 << 20) else "inputs smaller than L2"},
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(float(et[0]), 4),
                "copies": "every step's H2D / D2H in the region, on two side streams overlapping neighbouring steps"},
        "gpu_launches": args.steps,
        "roofline": roof,
        "device_error_word": int(t[2]),
    }
    if rank == 0:
        line["clocks"] = clocks.summary()
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_decode(cfg, w, target_s=args.cpu_seconds)
    del w
    torch.cuda.empty_cache()
    if world == 1 and not args.no_secondary:
        line["secondary"] = secondary_results(peaks, device)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU path (eval_cpu, restated by the oracle)
# ---------------------------------------------------------------------------

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cfg = decode_config(args.config)
    cfg["name"] = f"config{args.config[1]}"
    per_step = max(0.5, args.ref_seconds / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_baseline_decode(cfg, None, target_s=per_step / 4)
    vals, secs = [], 0.0
    last = None
    for _ in range(args.steps):
        last = cpu_baseline_decode(cfg, None, target_s=per_step)
        vals.append(last["value"])
        secs += last["seconds"]
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": "decode-attn KV GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs / args.steps * 1e3, 1), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 math over fp16 pages",
        "data": "synthetic (seeded; same distributions as our arm)",
        "config": {"workload": f"{cfg['name']} paged decode + prefix sharing", "model": cfg["model"],
                   "batch": cfg["B"], "q_heads": cfg["Hq"], "kv_heads": cfg["Hkv"], "head_dim": cfg["D"],
                   "page_size": cfg["ps"], "context": "uniform[4096,32768]"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": last["cores"], "kind": "port",
                         "sample": last["sample"]},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "MLX (the reference's runtime) is not installable offline; the reference's mx.cpu path for this "
                "op is PagedAttention::eval_cpu, timed here as its C restatement (oracle/nvm_oracle.c).",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c1", "c2a", "c3", "c4", "c5", "qkprep", "w4a16"], default="c3")
    ap.add_argument("--batch", type=int, default=None, help="override the config's batch (small profiling cases)")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
