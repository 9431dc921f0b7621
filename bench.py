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

Secondary lines (N=1 only) time configs 1, 4, 5 (decode GB/s), 2a and the 2b sweep
(chunked prefill, 512 new tokens against 0, 512, ..., 4096 paged tokens; TFLOPS), the
fused q/k-norm + RoPE + K/V write at the 2a token count (GB/s), the per-decode-step
batch metadata path and a whole decode step's attention path (host wall time) and the
W4A16 matmul at Qwen3-4B's MLP shapes (GB/s), one launch at a time with an L2 flush
between launches.

Every line carries ``parity``: after its timed region, the output of the last timed
launch is compared with the oracle (``oracle/``, the reference's CPU loops restated)
on the same bytes -- a seeded sample of sequences (for config 3 two whole shared-prefix
groups) with the pages they reference copied to the host, or a sample of heads over
all rows for prefill.  The process exits with status 3 after printing if any check is
over tolerance.  The CPU baselines (``cpu_baseline``; ``--impl reference``) time the
same oracle on the same workload definitions on the host cores, single-threaded (as
the reference's ``eval_cpu`` runs) and on all host threads.
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
# north-star tolerance of 16-bit / int8 attention outputs (fp32 accumulation)
ATOL16, RTOL16 = 2e-3, 1e-2
_PARITY_FAILED = []


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


def chunk_config(prior: int) -> dict:
    """Config 2b point: 4 sequences x 512 new tokens against `prior` paged tokens."""
    return dict(B=4, Hq=32, Hkv=8, L=512, D=128, ps=16, dtype=torch.bfloat16,
                ctx=("uniform", prior + 512, prior + 512), share=None, model="Qwen3-4B")


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
    """Algorithmic bytes of one decode call (logical K/V per kv head, Q, O, metadata).

    ``kv_unique`` counts the K/V of a shared-prefix page once per group (the bytes
    that have to come from DRAM at least once); ``kv`` counts them per sequence.
    """
    D, ps, L = cfg["D"], cfg["ps"], cfg["L"]
    per_token = D * 2 * 1 + 2 * 2 if cfg["dtype"] == torch.int8 else D * 2 * 2  # K+V (+ fp16 scales)
    qb = 2
    kv = int(ctx.sum()) * n_kv * per_token
    kv_unique = kv
    if cfg["share"] is not None:
        group, tokens = cfg["share"]
        n = len(ctx)
        dup = sum(max(0, min(group, n - g0) - 1) for g0 in range(0, n, group)) * tokens
        kv_unique = kv - dup * n_kv * per_token
    q = len(ctx) * n_q * L * D * qb
    o = len(ctx) * n_q * L * D * out_bytes
    meta = int(((ctx + ps - 1) // ps).sum()) * 4 + 4 * len(ctx)
    return dict(kv=kv, kv_unique=kv_unique, q=q, o=o, meta=meta, total=kv + q + o + meta,
                total_unique=kv_unique + q + o + meta)


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
                shard=sh, bytes=nbytes, cfg=cfg)


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


def host_cpu() -> dict:
    """The host CPU the baselines ran on: model name and usable hardware threads."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        nproc = len(os.sched_getaffinity(0))
    except AttributeError:
        nproc = os.cpu_count()
    return {"model": model, "nproc": nproc}


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


def time_launches(fn, iters: int, warmup: int, flush_buf=None):
    """Per-launch device ms with CUDA events on the current stream (L2 flushed between);
    returns (times, result of the last launch)."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    times, res = [], None
    for _ in range(iters):
        if flush_buf is not None:
            flush_l2(flush_buf)
        # keep the GPU busy (~200 us) while the host queues the start event and the
        # launch, so host-side delays never show up as idle time inside the events
        torch.cuda._sleep(400_000)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        res = fn()
        e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e))
    return times, res


def harness_floor_us(flush_buf, iters: int = 20) -> float:
    """Median event-to-event time of a one-element fill timed exactly like the kernels
    (L2 flush, GPU sleep, start event, launch, end event): the smallest interval this
    harness can report for any launch."""
    x = torch.zeros(1, device=flush_buf.device)
    times, _ = time_launches(lambda: x.fill_(1.0), iters, 3, flush_buf)
    return round(statistics.median(times) * 1000, 2)


def spread(times_ms: list[float], work: float, scale: float) -> dict:
    """Median, p10 and p90 of a rate work / time (scale converts to the unit)."""
    rates = sorted(work / (t * 1e-3) / scale for t in times_ms)
    q = lambda p: float(np.percentile(rates, p))  # noqa: E731
    return {"p10": round(q(10), 1), "p50": round(q(50), 1), "p90": round(q(90), 1), "launches": len(times_ms)}


# ---------------------------------------------------------------------------
# parity of the timed launches against the oracle (the checker, never measured)
# ---------------------------------------------------------------------------

def _oracle():
    # OpenMP worker threads must sleep, not spin, once a call is done: spinning
    # threads on every core delay the host's kernel launches in the GPU timings after it
    os.environ.setdefault("OMP_WAIT_POLICY", "PASSIVE")
    from oracle import oracle as o

    return o


def to_np(t: torch.Tensor) -> np.ndarray:
    """Tensor -> numpy; bf16 becomes uint16 bit patterns (the oracle's bf16 form)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def compare(got: np.ndarray, ref: np.ndarray, atol: float, rtol: float, rows: int, what: str) -> dict:
    """allclose(got, ref, atol, rtol) with the figures behind it.  max_rel is taken over
    the elements with |ref| >= atol / rtol, where the relative term dominates."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(got - ref)
    lim = atol + rtol * np.abs(ref)
    big = np.abs(ref) >= atol / rtol
    ok = bool(np.all(np.isfinite(got)) and np.all(d <= lim))
    res = {"ok": ok, "max_abs": float(d.max()) if d.size else 0.0,
           "max_rel": float((d[big] / np.abs(ref[big])).max()) if big.any() else 0.0,
           "worst_over_tol": float((d / lim).max()) if d.size else 0.0, "atol": atol, "rtol": rtol,
           "rows_checked": int(rows), "checked": what}
    if not ok:
        _PARITY_FAILED.append(what)
    return res


def parity_paged(w: dict, out: torch.Tensor, rows: np.ndarray, heads: np.ndarray | None = None) -> dict:
    """The timed call's output for sequences `rows` (and q heads `heads`, one per kv
    head, or all) against the oracle run on the same page bytes and block-table rows."""
    o = _oracle()
    dev = w["q"].device
    bt = w["bt"].cpu().numpy()[rows]
    cl = w["cl"].cpu().numpy()[rows]
    uniq = np.unique(bt[bt >= 0])
    remap = np.where(bt >= 0, np.searchsorted(uniq, np.maximum(bt, 0)), -1).astype(np.int32)
    idx = torch.from_numpy(uniq.astype(np.int64)).to(dev)
    sel = lambda t: None if t is None else to_np(t.index_select(0, idx))  # noqa: E731
    kp, vp, ks, vs = sel(w["kp"]), sel(w["vp"]), sel(w["ks"]), sel(w["vs"])
    ridx = torch.from_numpy(rows.astype(np.int64)).to(dev)
    q = w["q"].index_select(0, ridx)
    got = out.index_select(0, ridx)
    if heads is not None:
        hidx = torch.from_numpy(heads.astype(np.int64)).to(dev)
        q, got = q.index_select(1, hidx), got.index_select(1, hidx)
        # one q head per kv head: the oracle's grouping maps q head j to kv head j
        assert len(heads) == kp.shape[1]
    ref = o.paged_attention_ref(q.float().cpu().numpy(), kp, vp, remap, cl, w["ps"], ks, vs, mask="causal",
                                kv_is_bf16=w["kp"].dtype == torch.bfloat16, nthreads=o.max_threads())
    nrows = q.shape[0] * q.shape[1] * q.shape[2]
    what = f"{len(rows)} sequences x {q.shape[1]} q heads x {q.shape[2]} tokens, {len(uniq)} pages"
    return compare(got.float().cpu().numpy(), ref, ATOL16, RTOL16, nrows, what)


def sample_rows(cfg: dict, B_local: int, b_lo: int, seed: int, n: int = 16) -> np.ndarray:
    """Seeded sample of local sequence rows: two whole shared-prefix groups when the
    config shares prefixes, else n sequences."""
    rng = np.random.default_rng(seed)
    if cfg.get("share"):
        group = cfg["share"][0]
        groups = sorted({(b_lo + i) // group for i in range(B_local)})
        pick = set(rng.choice(groups, size=min(2, len(groups)), replace=False).tolist())
        return np.array([i for i in range(B_local) if (b_lo + i) // group in pick], dtype=np.int64)
    return np.sort(rng.choice(B_local, size=min(n, B_local), replace=False)).astype(np.int64)


def parity_dense(q, k, v, out, pairs) -> dict:
    """Dense causal prefill: (batch, q head) pairs over all rows against the oracle."""
    o = _oracle()
    g = q.shape[1] // k.shape[1]
    qs = torch.stack([q[b, h] for b, h in pairs])[:, None]
    ks = torch.stack([k[b, h // g] for b, h in pairs])[:, None]
    vs = torch.stack([v[b, h // g] for b, h in pairs])[:, None]
    got = torch.stack([out[b, h] for b, h in pairs])[:, None]
    ref = o.flash_attention_ref(qs.float().cpu().numpy(), ks.float().cpu().numpy(), vs.float().cpu().numpy(),
                                mask="causal", nthreads=o.max_threads())
    what = f"{len(pairs)} (batch, q head) pairs x {q.shape[2]} rows"
    return compare(got.float().cpu().numpy(), ref, ATOL16, RTOL16, len(pairs) * q.shape[2], what)


def one_head_per_group(Hq: int, Hkv: int) -> np.ndarray:
    g = Hq // Hkv
    return np.array([j * g + (j % g) for j in range(Hkv)], dtype=np.int64)


# ---------------------------------------------------------------------------
# CPU baselines: the oracle (the reference's eval_cpu restated) on the host cores
# ---------------------------------------------------------------------------

def _rand_pages(rng, cfg: dict, n: int, H: int):
    """K/V pages [n, H, page_size, D] of the workload's dtype and distribution (int8
    uniform with |N(0,1)|/127 fp16 scales, else N(0,1)).  Large banks repeat a 16 MB
    block of fresh values at shifting offsets: the values keep their distribution and
    every page still has its own addresses, at a fraction of the generation time."""
    D, ps = cfg["D"], cfg["ps"]
    o = _oracle()
    shape = (n, H, ps, D)
    total = n * H * ps * D

    def fill(make):
        base = make(min(total, 1 << 23))
        out = np.empty(total, dtype=base.dtype)
        pos, r = 0, 0
        while pos < total:
            m = min(base.size, total - pos)
            out[pos:pos + m] = np.roll(base, 7919 * r)[:m]
            pos, r = pos + m, r + 1
        return out.reshape(shape)

    if cfg["dtype"] == torch.int8:
        kp = fill(lambda m: rng.integers(-127, 128, m, dtype=np.int8))
        vp = fill(lambda m: rng.integers(-127, 128, m, dtype=np.int8))
        ks = (np.abs(rng.standard_normal((n, H, ps, 1))) / 127).astype(np.float16)
        vs = (np.abs(rng.standard_normal((n, H, ps, 1))) / 127).astype(np.float16)
        return kp, vp, ks, vs
    if cfg["dtype"] == torch.bfloat16:
        make = lambda m: o.f32_to_bf16_bits(rng.standard_normal(m, dtype=np.float32))  # noqa: E731
    else:
        make = lambda m: rng.standard_normal(m, dtype=np.float32).astype(np.float16)  # noqa: E731
    return fill(make), fill(make), None, None


_BANKS: dict = {}


def _page_bank(cfg: dict, n: int, H: int):
    key = (str(cfg["dtype"]), n, H, cfg["D"], cfg["ps"])
    if key not in _BANKS:
        _BANKS.clear()
        _BANKS[key] = _rand_pages(np.random.default_rng(98), cfg, n, H)
    return _BANKS[key]


def cpu_decode_sample(cfg: dict, nthreads: int, target_s: float, bank_pages: int = 4096, seed: int = 0) -> dict:
    """Time the oracle on sequences of the workload itself: the same context lengths and
    block tables (shared-prefix groups kept whole, in a seeded order) as the GPU run.
    Page contents come from a bank of `bank_pages` random pages of the workload's dtype
    (256 MB for 16-bit K+V at 8 kv heads, far above the host caches), page id p reading
    bank page p mod bank_pages, so shared-prefix pages stay shared."""
    o = _oracle()
    ctx = sample_context_lens(cfg, seed)
    bt, P = block_tables(cfg, ctx, seed)
    rng = np.random.default_rng(99)
    B, Hq, Hkv, L, D = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["L"], cfg["D"]
    if cfg["share"]:
        group = cfg["share"][0]
        order = [list(range(g * group, min(B, (g + 1) * group))) for g in rng.permutation((B + group - 1) // group)]
    else:
        order = [[int(b)] for b in rng.permutation(B)]
    if nthreads == 1:
        order = [[b] for grp in order for b in grp]
    bank = min(bank_pages, P)
    kp, vp, ks, vs = _page_bank(cfg, bank, Hkv)
    bf16 = cfg["dtype"] == torch.bfloat16
    total_t, total_b, used, calls = 0.0, 0, 0, 0
    for batch in order:
        rows = np.array(batch)
        bt_b = np.where(bt[rows] >= 0, bt[rows] % bank, -1).astype(np.int32)
        cl_b = ctx[rows].astype(np.int32)
        q = rng.standard_normal((len(rows), Hq, L, D)).astype(np.float32)
        if cfg["dtype"] != torch.float32:
            q = q.astype(np.float16).astype(np.float32) if not bf16 else o.bf16_bits_to_f32(o.f32_to_bf16_bits(q))
        t0 = time.perf_counter()
        o.paged_attention_ref(q.reshape(len(rows), Hq, L, D), kp, vp, bt_b, cl_b, cfg["ps"], ks, vs, mask="causal",
                              kv_is_bf16=bf16, nthreads=nthreads)
        total_t += time.perf_counter() - t0
        total_b += decode_bytes(cfg, ctx[rows], Hkv, Hq)["total"]
        used += len(rows)
        calls += 1
        if total_t > target_s:
            break
    share = f", {cfg['share'][0]}-sequence shared-prefix groups kept whole" if cfg["share"] else ""
    return dict(value=round(total_b / total_t / 1e9, 4), unit="GB/s", seconds=round(total_t, 2), sequences=used,
                sample=f"{used} of {B} sequences (all {Hq} q heads, their real context lengths and block tables"
                       f"{share}; page bytes from a {bank}-page random bank), {calls} oracle calls, "
                       f"{total_t:.1f} s on {nthreads} thread(s)")


def cpu_prefill_sample(prior: int, L: int, nthreads: int, target_s: float, heads: int, dense: bool = False) -> dict:
    """Time the oracle's prefill on `heads` q heads of one sequence, each with its own kv
    head (the per-head arithmetic of the 32/8-head config); TFLOP/s of visible pairs.
    dense: FlashAttention::eval_cpu over dense K/V (config 2a); else
    PagedAttention::eval_cpu of L new tokens against `prior` paged tokens (config 2b)."""
    o = _oracle()
    cfg = dict(D=128, ps=16, dtype=torch.bfloat16)
    rng = np.random.default_rng(7)
    ctx = prior + L
    npg = (ctx + 15) // 16
    if dense:
        k = o.bf16_bits_to_f32(o.f32_to_bf16_bits(rng.standard_normal((1, heads, ctx, 128)).astype(np.float32)))
        v = o.bf16_bits_to_f32(o.f32_to_bf16_bits(rng.standard_normal((1, heads, ctx, 128)).astype(np.float32)))
    else:
        kp, vp, _, _ = _rand_pages(rng, cfg, npg, heads)
        bt = np.arange(npg, dtype=np.int32)[None]
    flops_head = 4 * 128 * sum(prior + r + 1 for r in range(L))
    total_t, total_f, calls = 0.0, 0, 0
    while True:
        q = o.bf16_bits_to_f32(o.f32_to_bf16_bits(rng.standard_normal((1, heads, L, 128)).astype(np.float32)))
        t0 = time.perf_counter()
        if dense:
            o.flash_attention_ref(q, k, v, mask="causal", nthreads=nthreads)
        else:
            o.paged_attention_ref(q, kp, vp, bt, np.array([ctx], dtype=np.int32), 16, mask="causal",
                                  kv_is_bf16=True, nthreads=nthreads)
        total_t += time.perf_counter() - t0
        total_f += flops_head * heads
        calls += 1
        if total_t > target_s:
            break
    kind = "dense FlashAttention::eval_cpu" if dense else f"paged, against {prior} paged tokens"
    return dict(value=round(total_f / total_t / 1e12, 5), unit="TFLOP/s", seconds=round(total_t, 2),
                sample=f"{calls} call(s) of {heads} q head(s) x {L} new tokens ({kind}), "
                       f"{total_t:.1f} s on {nthreads} thread(s)")


def cpu_baseline_pair(measure, target_s: float) -> dict:
    """A baseline on one thread (how the reference's eval_cpu runs: one CPU task) and on
    every host thread (the oracle's OpenMP over query rows)."""
    o = _oracle()
    n = o.max_threads()
    allc = measure(n, target_s)
    one = measure(1, target_s)
    cpu = host_cpu()
    return {"value": allc["value"], "unit": allc["unit"], "cores": n, "kind": "port",
            "sample": allc["sample"], "single_thread": {"value": one["value"], "cores": 1, "sample": one["sample"]},
            "cpu_model": cpu["model"], "nproc": cpu["nproc"]}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_decode_step(w, out=None):
    from nano_vllm_b200 import paged_attention

    return paged_attention(w["q"], w["kp"], w["vp"], w["bt"], w["cl"], w["ps"], w["ks"], w["vs"], mask="causal",
                           out=out)


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
    # the host copy of the last step's result is the device result of that step
    e2e_ok = bool(torch.equal(out_h[(steps - 1) & 1], out_d[(steps - 1) & 1].cpu()))
    return ms, h2d, d2h, e2e_ok


def decode_line(name: str, peaks: dict, device, flush, cpu: bool, cpu_seconds: float) -> dict:
    cfg = decode_config(name)
    cfg["name"] = f"config{name[1]}"
    w = build_decode(cfg, 0, 1, device)
    times, out = time_launches(lambda: run_decode_step(w), 20, 3, flush)
    ms = statistics.median(times)
    gbs = w["bytes"]["total"] / (ms * 1e-3) / 1e9
    line = dict(workload=f"config{name[1]} decode {cfg['model']}", metric="decode-attn KV GB/s",
                value=round(gbs, 1), unit="GB/s", ms=round(ms, 4), spread=spread(times, w["bytes"]["total"], 1e9),
                roofline_frac=round(gbs / peaks["hbm"], 4), l2="flushed",
                parity=parity_paged(w, out, sample_rows(cfg, cfg["B"], 0, seed=11)))
    if name == "c1":
        # a 38 MB launch is near the harness's own floor: report it beside the number
        floor = harness_floor_us(flush)
        line["harness_floor_us"] = floor
        line["best_possible_frac_in_harness"] = round(
            w["bytes"]["total"] / ((w["bytes"]["total"] / (peaks["hbm"] * 1e9)) + floor * 1e-6) / 1e9 / peaks["hbm"], 4)
    if cpu:
        line["cpu_baseline"] = cpu_baseline_pair(lambda n, t: cpu_decode_sample(cfg, n, t), cpu_seconds)
    del w, out
    torch.cuda.empty_cache()
    return line


def short_decode_results(peaks: dict, device, flush, batches=(64, 128)) -> list[dict]:
    """Secondary lines: paged decode at a serving decode step's shape (Qwen3-4B heads
    32 / 8, d 128, bf16, page 16, contexts U[1024, 1100], no shared pages), B = 64 and
    128: one launch after an L2 flush like every other line, and the same launch back to
    back in a CUDA graph over enough copies of the pools (different pages, > 1 GB in all)
    that L2 holds none of them -- how a decode step's layers run, without the harness's
    per-launch floor.  Parity: the single launch against the oracle on sampled rows."""
    res = []
    for B in batches:
        cfg = dict(B=B, Hq=32, Hkv=8, L=1, D=128, ps=16, dtype=torch.bfloat16, ctx=("uniform", 1024, 1100),
                   share=None, model="Qwen3-4B")
        w = build_decode(cfg, 0, 1, device)
        nbytes = w["bytes"]["total"]
        times, out = time_launches(lambda: run_decode_step(w), 20, 3, flush)
        ms = statistics.median(times)
        gbs = nbytes / (ms * 1e-3) / 1e9
        parity = parity_paged(w, out, sample_rows(cfg, B, 0, seed=13))
        ncopy = max(4, int(1.2e9 // w["kp"].nbytes // 2) + 1)
        copies = [w] + [build_decode(cfg, 0, 1, device, seed=s) for s in range(1, ncopy)]
        outs = [torch.empty_like(out) for _ in copies]
        for c, o in zip(copies, outs):
            run_decode_step(c, out=o)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for c, o in zip(copies, outs):
                run_decode_step(c, out=o)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        g_us = e0.elapsed_time(e1) * 1000 / (reps * len(copies))
        g_bytes = sum(c["bytes"]["total"] for c in copies) / len(copies)
        g_gbs = g_bytes / (g_us * 1e-6) / 1e9
        res.append(dict(workload=f"decode at the decode-step shape Qwen3-4B, B={B}, ctx U[1024,1100], bf16",
                        metric="decode-attn KV GB/s", value=round(gbs, 1), unit="GB/s", ms=round(ms, 4),
                        bytes=nbytes, spread=spread(times, nbytes, 1e9), roofline_frac=round(gbs / peaks["hbm"], 4),
                        l2="flushed", graph_us_per_launch=round(g_us, 2), graph_gbs=round(g_gbs, 1),
                        graph_roofline_frac=round(g_gbs / peaks["hbm"], 4),
                        graph=f"{len(copies)} launches over distinct pools back to back, {reps} replays",
                        parity=parity))
        del graph, copies, outs, w, out
        torch.cuda.empty_cache()
    return res


def secondary_results(peaks: dict, device, cpu: bool, cpu_seconds: float) -> list[dict]:
    from nano_vllm_b200 import flash_attention

    res = []
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for name in ["c1", "c4", "c5"]:
        res.append(decode_line(name, peaks, device, flush, cpu, cpu_seconds))
    res.extend(short_decode_results(peaks, device, flush))
    # 2a: dense causal prefill, 4 x 2048, 32/8 heads, bf16
    gen = torch.Generator(device=device)
    gen.manual_seed(5)
    B, Hq, Hkv, L, D = 4, 32, 8, 2048, 128
    q = torch.randn(B, Hq, L, D, generator=gen, device=device).bfloat16()
    k = torch.randn(B, Hkv, L, D, generator=gen, device=device).bfloat16()
    v = torch.randn(B, Hkv, L, D, generator=gen, device=device).bfloat16()
    flops = 4 * D * Hq * B * (L * (L + 1) // 2)
    times, out = time_launches(lambda: flash_attention(q, k, v, mask="causal", out_dtype=torch.bfloat16), 10, 3,
                               flush)
    ms = statistics.median(times)
    tf = flops / (ms * 1e-3) / 1e12
    rng = np.random.default_rng(12)
    pairs = [(int(b), int(h)) for b, h in zip(rng.integers(0, B, 8), rng.choice(Hq, 8, replace=False))]
    line = dict(workload="config2a dense causal prefill Qwen3-4B 4x2048", metric="prefill attn TFLOPS",
                value=round(tf, 1), unit="TFLOP/s", ms=round(ms, 4), spread=spread(times, flops, 1e12),
                roofline_frac=round(tf / peaks["bf16"], 4), l2="flushed", parity=parity_dense(q, k, v, out, pairs))
    if cpu:
        line["cpu_baseline"] = cpu_baseline_pair(
            lambda n, t: cpu_prefill_sample(0, L, n, t, 16 if n > 1 else 1, dense=True), cpu_seconds)
    res.append(line)
    del q, k, v, out
    # 2b: chunked prefill, a 512-token chunk against c tokens of paged context
    for c in range(0, 4097, 512):
        cfg = chunk_config(c)
        w = build_decode(cfg, 0, 1, device)
        flops = 4 * D * Hq * 4 * sum(c + r + 1 for r in range(512))
        times, out = time_launches(lambda: run_decode_step(w), 10, 3, flush)
        ms = statistics.median(times)
        tf = flops / (ms * 1e-3) / 1e12
        rows = np.array([0, 3], dtype=np.int64)
        line = dict(workload=f"config2b chunked prefill 512 vs {c} paged", metric="prefill attn TFLOPS",
                    value=round(tf, 1), unit="TFLOP/s", ms=round(ms, 4), spread=spread(times, flops, 1e12),
                    roofline_frac=round(tf / peaks["bf16"], 4), l2="flushed",
                    parity=parity_paged(w, out, rows, one_head_per_group(Hq, Hkv)))
        if cpu and c in (0, 1024, 4096):
            line["cpu_baseline"] = cpu_baseline_pair(
                lambda n, t: cpu_prefill_sample(c, 512, n, t, 16 if n > 1 else 1), cpu_seconds)
        res.append(line)
        del w, out
    res.extend(qk_prep_results(peaks, device, flush))
    res.append(metadata_results(device))
    res.append(decode_step_results(device))
    res.extend(w4a16_results(peaks, device, flush))
    return res


def w4a16_results(peaks: dict, device, flush, shapes=(("gate_up", 2 * 9728, 2560), ("down", 2560, 9728)),
                  ms_rows=(1, 8), iters: int = 20, warmup: int = 3) -> list[dict]:
    """Secondary lines: W4A16 (4-bit, group 128) matmul at Qwen3-4B's decode shapes
    (gate+up projection K = 2 x 9728, N = 2560; down projection K = 2560, N = 9728),
    M = 1 and 8 activation rows, bf16; GB/s of weights + scales + biases + activations.
    Parity: the whole output against the oracle's QuantizedMatmul::eval_cpu within one
    bf16 unit in the last place (the kernel's per-group fp32 order differs)."""
    from nano_vllm_b200.layers.linear import quantized_matmul

    o = _oracle()
    res = []
    gen = torch.Generator(device=device)
    gen.manual_seed(11)
    for name, K, N in shapes:
        w = torch.randint(-2 ** 31, 2 ** 31 - 1, (K, N // 8), generator=gen, dtype=torch.int64,
                          device=device).to(torch.int32)
        s = (torch.rand(K, N // 128, generator=gen, device=device) * 0.02).bfloat16()
        b = (torch.rand(K, N // 128, generator=gen, device=device) * -0.1).bfloat16()
        w_np, s_np, b_np = w.cpu().numpy().view(np.uint32), to_np(s), to_np(b)
        for M in ms_rows:
            a = torch.randn(M, N, generator=gen, device=device).bfloat16()
            nbytes = K * N // 2 + 2 * K * (N // 128) * 2 + M * N * 2 + M * K * 2
            times, out = time_launches(lambda: quantized_matmul(s, b, 128, 4, a, w, True), iters, warmup, flush)
            ms = statistics.median(times)
            gbs = nbytes / (ms * 1e-3) / 1e9
            ref = o.bf16_bits_to_f32(o.quantized_matmul_ref(to_np(a), 2, w_np, s_np, b_np, nthreads=o.max_threads()))
            got = o.bf16_bits_to_f32(to_np(out))
            par = compare(got, ref, 1e-4 * float(np.abs(ref).max()) + 1e-6, 2.0 ** -7, M,
                          f"all {M} x {K} outputs (1 bf16 ulp)")
            res.append(dict(workload=f"W4A16 matmul {name} Qwen3-4B (K={K}, N={N}), M={M}, bf16",
                            metric="w4a16 GB/s", value=round(gbs, 1), unit="GB/s", ms=round(ms, 4), bytes=nbytes,
                            spread=spread(times, nbytes, 1e9), roofline_frac=round(gbs / peaks["hbm"], 4),
                            l2="flushed", parity=par))
        del w, s, b
    return res


def _replay_allocator(B: int, ctx: int, appends: int, page_size: int):
    """The reference's sequential page allocation (oracle.PagePoolRef / PagedCacheRef)
    for B requests prefilled with ctx tokens, then `appends` decode steps of one token
    each, request by request: block-table rows and lengths."""
    o = _oracle()
    pool = o.PagePoolRef(page_size)
    caches = [o.PagedCacheRef(pool) for _ in range(B)]
    for c in caches:
        c.append_chunk(ctx)
    for _ in range(appends):
        for c in caches:
            c.append_chunk(1)
    return [c.page_ids for c in caches], [ctx + appends] * B


def _table_parity(table, B: int, ctx: int, appends: int, page_size: int) -> dict:
    ids, lens = _replay_allocator(B, ctx, appends, page_size)
    bt = table.block_table.cpu().numpy()
    cl = table.context_lens.cpu().tolist()
    ok = cl == lens and all(bt[b, :len(r)].tolist() == r and (bt[b, len(r):] == -1).all() for b, r in enumerate(ids))
    if not ok:
        _PARITY_FAILED.append("device page table")
    return {"ok": bool(ok), "checked": f"block tables and lengths of {B} requests after {appends} appends "
                                       "equal the sequential allocator (bit-exact)"}


def decode_step_results(device, layers: int = 36, B: int = 64, ctx: int = 1024, steps: int = 20) -> dict:
    """Secondary line: the attention path of one decode step of a Qwen3-4B-shaped model
    (36 layers, 32 q / 8 kv heads, d 128, bf16, page 16), B requests of ctx tokens, host
    wall time per step: DevicePageTable.append once, then per layer the fused q/k norm +
    RoPE + K/V write and paged attention, with the metadata on the device throughout --
    launched eagerly, and as one CUDA graph replayed per step.  Parity: the page table
    against the sequential allocator, and the last layer's attention of the last step
    against the oracle on a sample of requests."""
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
    last_q = torch.empty(B, Hq, 1, D, dtype=torch.bfloat16, device=device)
    last_out = torch.empty(B, Hq, 1, D, dtype=torch.bfloat16, device=device)
    appends = [0]

    def step():
        table.append(ones, slot_mapping=slots)
        pos = (table.context_lens - 1).view(B, 1)
        for li in range(layers):
            x = qkv[li]
            q = x[..., :Hq * D].view(B, 1, Hq, D)
            k = x[..., Hq * D:(Hq + Hkv) * D].view(B, 1, Hkv, D)
            v = x[..., (Hq + Hkv) * D:].view(B, 1, Hkv, D)
            kp, vp = pools[li]
            last = li == layers - 1
            qr = qk_norm_rope_write(q, k, v, wq, wk, rope, pos, kp, vp, slots, eps=1e-6,
                                    out=last_q if last else None)
            paged_attention(qr, kp, vp, table.block_table, table.context_lens, ps, out_dtype=torch.bfloat16,
                            out=last_out if last else None)

    def eager():
        step()
        appends[0] += 1
        torch.cuda.synchronize()

    for _ in range(3):
        eager()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()

    def replay():
        graph.replay()
        appends[0] += 1
        torch.cuda.synchronize()

    out = {}
    for name, fn in (("eager", eager), ("graph", replay)):
        fn()
        t0 = time.perf_counter()
        for _ in range(steps):
            fn()
        out[name] = (time.perf_counter() - t0) / steps * 1e6
    table.check_status()
    par = _table_parity(table, B, ctx, appends[0], ps)
    w = dict(q=last_q, kp=pools[-1][0], vp=pools[-1][1], ks=None, vs=None, bt=table.block_table,
             cl=table.context_lens, ps=ps)
    att = parity_paged(w, last_out, np.arange(0, B, B // 8, dtype=np.int64))
    par = {"ok": par["ok"] and att["ok"], "page_table": par, "last_layer_attention": att}
    del graph, pools, qkv
    torch.cuda.empty_cache()
    return dict(workload=f"decode-step attention path, {layers} layers, B={B}, ctx {ctx}, Qwen3-4B heads, bf16: "
                         f"device append + per layer fused prep + paged attention",
                metric="host wall us per decode step", value=round(out["graph"], 1), unit="us",
                eager_us=round(out["eager"], 1), higher_is_better=False, parity=par)


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
    appends = [0]

    def device_step():
        dt.append(ones, slot_mapping=slots)
        write_slots(kt, vt, slots, kp, vp)
        appends[0] += 1
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
        appends[0] += 1
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
    par = _table_parity(dt, B, ctx, appends[0], ps)
    # the last step's K/V rows landed at the slots that step was given
    pg, off = slots // ps, slots % ps
    ok_kv = bool(torch.equal(kp[pg, :, off], kt) and torch.equal(vp[pg, :, off], vt))
    if not ok_kv:
        _PARITY_FAILED.append("metadata K/V write")
    par = {"ok": par["ok"] and ok_kv, "page_table": par,
           "kv_write": {"ok": ok_kv, "checked": f"the last step's {B} K and V rows at their slots (bit-exact)"}}
    del graph, kp, vp, pool, batch
    torch.cuda.empty_cache()
    return dict(workload=f"decode-step batch metadata + K/V write, B={B}, ctx {ctx}, 1 new token, kv heads 8, d 128",
                metric="host wall us per decode step", value=round(out["device"], 1), unit="us",
                host_path_us=round(out["host"], 1), graph_us=round(out["graph"], 1),
                speedup=round(out["host"] / out["device"], 1), higher_is_better=False, parity=par)


def qk_prep_bytes(T: int, Hq: int, Hkv: int, D: int, kv_bytes: int, scale_bytes: int) -> int:
    """Algorithmic bytes of one fused q/k-norm + RoPE + K/V write over T tokens: read q, k,
    v rows once, write q once and K/V (+ int8 scales) once, one fp32 cos and sin row,
    the position and the slot of every token (the norm weights are 2 * D elements)."""
    per_tok = (Hq + 2 * Hkv) * D * 2 + Hq * D * 2 + 2 * Hkv * (D * kv_bytes + scale_bytes) + D * 4 + 4 + 8
    return T * per_tok + 2 * D * 2


def _qk_prep_parity(q, k, v, wq, wk, rope, pos, kp, vp, ks, vs, slots, out, eps, n_tok: int = 64) -> dict:
    """Bit-exact check of a seeded sample of tokens: q rows out and the K/V (and int8
    scale) rows at their slots, against the oracle on the same input rows."""
    o = _oracle()
    B, L, Hq, D = q.shape
    Hkv = k.shape[2]
    T = B * L
    rng = np.random.default_rng(21)
    toks = np.sort(rng.choice(T, size=n_tok, replace=False))
    bi, li = toks // L, toks % L
    pick = lambda x: to_np(x.reshape(T, -1, D)[torch.from_numpy(toks).to(x.device)])  # noqa: E731
    s_np = slots.cpu().numpy()[toks]
    P, _, ps, _ = kp.shape
    # a compact pool of n_tok pages: sampled token i goes to page i, its own offset
    sl_local = np.arange(n_tok, dtype=np.int64) * ps + s_np % ps
    code = 2
    kv_code = 3 if kp.dtype == torch.int8 else 2
    kp_r = np.zeros((n_tok, Hkv, ps, D), dtype=np.int8 if kv_code == 3 else np.uint16)
    vp_r = np.zeros_like(kp_r)
    ks_r = None if ks is None else np.zeros((n_tok, Hkv, ps, 1), dtype=np.uint16)
    vs_r = None if vs is None else np.zeros_like(ks_r)
    q_ref, err = o.qk_norm_rope_write_ref(pick(q), pick(k), pick(v), code, to_np(wq), to_np(wk), eps,
                                          rope.cos_freqs.cpu().numpy(), rope.sin_freqs.cpu().numpy(),
                                          rope.traditional, pos.reshape(T).cpu().numpy()[toks], kp_r, vp_r, kv_code,
                                          ks_r, vs_r, code, sl_local)
    got_q = to_np(out[torch.from_numpy(bi).to(out.device), :, torch.from_numpy(li).to(out.device)])
    pg, off = torch.from_numpy(s_np // ps).to(kp.device), torch.from_numpy(s_np % ps).to(kp.device)
    ar = np.arange(n_tok)
    ok = err == 0 and np.array_equal(got_q, q_ref)
    ok = ok and np.array_equal(to_np(kp[pg, :, off]), kp_r[ar, :, s_np % ps])
    ok = ok and np.array_equal(to_np(vp[pg, :, off]), vp_r[ar, :, s_np % ps])
    if ks is not None:
        ok = ok and np.array_equal(to_np(ks[pg, :, off]), ks_r[ar, :, s_np % ps])
        ok = ok and np.array_equal(to_np(vs[pg, :, off]), vs_r[ar, :, s_np % ps])
    ok = bool(ok)
    if not ok:
        _PARITY_FAILED.append("qk prep")
    return {"ok": ok, "rows_checked": n_tok, "checked": f"{n_tok} tokens: q out, K / V rows"
            + (" and int8 scales" if ks is not None else "") + " at their slots (bit-exact)"}


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
        times, _ = time_launches(
            lambda: qk_norm_rope_write(q, k, v, wq, wk, rope, pos, kp, vp, slots, eps=1e-6, key_scales=ks,
                                       value_scales=vs, out=out), iters, warmup, flush)
        ms = statistics.median(times)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res.append(dict(workload=f"qk-norm+RoPE+KV write, {T} tokens (config2a shape), {kv} pages",
                        metric="qk-prep GB/s", value=round(gbs, 1), unit="GB/s", ms=round(ms, 4),
                        bytes=nbytes, spread=spread(times, nbytes, 1e9), roofline_frac=round(gbs / peaks["hbm"], 4),
                        l2="flushed", parity=_qk_prep_parity(q, k, v, wq, wk, rope, pos, kp, vp, ks, vs, slots, out,
                                                             1e-6)))
        del kp, vp, ks, vs
    return res


def _single_line(r: dict, args, peaks: dict, bound: str, extra: dict | None = None) -> dict:
    line = {"metric": r["metric"], "value": r["value"], "unit": r["unit"], "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True, "dtype": "bf16",
            "config": {"workload": r["workload"], "l2": "flushed between launches"},
            "roofline": {"bound": bound, "achieved": r["value"], "peak": peaks["hbm" if bound == "hbm" else "bf16"],
                         "unit": r["unit"], "frac": r["roofline_frac"], "peak_source": peaks["src"]},
            "spread": r.get("spread"), "parity": r.get("parity")}
    if "bytes" in r:
        line["roofline"]["algorithmic_bytes"] = r["bytes"]
    line.update(extra or {})
    return line


def run_qkprep(args):
    """The fused q/k-norm + RoPE + K/V write alone (bf16 or, with --kv int8, int8 pools),
    4 x 2048 tokens unless --batch says otherwise; one JSON line."""
    from nano_vllm_b200 import _native as nv

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    peaks = measured_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    r = qk_prep_results(peaks, device, flush, B=args.batch or 4, iters=args.steps, warmup=args.warmup,
                        kinds=(args.kv,))[0]
    print(json.dumps(_single_line(r, args, peaks, "hbm", {"device_error_word": nv.device_error(device)})), flush=True)


def run_shortdec(args):
    """Paged decode at the decode-step shape (B = 64 and 128, or --batch), single launch
    and back to back in a CUDA graph; one JSON line per batch."""
    from nano_vllm_b200 import _native as nv

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    peaks = measured_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for r in short_decode_results(peaks, device, flush, batches=(args.batch,) if args.batch else (64, 128)):
        extra = {k: r[k] for k in ("graph_us_per_launch", "graph_gbs", "graph_roofline_frac", "graph")}
        extra["device_error_word"] = nv.device_error(device)
        print(json.dumps(_single_line(r, args, peaks, "hbm", extra)), flush=True)


def run_w4a16(args):
    """The W4A16 matmul alone at Qwen3-4B's gate+up projection shape (M = --batch or 1
    activation rows); one JSON line."""
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    peaks = measured_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    r = w4a16_results(peaks, device, flush, shapes=(("gate_up", 2 * 9728, 2560),), ms_rows=(args.batch or 1,),
                      iters=args.steps, warmup=args.warmup)[0]
    print(json.dumps(_single_line(r, args, peaks, "hbm")), flush=True)


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
    times, out = time_launches(lambda: flash_attention(q, k, v, mask="causal", out_dtype=torch.bfloat16),
                               args.steps, args.warmup, flush)
    ms = statistics.median(times)
    tf = flops / (ms * 1e-3) / 1e12
    rng = np.random.default_rng(12)
    pairs = [(int(b), int(h)) for b, h in zip(rng.integers(0, B, 8), rng.choice(Hq, 8, replace=False))]
    r = dict(metric="prefill attn TFLOPS", value=round(tf, 1), unit="TFLOP/s", ms=round(ms, 4),
             workload=f"config2a dense causal prefill {B}x{L}, 32q/8kv, d128", roofline_frac=round(tf / peaks["bf16"], 4),
             spread=spread(times, flops, 1e12), parity=parity_dense(q, k, v, out, pairs))
    print(json.dumps(_single_line(r, args, peaks, "tensor", {"device_error_word": nv.device_error(device)})),
          flush=True)


def run_chunked(args):
    """Config 2b alone: 4 x 512 new tokens against --prior paged tokens; one JSON line."""
    from nano_vllm_b200 import _native as nv

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    peaks = measured_peaks()
    c = args.prior
    cfg = chunk_config(c)
    w = build_decode(cfg, 0, 1, device)
    flops = 4 * 128 * 32 * 4 * sum(c + r + 1 for r in range(512))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    times, out = time_launches(lambda: run_decode_step(w), args.steps, args.warmup, flush)
    ms = statistics.median(times)
    tf = flops / (ms * 1e-3) / 1e12
    r = dict(metric="prefill attn TFLOPS", value=round(tf, 1), unit="TFLOP/s", ms=round(ms, 4),
             workload=f"config2b chunked prefill 512 vs {c} paged", roofline_frac=round(tf / peaks["bf16"], 4),
             spread=spread(times, flops, 1e12),
             parity=parity_paged(w, out, np.array([0, 3]), one_head_per_group(32, 8)))
    print(json.dumps(_single_line(r, args, peaks, "tensor", {"device_error_word": nv.device_error(device)})),
          flush=True)


def run_step(args):
    """The 36-layer decode-step attention path alone (--steps timed steps); one JSON line."""
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    r = decode_step_results(device, B=args.batch or 64, steps=args.steps)
    line = {"metric": r["metric"], "value": r["value"], "unit": r["unit"], "n_gpus": 1, "steps": args.steps,
            "warmup": 3, "higher_is_better": False, "dtype": "bf16", "config": {"workload": r["workload"]},
            "eager_us": r["eager_us"], "parity": r["parity"]}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch.distributed as dist

    if args.config == "c2a":
        return run_prefill(args)
    if args.config == "c2b":
        return run_chunked(args)
    if args.config == "step":
        return run_step(args)
    if args.config == "qkprep":
        return run_qkprep(args)
    if args.config == "w4a16":
        return run_w4a16(args)
    if args.config == "shortdec":
        return run_shortdec(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        # NCCL's init log (one line per rank and channel setup) shows the ranks it joined
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")  # keep stdout for the JSON line
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
    out = None
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            evs[i][0].record(stream)
            out = run_decode_step(w)
            evs[i][1].record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms_total = t0.elapsed_time(t1)
    launch_times = [s.elapsed_time(e) for s, e in evs]
    launch_ms = statistics.mean(launch_times)
    from nano_vllm_b200 import _native as nv

    dev_err = nv.device_error(device)
    # parity of the last timed launch, on this rank's shard (every rank takes this step)
    par = parity_paged(w, out, sample_rows(cfg, w["q"].shape[0], w["shard"].b_lo, seed=7))
    t = torch.tensor([ms_total, float(w["bytes"]["total"]), float(dev_err), float(w["bytes"]["total_unique"]),
                      0.0 if par["ok"] else 1.0, par["max_abs"]], dtype=torch.float64, device=device)
    per_rank = [launch_ms]
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax[0:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(tmax[1:2], op=dist.ReduceOp.SUM)
        dist.all_reduce(tmax[2:3], op=dist.ReduceOp.MAX)
        dist.all_reduce(tmax[3:4], op=dist.ReduceOp.SUM)
        dist.all_reduce(tmax[4:6], op=dist.ReduceOp.MAX)
        t = tmax
        g = [torch.zeros(1, dtype=torch.float64, device=device) for _ in range(world)]
        dist.all_gather(g, torch.tensor([launch_ms], dtype=torch.float64, device=device))
        per_rank = [float(x.item()) for x in g]
    ms_per_step = float(t[0]) / args.steps
    total_bytes = float(t[1])
    value = total_bytes / (ms_per_step * 1e-3) / 1e9
    value_unique = float(t[3]) / (ms_per_step * 1e-3) / 1e9
    if world > 1:
        par = dict(par, ok=bool(t[4] == 0), max_abs=float(t[5]), ranks=world,
                   checked=par["checked"] + " on every rank's shard")
        if not par["ok"] and "headline" not in _PARITY_FAILED:
            _PARITY_FAILED.append("headline")

    # e2e through the public API with host buffers (every rank, max over ranks)
    e2e_ms, h2d, d2h, e2e_ok = e2e_decode(w, max(3, args.steps // 2), 2)
    et = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_value = total_bytes / (float(et[0]) * 1e-3) / 1e9

    achieved = w["bytes"]["total"] / (launch_ms * 1e-3) / 1e9
    achieved_unique = w["bytes"]["total_unique"] / (launch_ms * 1e-3) / 1e9
    roof = dict(bound="hbm", achieved=round(achieved, 1), peak=peaks["hbm"], unit="GB/s",
                frac=round(achieved / peaks["hbm"], 4), peak_source=peaks["src"],
                kernel="paged_mma_kernel (mma.sync m16n8k16, TMA-fed)",
                algorithmic_bytes_per_launch=w["bytes"]["total"],
                unique_bytes_per_launch=w["bytes"]["total_unique"],
                achieved_unique=round(achieved_unique, 1), frac_unique=round(achieved_unique / peaks["hbm"], 4))
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
        "value_unique_bytes": round(value_unique, 1),
        "spread": spread(launch_times, w["bytes"]["total"], 1e9),
        "per_rank_launch_ms": [round(x, 4) for x in per_rank],
        "rank_imbalance": round(max(per_rank) / min(per_rank), 4),
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(float(et[0]), 4), "result_copied_back": e2e_ok,
                "copies": "every step's H2D / D2H in the region, on two side streams overlapping neighbouring steps"},
        "gpu_launches": args.steps,
        "roofline": roof,
        "parity": par,
        "device_error_word": int(t[2]),
    }
    if rank == 0:
        line["clocks"] = clocks.summary()
    del w, out
    torch.cuda.empty_cache()
    cpu = world == 1 and not args.no_cpu_baseline
    if cpu:
        line["cpu_baseline"] = cpu_baseline_pair(lambda n, t_: cpu_decode_sample(cfg, n, t_), args.cpu_seconds)
    if world == 1 and not args.no_secondary:
        line["secondary"] = secondary_results(peaks, device, cpu, args.cpu_seconds_secondary)
    line["parity_failed"] = list(_PARITY_FAILED)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if _PARITY_FAILED:
        sys.exit(3)


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU path (eval_cpu, restated by the oracle)
# ---------------------------------------------------------------------------

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    o = _oracle()
    cfg = decode_config(args.config)
    cfg["name"] = f"config{args.config[1]}"
    n = o.max_threads()
    per_step = max(0.5, args.ref_seconds / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_decode_sample(cfg, n, per_step / 4)
    vals, secs = [], 0.0
    last = None
    for _ in range(args.steps):
        last = cpu_decode_sample(cfg, n, per_step)
        vals.append(last["value"])
        secs += last["seconds"]
    value = statistics.median(vals)
    one = cpu_decode_sample(cfg, 1, args.cpu_seconds)
    cpu = host_cpu()
    page = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.int8: "int8"}[cfg["dtype"]]
    line = {
        "impl": "reference", "metric": "decode-attn KV GB/s", "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs / args.steps * 1e3, 1), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": f"f32 math over {page} pages",
        "data": "synthetic (seeded; same context lengths and block tables as our arm)",
        "config": {"workload": f"{cfg['name']} paged decode" + (" + prefix sharing" if cfg["share"] else ""),
                   "model": cfg["model"], "batch": cfg["B"], "q_heads": cfg["Hq"], "kv_heads": cfg["Hkv"],
                   "head_dim": cfg["D"], "page_size": cfg["ps"], "context": str(cfg["ctx"]),
                   "shared_prefix_tokens": cfg["share"][1] if cfg["share"] else 0,
                   "parallelism": f"host CPU, {n} threads (rank 0 of {world})"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": n, "kind": "port",
                         "sample": last["sample"], "cpu_model": cpu["model"], "nproc": cpu["nproc"],
                         "single_thread": {"value": one["value"], "cores": 1, "sample": one["sample"]}},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "MLX (the reference's runtime) is not installable offline; the reference's mx.cpu path for this "
                "op is PagedAttention::eval_cpu, timed here as its C restatement (oracle/nvm_oracle.c) with "
                "OpenMP over query rows; single_thread is the same loop on one thread, as eval_cpu runs.",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c1", "c2a", "c2b", "c3", "c4", "c5", "qkprep", "w4a16", "step", "shortdec"],
                    default="c3")
    ap.add_argument("--prior", type=int, default=0, help="config 2b: paged tokens before the 512-token chunk")
    ap.add_argument("--batch", type=int, default=None, help="override the config's batch (small profiling cases)")
    ap.add_argument("--kv", choices=["bf16", "int8"], default="bf16", help="qkprep: page pool dtype")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--cpu-seconds-secondary", type=float, default=2.0)
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
