"""TEST INFRASTRUCTURE ONLY -- the parity checker for the CUDA hot path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module.  It wraps ``liboracle.so`` (built from ``nvm_oracle.c``,
a C restatement of the reference's ``eval_cpu`` loops) and restates in numpy /
plain Python the pieces of the reference that are Python-level:

* ``paged_attention_ref``  -- ``src/nano_vllm_metal/layers/attention.py:154-230``
  (routing: int8 + L==1 -> int8 decode loop, int8 + L>1 -> dequantise the whole
  pool to fp32 then the fp paged loop, else the fp paged loop),
* ``flash_attention_ref``  -- ``attention.py:103-151`` (mask handling),
* ``grouped_sdpa_ref``     -- ``attention.py:59-100`` (``causal_mask`` and
  ``scaled_dot_product_attention_grouped``, the reference tests' dense oracle),
* ``quantize_int8_ref``    -- ``src/nano_vllm_metal/cache/paged.py:152-158``,
* ``qk_norm_rope_write_ref`` -- ``src/nano_vllm_metal/models/qwen3.py:100-116``
  (q_norm / k_norm, RoPE of ``layers/rotary_embedding.py:74-124``, the paged write
  of K and V), with ``rope_tables_ref`` restating ``rotary_embedding.py:28-44``,
* ``PagePoolRef`` / ``PagedCacheRef`` -- the allocator and append bookkeeping of
  ``paged.py:60-75,197-210,424-459,491-559`` (page ids, page_lens, rewind),
* ``spec_accept_ref`` -- the per-request acceptance loop of speculative decoding,
  ``src/nano_vllm_metal/engine/generate.py:130-169``.

The reference itself cannot run here (MLX / Metal only) and publishes no golden
vectors; parity is pinned by re-running its own differential tests and
known-answer assertions (tests/test_oracle.py) and by tests/golden/ fixtures.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

OR_F32, OR_F16, OR_BF16, OR_I8 = 0, 1, 2, 3

_lib = None


def build(force: bool = False) -> str:
    """Compile liboracle.so from nvm_oracle.c with gcc (no CUDA involved)."""
    src = os.path.join(_HERE, "nvm_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        cmd = [
            "gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-std=c11",
            "-o", _LIB_PATH, src, "-lm",
        ]
        subprocess.check_call(cmd)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(_LIB_PATH)
        P, I64, F, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        _lib.oracle_paged_attention.argtypes = [P, P, P, I, P, P, P, I64, I64, I64, I64, I64, I64, I64, F, I, I]
        _lib.oracle_paged_attention_int8_decode.argtypes = [P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, F, I, I]
        _lib.oracle_flash_attention.argtypes = [P, P, P, P, I64, I64, I64, P, I64, I64, I64, I64, I64, I64, F, I, I]
        _lib.oracle_quantize_int8.argtypes = [P, I, I64, I64, P, P]
        _lib.oracle_qk_norm_rope_write.argtypes = [P, P, P, I, P, P, F, P, P, I64, I, P, P, P, P, I, P, P, I, P,
                                                   I64, I64, I64, I64, I64, I64]
        _lib.oracle_qk_norm_rope_write.restype = ctypes.c_int
        _lib.oracle_quantized_matmul.argtypes = [P, I, P, P, P, P, I64, I64, I64, I]
        _lib.oracle_max_threads.restype = ctypes.c_int
    return _lib


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------------------
# dtype helpers: bf16 is carried as uint16 bit patterns in numpy
# ---------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    out = ((u + rounding) >> np.uint32(16)).astype(np.uint16)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    out[nan] = ((u[nan] >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16)
    return out


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def to_f32(x: np.ndarray, dtype_code: int) -> np.ndarray:
    if dtype_code == OR_BF16:
        return bf16_bits_to_f32(x)
    return np.asarray(x).astype(np.float32)


def raw_code(x: np.ndarray, is_bf16: bool = False) -> int:
    if is_bf16:
        return OR_BF16
    if x.dtype == np.float32:
        return OR_F32
    if x.dtype == np.float16:
        return OR_F16
    if x.dtype == np.int8:
        return OR_I8
    raise TypeError(f"unsupported dtype {x.dtype}")


# ---------------------------------------------------------------------------
# attention oracles
# ---------------------------------------------------------------------------

def paged_attention_fp(q, key_pages, value_pages, kv_code, block_table, context_lens,
                       num_heads, scale, is_causal, nthreads=1):
    """PagedAttention::eval_cpu.  q [N, L, D] f32; pages raw (uint16 bits for bf16)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kp = np.ascontiguousarray(key_pages)
    vp = np.ascontiguousarray(value_pages)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    cl = np.ascontiguousarray(context_lens, dtype=np.int32)
    N, L, D = q.shape
    _, Hkv, ps, _ = kp.shape
    out = np.empty_like(q)
    lib().oracle_paged_attention(_ptr(q), _ptr(kp), _ptr(vp), kv_code, _ptr(bt), _ptr(cl), _ptr(out),
                                 N, L, D, Hkv, num_heads, ps, bt.shape[1], float(scale), int(bool(is_causal)),
                                 int(nthreads))
    return out


def paged_attention_int8_decode(q, key_pages, value_pages, key_scales_f32, value_scales_f32,
                                block_table, context_lens, num_heads, scale, is_causal, nthreads=1):
    """PagedAttentionInt8Decode::eval_cpu (L == 1)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    kp = np.ascontiguousarray(key_pages, dtype=np.int8)
    vp = np.ascontiguousarray(value_pages, dtype=np.int8)
    ks = np.ascontiguousarray(key_scales_f32, dtype=np.float32)
    vs = np.ascontiguousarray(value_scales_f32, dtype=np.float32)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    cl = np.ascontiguousarray(context_lens, dtype=np.int32)
    N, L, D = q.shape
    assert L == 1
    _, Hkv, ps, _ = kp.shape
    out = np.empty_like(q)
    lib().oracle_paged_attention_int8_decode(_ptr(q), _ptr(kp), _ptr(vp), _ptr(ks), _ptr(vs), _ptr(bt), _ptr(cl),
                                             _ptr(out), N, D, Hkv, num_heads, ps, bt.shape[1], float(scale),
                                             int(bool(is_causal)), int(nthreads))
    return out


def paged_attention_ref(query, key_pages, value_pages, block_table, context_lens, page_size,
                        key_scales=None, value_scales=None, scale=None, mask=None,
                        kv_is_bf16=False, scales_are_bf16=False, nthreads=1):
    """layers/attention.py:154-230 restated over numpy arrays.

    query [B, Hq, L, D] (any float; cast to fp32 like the reference).  Pages in
    their storage dtype (uint16 bit patterns when ``kv_is_bf16``).  Returns fp32
    [B, Hq, L, D].
    """
    if mask is not None and mask != "causal":
        raise NotImplementedError("Paged attention only supports mask=None or causal")
    B, Hq, L, D = query.shape
    Hkv = key_pages.shape[1]
    assert Hq % Hkv == 0
    factor = scale if scale is not None else 1.0 / (D ** 0.5)
    q = np.ascontiguousarray(np.asarray(query, dtype=np.float32).reshape(B * Hq, L, D))
    causal = mask == "causal"
    if key_pages.dtype == np.int8:
        assert key_scales is not None and value_scales is not None
        ks = to_f32(key_scales, OR_BF16 if scales_are_bf16 else raw_code(key_scales))
        vs = to_f32(value_scales, OR_BF16 if scales_are_bf16 else raw_code(value_scales))
        if L == 1:
            out = paged_attention_int8_decode(q, key_pages, value_pages, ks, vs, block_table, context_lens,
                                              Hq, np.float32(factor), causal, nthreads)
        else:
            kf = key_pages.astype(np.float32) * ks
            vf = value_pages.astype(np.float32) * vs
            out = paged_attention_fp(q, kf, vf, OR_F32, block_table, context_lens, Hq, np.float32(factor), causal,
                                     nthreads)
    else:
        code = OR_BF16 if kv_is_bf16 else raw_code(key_pages)
        out = paged_attention_fp(q, key_pages, value_pages, code, block_table, context_lens, Hq,
                                 np.float32(factor), causal, nthreads)
    return out.reshape(B, Hq, L, D)


def flash_attention_ref(query, key, value, scale=None, mask=None, nthreads=1):
    """layers/attention.py:103-151 + FlashAttention::eval_cpu.  All inputs fp32.

    query [B, Hq, L, E], key/value [B, Hkv, S, E]; mask None, "causal" or an array
    broadcastable to [B, Hq, L, S].
    """
    q = np.ascontiguousarray(query, dtype=np.float32)
    k = np.ascontiguousarray(key, dtype=np.float32)
    v = np.ascontiguousarray(value, dtype=np.float32)
    *batch, Hq, L, E = q.shape
    Hkv, S = k.shape[-3], k.shape[-2]
    factor = scale if scale is not None else 1.0 / (E ** 0.5)
    N = int(np.prod(batch, dtype=np.int64)) * Hq
    qf = q.reshape(N, L, E)
    kf = k.reshape(-1, S, E)
    vf = v.reshape(-1, S, E)
    is_causal = isinstance(mask, str) and mask == "causal"
    if isinstance(mask, str):
        assert mask == "causal"
        m = None
    elif mask is None:
        m = None
    else:
        m = np.ascontiguousarray(np.broadcast_to(np.asarray(mask, dtype=np.float32), (*batch, Hq, L, S))).reshape(N, L, S)
    out = np.empty((N, L, E), dtype=np.float32)
    if m is None:
        mp, sn, sl, ss = None, 0, 0, 0
    else:
        mp, sn, sl, ss = _ptr(m), L * S, S, 1
    lib().oracle_flash_attention(_ptr(qf), _ptr(kf), _ptr(vf), mp, sn, sl, ss, _ptr(out), N, L, S, E, Hkv, Hq,
                                 float(np.float32(factor)), int(is_causal), int(nthreads))
    return out.reshape(*batch, Hq, L, E)


def causal_mask_ref(L: int, S: int) -> np.ndarray:
    """attention.py:59-61: allowed = tril(ones(L, S), k=S-L); 0 where allowed, -inf elsewhere."""
    allowed = np.tril(np.ones((L, S), dtype=bool), k=S - L)
    return np.where(allowed, 0.0, -np.inf)


def grouped_sdpa_ref(query, key, value, scale=None, mask=None):
    """attention.py:64-100 (scaled_dot_product_attention_grouped), in float64."""
    q = np.asarray(query, dtype=np.float64)
    k = np.asarray(key, dtype=np.float64)
    v = np.asarray(value, dtype=np.float64)
    Hq, L, D = q.shape[-3:]
    Hkv, S, _ = k.shape[-3:]
    batch = q.shape[:-3]
    rep = Hq // Hkv
    q = q.reshape(*batch, Hkv, rep, L, D)
    k = k.reshape(*batch, Hkv, 1, S, D)
    v = v.reshape(*batch, Hkv, 1, S, D)
    factor = scale if scale is not None else 1.0 / (D ** 0.5)
    scores = np.matmul(q, np.swapaxes(k, -1, -2)) * factor
    if isinstance(mask, str):
        assert mask == "causal"
        scores = scores + causal_mask_ref(L, S)
    elif mask is not None:
        mk = np.broadcast_to(np.asarray(mask, dtype=np.float64), (*batch, Hq, L, S)).reshape(*batch, Hkv, rep, L, S)
        scores = scores + mk
    scores = scores - scores.max(axis=-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.matmul(p, v).reshape(*batch, Hq, L, D)


# ---------------------------------------------------------------------------
# int8 quantiser
# ---------------------------------------------------------------------------

def quantize_int8_ref(x: np.ndarray, in_code: int):
    """paged.py:152-158 over rows of the last axis.  Returns (int8 values, scale bits).

    ``x`` holds raw values (uint16 bit patterns for bf16).  The scale comes back in
    the input dtype's raw form: float32 array for F32, float16 for F16, uint16 bits
    for BF16.
    """
    x = np.ascontiguousarray(x)
    D = x.shape[-1]
    rows = x.size // D
    q = np.empty(x.shape, dtype=np.int8)
    if in_code == OR_F32:
        s = np.empty(x.shape[:-1] + (1,), dtype=np.float32)
    elif in_code == OR_F16:
        s = np.empty(x.shape[:-1] + (1,), dtype=np.float16)
    else:
        s = np.empty(x.shape[:-1] + (1,), dtype=np.uint16)
    lib().oracle_quantize_int8(_ptr(x), in_code, rows, D, _ptr(q), _ptr(s))
    return q, s


# ---------------------------------------------------------------------------
# fused q/k norm + RoPE + paged write
# ---------------------------------------------------------------------------

def rope_tables_ref(dims: int, seq_len: int, base: float = 10000):
    """rotary_embedding.py:28-44: fp32 cos/sin tables [seq_len, dims // 2]."""
    half = dims // 2
    positions = np.arange(seq_len, dtype=np.float32)
    dim_indices = np.arange(half, dtype=np.float32)
    inv_freqs = np.power(np.float32(base), -(dim_indices / np.float32(half))).astype(np.float32)
    freqs = np.outer(positions, inv_freqs).astype(np.float32)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def qk_norm_rope_write_ref(q, k, v, dtype_code, wq, wk, eps, cos_t, sin_t, traditional, positions,
                           k_pages, v_pages, kv_code, k_scales, v_scales, scale_code, slots):
    """qwen3.py:100-116 restated in C (nvm_oracle.c).  q [T, Hq, D], k/v [T, Hkv, D] raw
    values of dtype_code (uint16 bits for bf16); wq/wk [D] raw or None (RoPE only);
    cos_t/sin_t fp32 [rows, D/2]; positions int32 [T]; slots int64 [T].  The pools
    [P, Hkv, page_size, D] (and the int8 scales [P, Hkv, page_size, 1]) are written in
    place.  Returns (q_out [T, Hq, D] raw, error flag)."""
    q = np.ascontiguousarray(q)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    P, _, ps, _ = k_pages.shape
    for a in (k_pages, v_pages, k_scales, v_scales):
        if a is not None and not a.flags.c_contiguous:
            raise ValueError("pools and scales must be C-contiguous (written in place)")
    cos_t = np.ascontiguousarray(cos_t, dtype=np.float32)
    sin_t = np.ascontiguousarray(sin_t, dtype=np.float32)
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    sl = np.ascontiguousarray(slots, dtype=np.int64)
    wq_c = None if wq is None else np.ascontiguousarray(wq)
    wk_c = None if wk is None else np.ascontiguousarray(wk)
    q_out = np.empty_like(q)
    err = lib().oracle_qk_norm_rope_write(
        _ptr(q), _ptr(k), _ptr(v), dtype_code, None if wq_c is None else _ptr(wq_c),
        None if wk_c is None else _ptr(wk_c), float(eps), _ptr(cos_t), _ptr(sin_t), cos_t.shape[0],
        1 if traditional else 0, _ptr(pos), _ptr(q_out), _ptr(k_pages), _ptr(v_pages), kv_code,
        None if k_scales is None else _ptr(k_scales), None if v_scales is None else _ptr(v_scales), scale_code,
        _ptr(sl), T, Hq, Hkv, D, P, ps)
    return q_out, int(err)


# ---------------------------------------------------------------------------
# W4A16 quantized matmul
# ---------------------------------------------------------------------------

def quantized_matmul_ref(a, dtype_code, b, scales, biases, nthreads=1):
    """QuantizedMatmul::eval_cpu (quantized_matmul.cpp:80-148).  a [M, N] raw (uint16
    bits for bf16), b [K, N / 8] uint32, scales / biases [K, N / 128] raw.  Returns the
    raw [M, K] output."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b, dtype=np.uint32)
    sc = np.ascontiguousarray(scales)
    bi = np.ascontiguousarray(biases)
    M, N = a.shape
    K = b.shape[0]
    out = np.empty((M, K), dtype=a.dtype)
    lib().oracle_quantized_matmul(_ptr(a), dtype_code, _ptr(b), _ptr(sc), _ptr(bi), _ptr(out), M, N, K, nthreads)
    return out


def quantize_w4_ref(w: np.ndarray, group_size: int = 128):
    """Affine 4-bit quantisation of float32 weights [K, N] per group: scale = (max - min) / 15,
    bias = min, q = round((w - bias) / scale) clipped to [0, 15]; returns (packed uint32
    [K, N / 8], scales, biases) as float32 (test-input generator, not the reference's)."""
    K, N = w.shape
    g = w.reshape(K, N // group_size, group_size)
    lo, hi = g.min(-1), g.max(-1)
    scale = np.where(hi > lo, (hi - lo) / 15.0, 1.0).astype(np.float32)
    q = np.clip(np.rint((g - lo[..., None]) / scale[..., None]), 0, 15).astype(np.uint32).reshape(K, N)
    packed = np.zeros((K, N // 8), dtype=np.uint32)
    for j in range(8):
        packed |= q[:, j::8] << np.uint32(4 * j)
    return packed, scale, lo.astype(np.float32)


# ---------------------------------------------------------------------------
# speculative-decoding acceptance (pure Python)
# ---------------------------------------------------------------------------

def spec_accept_ref(candidates, verified, eos_id=None, budget=None):
    """The acceptance loop of speculative_generate (engine/generate.py:130-169) for one
    request: candidates = [last token, drafts...], verified = the target's argmax at
    each position.  Returns (emitted tokens, next token or None, target rewind, draft
    rewind, finished).  budget = tokens the request may still emit (None = unlimited),
    standing for the reference's max_tokens check after every emitted token."""
    k1 = len(candidates)
    comparable = [candidates[0]] + list(verified[:-1])
    emitted = []
    for i in range(k1):
        if comparable[i] != candidates[i]:
            rejected = k1 - i  # generate.py:145-153
            nxt = comparable[i]
            return emitted, nxt, rejected, rejected - 1, eos_id is not None and nxt == eos_id
        if eos_id is not None and comparable[i] == eos_id:  # _decode_one returns False
            return emitted, None, 0, 0, True
        emitted.append(comparable[i])
        if budget is not None and len(emitted) >= budget:  # max_tokens reached
            return emitted, None, 0, 0, True
    return emitted, verified[-1], 0, 0, False


# ---------------------------------------------------------------------------
# allocator / append bookkeeping (pure Python, no storage)
# ---------------------------------------------------------------------------

class PagePoolRef:
    """TinyKvPagedPool bookkeeping (paged.py:29-75,96-122,197-210) without storage."""

    def __init__(self, page_size: int):
        self.page_size = page_size
        self.free_page_ids: list[int] = []
        self.used_page_ids: set[int] = set()
        self.num_allocated_pages = 0
        self.ref_counts: dict[int, int] = {}
        self.capacity = 0

    @property
    def num_pages(self) -> int:
        return self.num_allocated_pages

    def allocate_page(self) -> int:
        if self.free_page_ids:
            pid = self.free_page_ids.pop()
        else:
            pid = self.num_pages
            self.num_allocated_pages += 1
        self.used_page_ids.add(pid)
        self.ref_counts[pid] = 1
        return pid

    def incref(self, pid: int) -> None:
        if pid not in self.used_page_ids:
            raise ValueError(f"Page {pid} is free")
        self.ref_counts[pid] += 1

    def free_page(self, pid: int) -> None:
        if pid not in self.used_page_ids:
            raise ValueError(f"Page {pid} is already free")
        self.ref_counts[pid] -= 1
        if self.ref_counts[pid] > 0:
            return
        del self.ref_counts[pid]
        self.used_page_ids.remove(pid)
        self.free_page_ids.append(pid)

    def grow_capacity(self) -> int:
        """_ensure_page_storage's capacity policy (paged.py:102-122)."""
        if self.capacity >= self.num_pages:
            return self.capacity
        if self.num_pages <= 16:
            self.capacity = self.num_pages
        else:
            self.capacity = max(self.num_pages, self.capacity * 2)
        return self.capacity


class PagedCacheRef:
    """TinyKvPagedCache bookkeeping (paged.py:407-459,491-559).  Records writes."""

    def __init__(self, pool: PagePoolRef):
        self.pool = pool
        self.page_size = pool.page_size
        self.page_ids: list[int] = []
        self.page_lens: list[int] = []
        self.offset = 0

    @property
    def num_pages(self) -> int:
        return len(self.page_ids)

    def append_chunk(self, S: int) -> list[int]:
        """Returns the slot (page_id*page_size + offset) of each of the S new tokens."""
        slots: list[int] = []
        start = 0
        if self.page_ids and self.page_lens[-1] < self.page_size:
            pid = self.page_ids[-1]
            page_start = self.page_lens[-1]
            take = min(self.page_size - page_start, S)
            self.pool.grow_capacity()
            slots += [pid * self.page_size + page_start + i for i in range(take)]
            self.page_lens[-1] += take
            start += take
        while start < S:
            end = min(start + self.page_size, S)
            pid = self.pool.allocate_page()
            self.pool.grow_capacity()
            slots += [pid * self.page_size + i for i in range(end - start)]
            self.page_ids.append(pid)
            self.page_lens.append(end - start)
            start = end
        self.offset += S
        return slots

    def block_table(self, max_pages: int | None = None) -> list[list[int]]:
        if max_pages is None:
            max_pages = self.num_pages
        assert max_pages >= self.num_pages
        return [self.page_ids + [-1] * (max_pages - self.num_pages)]

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

    def attach(self, pages: list[int]) -> None:
        """PrefixCache.attach for this layer (paged.py:305-328): a fresh cache takes shared
        full pages, each gaining a reference."""
        assert self.offset == 0 and self.num_pages == 0, "attach expects a fresh cache"
        for pid in pages:
            self.pool.incref(pid)
            self.page_ids.append(pid)
            self.page_lens.append(self.page_size)
        self.offset = len(pages) * self.page_size


class PagedStoreRef:
    """Numpy page storage with the reference's semantics (paged.py:96-195,461-475).

    Bookkeeping comes from ``PagePoolRef``; storage grows to the pool's capacity
    (zero pages, unit scales, old pages copied); ``kv_bits=8`` stores int8 pages
    plus scales in the input dtype via ``quantize_int8_ref``.  Values are raw
    arrays (uint16 bit patterns for bf16 when ``is_bf16``).
    """

    def __init__(self, page_size: int, kv_bits: int | None = None, is_bf16: bool = False):
        self.pool = PagePoolRef(page_size)
        self.kv_bits = kv_bits
        self.is_bf16 = is_bf16
        self.key_pages = None
        self.value_pages = None
        self.key_scales = None
        self.value_scales = None

    def _ensure(self, H: int, D: int, dtype) -> None:
        cap = self.pool.capacity
        if self.key_pages is not None and self.key_pages.shape[0] == cap:
            return
        sdt = np.int8 if self.kv_bits == 8 else dtype
        nk = np.zeros((cap, H, self.pool.page_size, D), dtype=sdt)
        nv_ = np.zeros_like(nk)
        if self.key_pages is not None:
            old = self.key_pages.shape[0]
            nk[:old], nv_[:old] = self.key_pages, self.value_pages
        self.key_pages, self.value_pages = nk, nv_
        if self.kv_bits == 8:
            one = np.uint16(0x3F80) if self.is_bf16 else np.dtype(dtype).type(1)
            nks = np.full((cap, H, self.pool.page_size, 1), one, dtype=dtype)
            nvs = nks.copy()
            if self.key_scales is not None:
                old = self.key_scales.shape[0]
                nks[:old], nvs[:old] = self.key_scales, self.value_scales
            self.key_scales, self.value_scales = nks, nvs

    def write(self, cache: "PagedCacheRef", key: np.ndarray, value: np.ndarray) -> list[int]:
        """Append key/value [1, H, S, D] to ``cache``; returns the slots written."""
        _, H, S, D = key.shape
        slots = cache.append_chunk(S)
        self._ensure(H, D, key.dtype)
        ps = self.pool.page_size
        code = OR_BF16 if self.is_bf16 else raw_code(key)
        for i, slot in enumerate(slots):
            pid, off = divmod(slot, ps)
            if self.kv_bits == 8:
                qk, sk = quantize_int8_ref(np.ascontiguousarray(key[0, :, i, :]), code)
                qv, sv = quantize_int8_ref(np.ascontiguousarray(value[0, :, i, :]), code)
                self.key_pages[pid, :, off, :], self.value_pages[pid, :, off, :] = qk, qv
                self.key_scales[pid, :, off, :], self.value_scales[pid, :, off, :] = sk, sv
            else:
                self.key_pages[pid, :, off, :] = key[0, :, i, :]
                self.value_pages[pid, :, off, :] = value[0, :, i, :]
        return slots

    def gather_dense(self, cache: "PagedCacheRef"):
        """Dense [1, H, offset, D] K/V (fp32 dequantised for int8, like read_page)."""
        ks, vs = [], []
        for pid, plen in zip(cache.page_ids, cache.page_lens):
            if self.kv_bits == 8:
                sc = OR_BF16 if self.is_bf16 else raw_code(self.key_scales)
                k = self.key_pages[pid:pid + 1].astype(np.float32) * to_f32(self.key_scales[pid:pid + 1], sc)
                v = self.value_pages[pid:pid + 1].astype(np.float32) * to_f32(self.value_scales[pid:pid + 1], sc)
            else:
                k, v = self.key_pages[pid:pid + 1], self.value_pages[pid:pid + 1]
            ks.append(k[:, :, :plen])
            vs.append(v[:, :, :plen])
        return np.concatenate(ks, axis=2), np.concatenate(vs, axis=2)
