"""Generate the committed oracle fixtures in tests/golden/ (TEST INFRASTRUCTURE).

    python tests/golden/make_golden.py

Each ``<case>.npz`` holds seeded inputs and the oracle's outputs (``out_*``).
``tests/test_oracle.py`` re-runs ``run_case`` and requires bit-identical results,
and the GPU parity tests compare the CUDA kernels against the same arrays.
bf16 tensors are stored as uint16 bit patterns with ``*_is_bf16`` flags.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _pool(rng, P, H, ps, D, kind):
    if kind == "f32":
        return rng.standard_normal((P, H, ps, D)).astype(np.float32)
    if kind == "f16":
        return rng.standard_normal((P, H, ps, D)).astype(np.float16)
    from oracle import oracle as o

    return o.f32_to_bf16_bits(rng.standard_normal((P, H, ps, D)).astype(np.float32))


def make_cases():
    from oracle import oracle as o

    cases = {}
    rng = np.random.default_rng(1234)

    # paged fp16 decode with a hole, an empty sequence and a clipped context
    P, H, ps, D = 12, 2, 16, 64
    cases["paged_f16_decode"] = dict(
        kind=np.array("paged"), q=rng.standard_normal((4, 8, 1, D)).astype(np.float32),
        k=_pool(rng, P, H, ps, D, "f16"), v=_pool(rng, P, H, ps, D, "f16"),
        bt=np.array([[3, 7, -1, 1], [0, 2, 4, 5], [6, -1, -1, -1], [8, 9, 10, 11]], dtype=np.int32),
        cl=np.array([50, 64, 0, 70], dtype=np.int32), causal=np.array(1), kv_is_bf16=np.array(0))
    # paged bf16 multi-token verify (L=5, causal)
    P, H, ps, D = 10, 2, 16, 128
    cases["paged_bf16_verify"] = dict(
        kind=np.array("paged"), q=rng.standard_normal((2, 8, 5, D)).astype(np.float32),
        k=_pool(rng, P, H, ps, D, "bf16"), v=_pool(rng, P, H, ps, D, "bf16"),
        bt=np.array([[9, 1, 5, 3, -1], [0, 2, 4, 6, 8]], dtype=np.int32),
        cl=np.array([61, 80], dtype=np.int32), causal=np.array(1), kv_is_bf16=np.array(1))
    # int8 decode (fp16 scales)
    P, H, ps, D = 8, 2, 16, 128
    kq = rng.integers(-127, 128, size=(P, H, ps, D), dtype=np.int8)
    vq = rng.integers(-127, 128, size=(P, H, ps, D), dtype=np.int8)
    ks = (np.abs(rng.standard_normal((P, H, ps, 1))) / 127).astype(np.float16)
    vs = (np.abs(rng.standard_normal((P, H, ps, 1))) / 127).astype(np.float16)
    cases["paged_i8_decode"] = dict(
        kind=np.array("paged_i8"), q=rng.standard_normal((2, 8, 1, D)).astype(np.float16).astype(np.float32),
        k=kq, v=vq, ks=ks, vs=vs, bt=np.array([[7, 1, 3, -1], [0, 2, 4, 6]], dtype=np.int32),
        cl=np.array([40, 64], dtype=np.int32), causal=np.array(1))
    # int8 with L=3 (the reference dequantises the pool, attention.py:204-215)
    cases["paged_i8_multi"] = dict(
        kind=np.array("paged_i8"), q=rng.standard_normal((2, 8, 3, D)).astype(np.float32),
        k=kq, v=vq, ks=ks, vs=vs, bt=np.array([[5, 4, -1, -1], [1, 2, 3, 0]], dtype=np.int32),
        cl=np.array([30, 57], dtype=np.int32), causal=np.array(1))
    # dense flash attention, fp32, additive mask and causal
    cases["flash_mask"] = dict(
        kind=np.array("flash"), q=rng.uniform(size=(2, 6, 7, 32)).astype(np.float32),
        k=rng.uniform(size=(2, 3, 9, 32)).astype(np.float32), v=rng.uniform(size=(2, 3, 9, 32)).astype(np.float32),
        mask=rng.uniform(size=(2, 6, 7, 9)).astype(np.float32), causal=np.array(0), scale=np.array(0.9, np.float32))
    cases["flash_causal"] = dict(
        kind=np.array("flash"), q=rng.standard_normal((1, 4, 40, 64)).astype(np.float32),
        k=rng.standard_normal((1, 2, 70, 64)).astype(np.float32),
        v=rng.standard_normal((1, 2, 70, 64)).astype(np.float32),
        mask=np.zeros((0,), np.float32), causal=np.array(1), scale=np.array(0.125, np.float32))
    # int8 quantiser on bf16 and fp16 rows
    x = (rng.standard_normal((3, 2, 16, 128)) * 3).astype(np.float32)
    cases["quant_bf16"] = dict(kind=np.array("quant"), x=o.f32_to_bf16_bits(x), code=np.array(2))
    cases["quant_f16"] = dict(kind=np.array("quant"), x=x.astype(np.float16), code=np.array(1))
    # fused q/k RMSNorm + RoPE + paged K/V write (Qwen3-0.6B heads 16 / 8, d 128): bf16
    # pools with halves rotation, and int8 pools (bf16 scales) with the traditional one
    T, Hq, Hkv, D, P, ps = 6, 16, 8, 128, 3, 4
    for name, kv_code, trad in [("qkprep_bf16", 2, 0), ("qkprep_i8_trad", 3, 1)]:
        cos_t, sin_t = o.rope_tables_ref(D, 64, 1000000)
        slots = rng.permutation(P * ps)[:T].astype(np.int64)
        slots[2] = -1
        cases[name] = dict(
            kind=np.array("qkprep"),
            q=o.f32_to_bf16_bits((rng.standard_normal((T, Hq, D)) * 4).astype(np.float32)),
            k=o.f32_to_bf16_bits((rng.standard_normal((T, Hkv, D)) * 2).astype(np.float32)),
            v=o.f32_to_bf16_bits(rng.standard_normal((T, Hkv, D)).astype(np.float32)),
            wq=o.f32_to_bf16_bits(rng.uniform(0.5, 1.5, D).astype(np.float32)),
            wk=o.f32_to_bf16_bits(rng.uniform(0.5, 1.5, D).astype(np.float32)),
            eps=np.array(1e-6, np.float32), cos=cos_t, sin=sin_t, trad=np.array(trad),
            pos=rng.integers(0, 64, T).astype(np.int32), slots=slots, kv_code=np.array(kv_code),
            P=np.array(P), ps=np.array(ps))
    return cases


def run_case(o, data: dict) -> dict:
    """Oracle outputs for one fixture (keys ``out_*``)."""
    kind = str(data["kind"])
    if kind == "paged":
        out = o.paged_attention_ref(data["q"], data["k"], data["v"], data["bt"], data["cl"], data["k"].shape[2],
                                    mask="causal" if int(data["causal"]) else None,
                                    kv_is_bf16=bool(int(data["kv_is_bf16"])))
        return {"out": out}
    if kind == "paged_i8":
        out = o.paged_attention_ref(data["q"], data["k"], data["v"], data["bt"], data["cl"], data["k"].shape[2],
                                    data["ks"], data["vs"], mask="causal" if int(data["causal"]) else None)
        return {"out": out}
    if kind == "flash":
        mask = "causal" if int(data["causal"]) else (data["mask"] if data["mask"].size else None)
        return {"out": o.flash_attention_ref(data["q"], data["k"], data["v"], scale=float(data["scale"]), mask=mask)}
    if kind == "quant":
        q, s = o.quantize_int8_ref(data["x"], int(data["code"]))
        return {"out_q": q, "out_s": s}
    if kind == "qkprep":
        T, Hkv, D = data["k"].shape
        P, ps, kv_code = int(data["P"]), int(data["ps"]), int(data["kv_code"])
        kp = np.zeros((P, Hkv, ps, D), dtype=np.int8 if kv_code == 3 else np.uint16)
        vp = np.zeros_like(kp)
        ks = vs = None
        if kv_code == 3:
            ks = np.zeros((P, Hkv, ps, 1), dtype=np.uint16)
            vs = np.zeros_like(ks)
        q_out, err = o.qk_norm_rope_write_ref(data["q"], data["k"], data["v"], 2, data["wq"], data["wk"],
                                              float(data["eps"]), data["cos"], data["sin"], bool(int(data["trad"])),
                                              data["pos"], kp, vp, kv_code, ks, vs, 2, data["slots"])
        assert err == 0
        out = {"out_q": q_out, "out_kp": kp, "out_vp": vp}
        if kv_code == 3:
            out.update(out_ks=ks, out_vs=vs)
        return out
    raise ValueError(kind)


def main():
    root = os.path.dirname(os.path.dirname(HERE))
    sys.path.insert(0, root)
    from oracle import oracle as o

    o.build()
    for name, data in make_cases().items():
        data.update(run_case(o, data))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **data)
        print(name, sum(v.nbytes for v in data.values()))


if __name__ == "__main__":
    main()
