"""The C ABI library loads and exports every declared symbol; host-side validation.

No kernel is launched here: every call below fails validation (or only computes a
size) before touching a device, so these run on a CPU-only machine.
"""

import ctypes
import os
import re

import pytest
import torch

from nano_vllm_b200 import _native as nv
from nano_vllm_b200 import flash_attention, paged_attention

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nvm_attn.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(nvm_\w+)\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ["nvm_paged_attention", "nvm_paged_attention_workspace_size", "nvm_flash_attention",
              "nvm_reshape_and_cache", "nvm_paged_append", "nvm_status_string", "nvm_last_error",
              "nvm_device_error", "nvm_version"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    L = nv.lib()
    for s in declared_symbols():
        assert hasattr(L, s), s
        assert s in nv.SIGNATURES, f"{s} has no ctypes signature"
    assert nv.lib().nvm_version().decode().startswith("nvm_attn")


def test_library_has_no_torch_or_python_dependency():
    import subprocess

    out = subprocess.run(["ldd", nv.LIB_PATH], capture_output=True, text=True).stdout
    assert "libtorch" not in out and "libpython" not in out and "libc10" not in out


def test_status_strings():
    L = nv.lib()
    assert L.nvm_status_string(0) == b"NVM_OK"
    assert L.nvm_status_string(-1) == b"NVM_ERR_INVALID_ARGUMENT"
    assert L.nvm_status_string(-5) == b"NVM_ERR_DEVICE_TIMEOUT"
    assert L.nvm_status_string(-6) == b"NVM_ERR_OUT_OF_PAGES"


def _paged_call(**kw):
    args = dict(q=None, q_dtype=0, k=None, v=None, kv_dtype=2, ks=None, vs=None, sdt=1, bt=None, cl=None,
                out=None, out_dtype=0, B=1, Hq=4, Hkv=2, L=1, D=128, P=4, ps=16, mp=4, scale=0.1, causal=1)
    args.update(kw)
    a = args
    return nv.lib().nvm_paged_attention(a["q"], a["q_dtype"], a["k"], a["v"], a["kv_dtype"], a["ks"], a["vs"],
                                        a["sdt"], a["bt"], a["cl"], a["out"], a["out_dtype"], a["B"], a["Hq"],
                                        a["Hkv"], a["L"], a["D"], a["P"], a["ps"], a["mp"], a["scale"], a["causal"],
                                        None, 0, None)


def test_paged_validation_messages():
    L = nv.lib()
    assert _paged_call(Hq=3, Hkv=2) == -1
    assert L.nvm_last_error().decode() == "paged_attention: num_heads must be divisible by num_kv_heads"
    assert _paged_call(q_dtype=3) == -1
    assert L.nvm_last_error().decode().startswith("paged_attention: q must be")
    assert _paged_call(kv_dtype=4) == -1
    assert _paged_call(D=512) == -2
    assert _paged_call(kv_dtype=3) == -1  # int8 without scales
    assert L.nvm_last_error().decode().startswith("paged_attention_int8_decode:")
    assert _paged_call() == -1  # null pointers with B > 0
    assert _paged_call(B=0) == 0  # empty batch is a no-op


def test_other_entry_point_validation():
    L = nv.lib()
    assert L.nvm_flash_attention(None, None, None, 3, None, 0, 0, 0, None, 0, 1, 4, 2, 8, 8, 64, 0.1, 1, None) == -1
    assert L.nvm_last_error().decode().startswith("flash_attention:")
    assert L.nvm_reshape_and_cache(None, None, 1, 0, 0, None, None, 2, None, None, 1, None, 4, 2, 8, 4, 16,
                                   None) == -1
    assert L.nvm_last_error().decode().startswith("write_page_slice:")
    assert L.nvm_paged_append(None, None, None, None, None, None, None, None, 0, None, 5000, 4, 16, 8, None) == -1


def test_workspace_sizes():
    L = nv.lib()
    # single-chunk shapes need none; long decodes get a split-K workspace
    assert L.nvm_paged_attention_workspace_size(4, 32, 8, 2048, 128, 2048, 1, 2) == 0
    c3 = L.nvm_paged_attention_workspace_size(256, 32, 8, 1, 128, 16, 2048, 2)
    assert 0 < c3 < (1 << 30)
    # n8 decode, 64 sequences x 8 kv heads of up to 32K keys (config 4's shape): chunks of
    # 160 tiles (about six waves of 8 CTAs per SM), 13 per unit; tickets + (m, l) + O rows
    units, chunks, rows, d = 64 * 8, 13, 8, 128
    assert L.nvm_paged_attention_workspace_size(64, 64, 8, 1, d, 16, 2048, 2) == \
        (1 << 20) + units * chunks * rows * 8 + units * chunks * rows * d * 4
    assert L.nvm_paged_attention_workspace_size(16, 16, 8, 1, 4, 4, 64, 0) == 0  # generic kernel, no workspace


def test_wrappers_fail_loudly_without_cuda():
    q = torch.zeros(1, 4, 1, 8)
    kp = torch.zeros(2, 2, 4, 8)
    bt = torch.zeros(1, 2, dtype=torch.int32)
    cl = torch.ones(1, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA device"):
        paged_attention(q, kp, kp, bt, cl, 4)
    with pytest.raises(NotImplementedError):
        paged_attention(q, kp, kp, bt, cl, 4, mask=torch.zeros(1))
    with pytest.raises(RuntimeError, match="CUDA device"):
        flash_attention(q, kp[:1], kp[:1])


def test_new_entry_points_validate_before_launch():
    """Argument errors of the fused prep, the W4A16 matmul and the device page-table
    calls come back as status codes with the operator's name, without a GPU."""
    L = nv.lib()
    # fused prep: fp32 inputs are refused
    st = L.nvm_qk_norm_rope_write(None, None, None, nv.NVM_F32, 0, 0, None, None, 1e-6, None, None, 1, 0, None,
                                  None, 0, None, None, nv.NVM_F32, None, None, nv.NVM_F16, None, 1, 1, 1, 128, 1, 16,
                                  None)
    assert st == -1 and L.nvm_last_error().decode().startswith("qk_norm_rope_write:")
    # W4A16: bits and group size as the reference requires
    assert L.nvm_w4a16_matmul(None, nv.NVM_BF16, None, None, None, None, 1, 128, 4, 128, 8, None) == -1
    assert "bits must be 4" in L.nvm_last_error().decode()
    assert L.nvm_w4a16_matmul(None, nv.NVM_BF16, None, None, None, None, 1, 128, 4, 64, 4, None) == -1
    assert "group_size must be 128" in L.nvm_last_error().decode()
    assert L.nvm_w4a16_matmul(None, nv.NVM_BF16, None, None, None, None, 1, 100, 4, 128, 4, None) == -1
    assert "divisible by group_size" in L.nvm_last_error().decode()
    # device page tables: batch bound
    assert L.nvm_paged_rewind(None, None, None, None, None, None, None, None, 5000, 4, 16, 8, None) == -1
    assert L.nvm_last_error().decode().startswith("rewind:")
    assert L.nvm_paged_attach(None, None, None, None, None, None, 5000, 4, 16, 2, 8, None) == -1
    assert L.nvm_last_error().decode().startswith("attach:")


def test_new_wrappers_fail_loudly_without_cuda():
    from nano_vllm_b200.layers.linear import quantized_matmul
    from nano_vllm_b200.layers.qk_prep import qk_norm_rope_write
    from nano_vllm_b200.layers.rotary_embedding import RoPE

    a = torch.zeros(1, 128, dtype=torch.bfloat16)
    b = torch.zeros(4, 16, dtype=torch.int32)
    s = torch.ones(4, 1, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA device"):
        quantized_matmul(s, s, 128, 4, a, b, True)
    q = torch.zeros(1, 1, 4, 128, dtype=torch.bfloat16)
    kv = torch.zeros(1, 1, 2, 128, dtype=torch.bfloat16)
    w = torch.ones(128, dtype=torch.bfloat16)
    pages = torch.zeros(1, 2, 16, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA device"):
        qk_norm_rope_write(q, kv, kv, w, w, RoPE(128, 8), torch.zeros(1, 1, dtype=torch.int32), pages, pages.clone(),
                           torch.zeros(1, dtype=torch.int64))


def test_selftest_limit_validated_before_any_device_work():
    L = nv.lib()
    for bad in (0, 999, 100_000_001):
        assert L.nvm_selftest_wait_expiry(bad, None, None) == -1
        assert L.nvm_last_error().decode().startswith("selftest_wait_expiry: limit")
