"""nvm_paged_attention_noalloc: the paged-attention entry point that allocates nothing.

Some callers cannot allocate device memory on their hot path (an engine that hands all
free HBM to its KV page pools, a decode loop that cannot pay cudaMalloc's implicit
synchronisation, a host without a device allocator).  This entry point takes no
workspace and keeps its split-K scratch in an array built into the library.  The tests
call it through the C ABI on calls whose contexts are long enough to be split across
CTAs -- the mma.sync decode kernel, and the tcgen05 kernel's grouped mode, whose work
and exit counters also live in the scratch -- twice in a row (the array keeps the
previous call's contents), and compare each result with the workspace-taking entry
point under the tolerance the other parity tests use.  A fresh process checks the
set-up rule: the first call on a device, even one that needs no scratch, is the one
that takes the array's device memory, and later calls take none.  This file is
collected last.
"""

import os
import subprocess
import sys
import textwrap

import pytest
import torch

from gpu_helpers import random_paged_problem
from nano_vllm_b200 import _native as nv

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=1e-2)
HERE = os.path.dirname(os.path.abspath(__file__))


def _args(prob, out):
    q, kp, vp, bt, cl = prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"]
    B, Hq, L, D = q.shape
    P, Hkv, ps, _ = kp.shape
    return [q.data_ptr(), nv.dtype_code(q.dtype), kp.data_ptr(), vp.data_ptr(), nv.dtype_code(kp.dtype),
            None, None, nv.NVM_F16, bt.data_ptr(), cl.data_ptr(), out.data_ptr(), nv.NVM_F32,
            B, Hq, Hkv, L, D, P, ps, bt.shape[1], float(D) ** -0.5, 1]


# (B, Hq, Hkv, L, context range): an L = 1 decode (g * L = 4 rows per kv head, the
# mma.sync kernel; 1280 units, more than the SMs hold at once, so each is split into two
# chunks merged through the scratch) and an L = 4 verify-like call (g * L = 16 rows: the
# tcgen05 grouped mode, split over key chunks with its persistent work counters)
CASES = {"decode_mma": (160, 32, 8, 1, 600, 1000), "grouped_tcgen05": (16, 32, 8, 4, 6000, 12000)}


@pytest.mark.parametrize("case", sorted(CASES))
def test_noalloc_matches_workspace_entry_point(cuda, case):
    L = nv.lib()
    B, Hq, Hkv, Lq, lo, hi = CASES[case]
    gen = torch.Generator().manual_seed(77)
    prob = random_paged_problem(gen, B, Hq, Hkv, Lq, 128, 16, torch.bfloat16, lo, hi)
    D = prob["q"].shape[3]
    stream = nv.stream_ptr(cuda)
    ws_bytes = L.nvm_paged_attention_workspace_size(B, Hq, Hkv, Lq, D, 16, prob["bt"].shape[1], nv.NVM_BF16)
    assert ws_bytes > (1 << 20), "the case must exercise the split-K scratch beyond the tickets"
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda)
    ref = torch.empty(B, Hq, Lq, D, dtype=torch.float32, device=cuda)
    nv.check(L.nvm_paged_attention(*_args(prob, ref), ws.data_ptr(), ws_bytes, stream))
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        nv.check(L.nvm_paged_attention_noalloc(*_args(prob, out), stream))
        torch.cuda.synchronize()
        torch.testing.assert_close(out, ref, **TOL)
    assert nv.device_error(cuda) == 0


def test_noalloc_rejects_oversized_plans(cuda):
    L = nv.lib()
    # 2048 sequences x 8 kv heads of up to 512 pages: the split-K plan exceeds 32 MiB
    need = L.nvm_paged_attention_workspace_size(2048, 64, 8, 1, 128, 16, 2048, nv.NVM_BF16)
    assert need > (32 << 20)
    st = L.nvm_paged_attention_noalloc(1, nv.NVM_BF16, 1, 1, nv.NVM_BF16, None, None, nv.NVM_F16, 1, 1, 1,
                                       nv.NVM_F32, 2048, 64, 8, 1, 128, 1, 16, 2048, 0.1, 1, None)
    assert st == -3
    assert "built-in limit" in L.nvm_last_error().decode()


_FRESH_PROCESS = textwrap.dedent("""
    import sys
    import torch
    sys.path[:0] = {paths!r}
    from gpu_helpers import random_paged_problem
    from test_zz_no_alloc import _args
    from nano_vllm_b200 import _native as nv

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    gen = torch.Generator().manual_seed(5)
    short = random_paged_problem(gen, 2, 32, 8, 1, 128, 16, torch.bfloat16, 40, 60)
    long_ = random_paged_problem(gen, 160, 32, 8, 1, 128, 16, torch.bfloat16, 600, 1000)
    mp_s, mp_l = short["bt"].shape[1], long_["bt"].shape[1]
    out_s = torch.empty(2, 32, 1, 128, dtype=torch.float32, device=dev)
    out_l = torch.empty(160, 32, 1, 128, dtype=torch.float32, device=dev)
    ref = torch.empty_like(out_l)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(dev)[0]
    L = nv.lib()
    assert L.nvm_paged_attention_workspace_size(2, 32, 8, 1, 128, 16, mp_s, nv.NVM_BF16) == 0
    need = L.nvm_paged_attention_workspace_size(160, 32, 8, 1, 128, 16, mp_l, nv.NVM_BF16)
    assert 0 < need <= ws.numel()
    stream = nv.stream_ptr(dev)
    # the first call on the device needs no scratch and sets up the array all the same
    nv.check(L.nvm_paged_attention_noalloc(*_args(short, out_s), stream))
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info(dev)[0]
    nv.check(L.nvm_paged_attention(*_args(long_, ref), ws.data_ptr(), need, stream))
    for _ in range(2):
        out_l.fill_(float("nan"))
        nv.check(L.nvm_paged_attention_noalloc(*_args(long_, out_l), stream))
        torch.cuda.synchronize()
        torch.testing.assert_close(out_l, ref, atol=2e-3, rtol=1e-2)
    free2 = torch.cuda.mem_get_info(dev)[0]
    assert nv.device_error(dev) == 0
    print("taken_by_first_call_mib", (free0 - free1) / 2**20, "taken_later_mib", (free1 - free2) / 2**20)
    assert free0 - free1 >= (32 << 20), "the first call must take the scratch array's memory"
    assert free1 - free2 <= (8 << 20), "later calls must take no device memory"
""")


def test_noalloc_first_call_sets_up_the_device(cuda):
    """Fresh process: the device memory behind the array is taken by the first call,
    even one that needs no scratch; later calls that use the scratch take none and
    equal the workspace entry point."""
    paths = [HERE, os.path.join(os.path.dirname(HERE), "nano-vllm-metal_b200")]
    code = _FRESH_PROCESS.format(paths=paths)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "taken_by_first_call_mib" in r.stdout
