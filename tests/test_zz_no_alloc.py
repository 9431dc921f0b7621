"""nvm_paged_attention_noalloc: the paged-attention entry point that allocates nothing.

Some callers cannot allocate device memory on their hot path (an engine that hands all
free HBM to its KV page pools, a decode loop that cannot pay cudaMalloc's implicit
synchronisation, a host without a device allocator).  This entry point takes no
workspace and keeps its split-K scratch in an array built into the library.  The test
calls it through the C ABI on a decode whose contexts are long enough to be split
across CTAs, twice in a row (the array keeps the previous call's contents), and
compares each result with the workspace-taking entry point under the tolerance the
other parity tests use.  It lives in its own file, collected last.
"""

import pytest
import torch

from gpu_helpers import random_paged_problem
from nano_vllm_b200 import _native as nv

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=1e-2)


def _args(prob, out):
    q, kp, vp, bt, cl = prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"]
    B, Hq, L, D = q.shape
    P, Hkv, ps, _ = kp.shape
    return [q.data_ptr(), nv.dtype_code(q.dtype), kp.data_ptr(), vp.data_ptr(), nv.dtype_code(kp.dtype),
            None, None, nv.NVM_F16, bt.data_ptr(), cl.data_ptr(), out.data_ptr(), nv.NVM_F32,
            B, Hq, Hkv, L, D, P, ps, bt.shape[1], float(D) ** -0.5, 1]


def test_noalloc_matches_workspace_entry_point(cuda):
    L = nv.lib()
    gen = torch.Generator().manual_seed(77)
    prob = random_paged_problem(gen, 24, 32, 8, 1, 128, 16, torch.bfloat16, 2000, 6000)
    B, Hq, Lq, D = prob["q"].shape
    stream = nv.stream_ptr(cuda)
    ws_bytes = L.nvm_paged_attention_workspace_size(B, Hq, 8, Lq, D, 16, prob["bt"].shape[1], nv.NVM_BF16)
    assert ws_bytes > 0, "the case must exercise the split-K scratch"
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
