"""Failure detection on the GPU without a GPU fault.

Every spin-wait in the library's kernels is bounded; when one expires the kernel
records a code in the per-device error word, drains what it issued and returns.  Here
a diagnostic kernel waits, through the kernels' own bounded-wait loop, on an mbarrier
that nothing arrives on, with a 1 ms limit: the host must read code 1 from
nvm_device_error(), the word must clear, and the device must keep giving correct
results.  A wait that expired inside a split-K call may leave its tickets non-zero, so
the Python layer re-zeroes the cached workspaces after any non-zero word; the second
test plants such tickets and checks the next call.
"""

import pytest
import torch

from gpu_helpers import TOL16, assert_close, oracle_paged, random_paged_problem
from nano_vllm_b200 import paged_attention
from nano_vllm_b200 import _native as nv

pytestmark = pytest.mark.gpu
LIMIT_NS = 1_000_000  # 1 ms


def _expire(cuda):
    waited = torch.zeros(1, dtype=torch.int64, device=cuda)
    nv.check(nv.lib().nvm_selftest_wait_expiry(LIMIT_NS, waited.data_ptr(), nv.stream_ptr(cuda)))
    return waited


def test_wait_expiry_is_reported_and_cleared(cuda):
    assert nv.device_error(cuda) == 0
    waited = _expire(cuda)
    assert nv.device_error(cuda) == 1  # kDevErrFullWait: a wait for a phase expired
    assert LIMIT_NS <= int(waited.item()) < 1_000_000_000
    assert nv.device_error(cuda) == 0  # the read cleared it


def test_expiry_resets_cached_split_k_workspace(cuda, oracle):
    gen = torch.Generator().manual_seed(31)
    prob = random_paged_problem(gen, 24, 32, 8, 1, 128, 16, torch.bfloat16, 2000, 6000)
    args = (prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], prob["ps"])
    first = paged_attention(*args, mask="causal")
    assert_close(first, oracle_paged(oracle, prob), TOL16)
    ws = nv._workspaces[(cuda.index or 0, nv.stream_ptr(cuda))]
    ws[: 1 << 20].fill_(3)  # tickets as a call that gave up half way could leave them
    _expire(cuda)
    assert nv.device_error(cuda) == 1
    assert int(ws.count_nonzero()) == 0
    second = paged_attention(*args, mask="causal")
    assert torch.equal(first, second)
    assert nv.device_error(cuda) == 0
