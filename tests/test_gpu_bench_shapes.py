"""GPU parity at the sizes bench.py times (not reduced shapes).

The split-K chunk planner, the six-wave sizing of the decode kernel and the persistent
longest-first work list of the grouped tcgen05 mode all depend on the batch and the
longest context, so the launches the benchmark times are checked here as they are:
the workloads come from bench.py's own builders (same seeds, sizes, block tables and
shared-prefix layout), and the output of the call is compared with the oracle on the
pages of a seeded sample of sequences (config 3: two whole 16-sequence shared-prefix
groups), or on a sample of heads over all rows for prefill.  Tolerance: the
north-star max-abs 2e-3 / rel 1e-2.
"""

import numpy as np
import pytest
import torch

import bench
from nano_vllm_b200 import flash_attention
from nano_vllm_b200 import _native as nv

pytestmark = pytest.mark.gpu


def _check(par):
    assert par["ok"], par
    assert par["rows_checked"] > 0


@pytest.mark.parametrize("name", ["c1", "c3", "c4", "c5"])
def test_decode_configs_at_bench_size(cuda, name):
    cfg = bench.decode_config(name)
    w = bench.build_decode(cfg, 0, 1, cuda)
    out = bench.run_decode_step(w)
    torch.cuda.synchronize()
    for seed in (7, 11):  # the samples bench.py checks (headline, secondary lines)
        _check(bench.parity_paged(w, out, bench.sample_rows(cfg, cfg["B"], 0, seed=seed)))
    again = bench.run_decode_step(w)  # tickets left zero: a second call is identical
    assert torch.equal(out, again)
    assert nv.device_error(cuda) == 0


@pytest.mark.parametrize("world,rank", [(8, 0), (8, 7), (4, 1), (2, 0)])
def test_config3_rank_shards(cuda, world, rank):
    """One rank's kv-head shard of config 3 as the multi-GPU bench builds it (the planner
    sizes its chunks from the shard's units, e.g. the 128-tile floor at 8 ranks)."""
    cfg = bench.decode_config("c3")
    w = bench.build_decode(cfg, rank, world, cuda)
    out = bench.run_decode_step(w)
    torch.cuda.synchronize()
    _check(bench.parity_paged(w, out, bench.sample_rows(cfg, w["q"].shape[0], w["shard"].b_lo, seed=7)))
    assert nv.device_error(cuda) == 0


def test_dense_prefill_config2a_full_shape(cuda):
    gen = torch.Generator(device=cuda)
    gen.manual_seed(5)
    B, Hq, Hkv, L, D = 4, 32, 8, 2048, 128
    q = torch.randn(B, Hq, L, D, generator=gen, device=cuda).bfloat16()
    k = torch.randn(B, Hkv, L, D, generator=gen, device=cuda).bfloat16()
    v = torch.randn(B, Hkv, L, D, generator=gen, device=cuda).bfloat16()
    out = flash_attention(q, k, v, mask="causal", out_dtype=torch.bfloat16)
    rng = np.random.default_rng(12)
    pairs = [(int(b), int(h)) for b, h in zip(rng.integers(0, B, 8), rng.choice(Hq, 8, replace=False))]
    _check(bench.parity_dense(q, k, v, out, pairs))
    assert nv.device_error(cuda) == 0


@pytest.mark.parametrize("prior", [0, 512, 4096])
def test_chunked_prefill_config2b(cuda, prior):
    cfg = bench.chunk_config(prior)
    w = bench.build_decode(cfg, 0, 1, cuda)
    out = bench.run_decode_step(w)
    _check(bench.parity_paged(w, out, np.array([0, 3]), bench.one_head_per_group(32, 8)))
    assert nv.device_error(cuda) == 0
