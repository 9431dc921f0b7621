"""KV-head sharding across ranks (the N>1 path of bench.py) on CPU with gloo.

Two, four and eight gloo ranks each compute their shard of a paged decode with the oracle, gather
the shards on rank 0, and the stitched result must equal the unsharded oracle
output bit for bit (attention is independent per kv head, so no collective is on
the data path; the gather here is only the check).
"""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from nano_vllm_b200.sharding import kv_head_shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _problem():
    rng = np.random.default_rng(7)
    B, Hq, Hkv, L, D, ps, P = 4, 8, 4, 2, 32, 8, 24
    q = rng.standard_normal((B, Hq, L, D)).astype(np.float32)
    kp = rng.standard_normal((P, Hkv, ps, D)).astype(np.float32)
    vp = rng.standard_normal((P, Hkv, ps, D)).astype(np.float32)
    bt = rng.permutation(P)[: B * 5].reshape(B, 5).astype(np.int32)
    cl = np.array([33, 7, 40, 1], dtype=np.int32)
    return q, kp, vp, bt, cl, ps


def _worker(rank, world, port, result_path):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch
    import torch.distributed as dist
    from oracle import oracle as o

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, kp, vp, bt, cl, ps = _problem()
    B, Hq, L, D = q.shape
    Hkv = kp.shape[1]
    sh = kv_head_shard(rank, world, Hq, Hkv, B)
    part = o.paged_attention_ref(q[sh.b_lo:sh.b_hi, sh.q_lo:sh.q_hi], kp[:, sh.kv_lo:sh.kv_hi],
                                 vp[:, sh.kv_lo:sh.kv_hi], bt[sh.b_lo:sh.b_hi], cl[sh.b_lo:sh.b_hi], ps,
                                 mask="causal")
    full = np.zeros((B, Hq, L, D), dtype=np.float32)
    full[sh.b_lo:sh.b_hi, sh.q_lo:sh.q_hi] = part
    t = torch.from_numpy(full)
    dist.all_reduce(t)  # shards are disjoint: the sum stitches them
    if rank == 0:
        np.save(result_path, t.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_decode_equals_unsharded(oracle, tmp_path, world):
    # every (sequence, q head) is owned by exactly one rank (at 8 ranks the 4 kv heads
    # are also split by batch halves) ...
    q, kp, vp, bt, cl, ps = _problem()
    B, Hq = q.shape[:2]
    cover = np.zeros((B, Hq), dtype=int)
    for r in range(world):
        sh = kv_head_shard(r, world, Hq, kp.shape[1], B)
        cover[sh.b_lo:sh.b_hi, sh.q_lo:sh.q_hi] += 1
    assert (cover == 1).all()
    # ... and the stitched shards computed by `world` gloo ranks equal the unsharded result
    path = str(tmp_path / "out.npy")
    mp.start_processes(_worker, args=(world, _free_port(), path), nprocs=world, join=True, start_method="spawn")
    q, kp, vp, bt, cl, ps = _problem()
    ref = oracle.paged_attention_ref(q, kp, vp, bt, cl, ps, mask="causal")
    np.testing.assert_array_equal(np.load(path), ref)


def test_shard_shapes():
    assert kv_head_shard(1, 2, 32, 8, 256) == kv_head_shard(1, 2, 32, 8, 256)
    s = kv_head_shard(3, 8, 32, 4, 128)  # 4 kv heads on 8 ranks: head 1, second batch half
    assert (s.kv_lo, s.kv_hi, s.q_lo, s.q_hi, s.b_lo, s.b_hi) == (1, 2, 8, 16, 64, 128)
    with pytest.raises(ValueError):
        kv_head_shard(0, 3, 32, 8, 4)
