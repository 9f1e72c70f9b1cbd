"""Two-GPU tests of the key-sharded indexer's exact merge (skipped with fewer
than two GPUs): two processes, one per GPU, merge their local top-K
candidates three times in a row through

  * the P2P exchange: payloads staged in CUDA IPC slots, read by the merge
    kernel with plain peer loads after a bounded wait on the peer's seq flag
    (reference/sparse_attn_indexer.py:885-952, dsa.cu:2184-2409);
  * the NCCL all-gather followed by the fused merge kernel (sai.py:953-1006);
  * the NCCL all-gather followed by the torch.topk epilogue (sai.py:1007-1030).

Each rank's result must equal the oracle's exact merge (as sets for the torch
epilogue, whose output is not sorted). NVLS is off, the process group has a
short timeout, and a rank leaves only between merges.
"""
import datetime
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import dsa_oracle as O

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=60))
    try:
        sai = importlib.import_module("glm5-on-v100_b200.sparse_attn_indexer")
        K, R = 64, 9
        results = []
        for it in range(3):
            rng = np.random.default_rng(100 + it)
            vals = rng.standard_normal((world, R, K)).astype(np.float32)
            vals[:, 3, 10:] = -np.inf  # a row with few finite candidates
            pos = rng.permutation(100000)[: world * R * K].reshape(world, R, K).astype(np.int32)
            pend = [(0, R, torch.from_numpy(vals[rank]).cuda(), torch.from_numpy(pos[rank]).cuda())]
            out = torch.full((R, K), -9, dtype=torch.int32, device="cuda")
            shard = sai.ShardConfig(tp=world, rank=rank, cpu_group=cpu, merge=mode, rows_cap=32)
            sai.merge_shards(pend, out, K, shard)
            torch.cuda.synchronize()
            allf = np.concatenate([vals, pos.view(np.float32)], axis=2)
            results.append((out.cpu().numpy(), O.shard_merge(allf, K)))
        q.put((rank, results, bool(sai._P2P_FAILED)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["p2p", "fused", "torch"])
def test_sharded_merge_two_gpus(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()  # both ranks rendezvous on it
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for rank, results, p2p_failed in res:
        if mode == "p2p":
            assert not p2p_failed, "the P2P exchange fell back to the all-gather path"
        for got, exp in results:
            if mode == "torch":
                np.testing.assert_array_equal(np.sort(got, axis=1), np.sort(exp, axis=1))
            else:
                np.testing.assert_array_equal(got, exp)
