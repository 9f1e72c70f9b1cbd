"""Multi-GPU tests of the key-sharded indexer's exact merge (2, 4 and 8
ranks; each skipped with fewer GPUs): one process per GPU, merge their local top-K
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
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import dsa_oracle as O

pytestmark = pytest.mark.gpu


def _rendezvous():
    """A fresh file-store path for one test's process group (no TCP port that
    a previous test's store may still hold)."""
    return os.path.join(tempfile.mkdtemp(prefix="dsa_pg_"), "store")


def _worker(rank, world, store, mode, q):
    os.environ.update(NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method="file://" + store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=60))
    try:
        sai = importlib.import_module("glm5-on-v100_b200.sparse_attn_indexer")
        K, R = 64, 9
        results = []
        shard = sai.ShardConfig(tp=world, rank=rank, cpu_group=cpu, merge=mode, rows_cap=32)
        for it in range(3):
            rng = np.random.default_rng(100 + it)
            vals = rng.standard_normal((world, R, K)).astype(np.float32)
            vals[:, 3, 10:] = -np.inf  # a row with few finite candidates
            pos = rng.permutation(100000)[: world * R * K].reshape(world, R, K).astype(np.int32)
            pend = [(0, R, torch.from_numpy(vals[rank]).cuda(), torch.from_numpy(pos[rank]).cuda())]
            out = torch.full((R, K), -9, dtype=torch.int32, device="cuda")
            sai.merge_shards(pend, out, K, shard)
            torch.cuda.synchronize()
            allf = np.concatenate([vals, pos.view(np.float32)], axis=2)
            results.append((out.cpu().numpy(), O.shard_merge(allf, K)))
        q.put((rank, results, bool(shard.p2p_failed)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["p2p", "fused", "torch"])
def test_sharded_merge_gpus(mode, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store = _rendezvous()  # both ranks rendezvous on it
    procs = [ctx.Process(target=_worker, args=(r, world, store, mode, q)) for r in range(world)]
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


def _decode_worker(rank, world, store, mode, q):
    """One rank of the key-sharded decode layer: this rank scores its key span
    of every row, the exchange merges the local top-K lists into the global
    top-K on every rank, and sparse MLA decode runs on this rank's heads."""
    os.environ.update(NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method="file://" + store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=60))
    try:
        sai = importlib.import_module("glm5-on-v100_b200.sparse_attn_indexer")
        ops = importlib.import_module("glm5-on-v100_b200.ops")
        rng = np.random.default_rng(77)  # identical inputs on every rank (replicated caches)
        B, page, n_pages, mb, Hi, H, K = 5, 64, 48, 8, 32, 64, 128
        k_rows = O.idxk_encode_rows(rng.standard_normal((n_pages * page, 128)).astype(np.float32))
        lat_rows = O.dsmla_encode_rows(rng.standard_normal((n_pages * page, 576)).astype(np.float32))
        kc = torch.from_numpy(k_rows.reshape(n_pages, page, 132)).to(dev)
        kv = torch.from_numpy(lat_rows.reshape(n_pages, page, 656)).to(dev)
        bt_np = np.stack([rng.permutation(n_pages)[:mb] for _ in range(B)]).astype(np.int32)
        seq_np = np.array([512, 500, 200, 64, 301], np.int32)  # row 2 ends before rank 1's span
        bt, seq = torch.from_numpy(bt_np).to(dev), torch.from_numpy(seq_np).to(dev)
        w = torch.from_numpy((rng.standard_normal((B, Hi)) / Hi ** 0.5).astype(np.float32)).to(dev)
        shard = sai.ShardConfig(tp=world, rank=rank, cpu_group=cpu, merge=mode, decode=True, rows_cap=16)
        h0, h1 = rank * H // world, (rank + 1) * H // world
        scale = 1.0 / np.sqrt(192.0)
        checks = []
        for it in range(3):
            qi = torch.from_numpy(rng.standard_normal((B, Hi, 128)).astype(np.float32)).to(dev).to(torch.bfloat16)
            qa = torch.from_numpy(rng.standard_normal((B, H, 576)).astype(np.float32)).to(dev).to(torch.bfloat16)
            out = torch.full((B, K), -9, dtype=torch.int32, device=dev)
            sai.decode_indexer_sharded(qi, kc, w, bt, seq, K, out, shard)
            score = torch.empty(B, mb * page, dtype=torch.float32, device=dev)
            ops.sm70_indexer_logits(score, qi, kc, w, bt, seq)  # unsharded scores, same per-key arithmetic
            q_loc = qa[:, h0:h1].contiguous()
            o = torch.empty(B, h1 - h0, 512, dtype=torch.bfloat16, device=dev)
            lse = torch.empty(B, h1 - h0, dtype=torch.float32, device=dev)
            ops.sm70_sparse_mla_decode(o, lse, q_loc, kv, out, bt, seq, scale)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            exp = O.topk_rows(score.cpu().numpy(), seq_np, K)
            o_ref, lse_ref = O.sparse_mla_decode(q_loc.float().cpu().numpy(), O.dsmla_decode_rows(lat_rows), got,
                                                 bt_np, seq_np, page, scale)
            of = o.float().cpu().numpy()
            den = np.maximum(np.linalg.norm(o_ref, axis=-1), 1e-30)
            rnd = torch.from_numpy(o_ref.astype(np.float32)).to(torch.bfloat16).float().numpy()
            excess = (np.linalg.norm(of - o_ref, axis=-1) - np.linalg.norm(rnd - o_ref, axis=-1)) / den
            checks.append((np.sort(got, axis=1), np.sort(exp, axis=1), float(excess.max()),
                           float(np.abs(lse.cpu().numpy() - lse_ref).max())))
        failed = ops.p2p_failed(dev)
        q.put((rank, checks, bool(shard.p2p_failed) or failed))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["p2p", "fused"])
def test_sharded_decode_layer_gpus(mode, world):
    """Key-sharded decode indexer (each rank scores its 1/world share of every row's keys;
    device-sequenced P2P exchange, or NCCL all-gather + fused merge) and
    head-split sparse MLA decode: every rank's global top-K equals the
    oracle's top-K over all keys, and its head slice of o / lse matches the
    oracle (2e-3 relative; bf16 output rounding included in the bound)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store = _rendezvous()
    procs = [ctx.Process(target=_decode_worker, args=(r, world, store, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for rank, checks, failed in res:
        assert not failed, "the exchange reported a failed wait"
        for got, exp, rel, dlse in checks:
            np.testing.assert_array_equal(got, exp)
            assert rel <= 2e-3, rel  # relative error beyond the bf16 output's own rounding
            assert dlse <= 2e-3, dlse
