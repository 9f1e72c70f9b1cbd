"""Host logic of the indexer orchestration and the MLA glue, on CPU (no GPU):
shard spans, sub-blocks, payload packing, merge destinations, the torch merge
epilogue, spec-row expansion, per-token prefill metadata, the P2P exchange's
slot and flag protocol against a fake IPC backend (two ranks as threads), a
schedule model of the decode exchange's slot reuse, and the key-sharded merge
across two gloo ranks (separate processes).

Mirrors the reference's orchestration (reference/sparse_attn_indexer.py:
44-106, :726-1030; reference/triton_mla.py:261-279, :414-466).
"""
import importlib
import os
import socket
import threading
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import dsa_oracle as O

sai = importlib.import_module("glm5-on-v100_b200.sparse_attn_indexer")
mla = importlib.import_module("glm5-on-v100_b200.mla_sparse")


# ------------------------------------------------------------ pure helpers
@pytest.mark.parametrize("max_kv,tp,page", [(65536, 4, 64), (180224, 8, 64), (1000, 3, 16), (64, 8, 64)])
def test_shard_span_covers_keys_contiguously(max_kv, tp, page):
    spans = [sai.shard_span(max_kv, tp, r, page) for r in range(tp)]
    assert spans == [O.shard_span(max_kv, tp, r, page) for r in range(tp)]
    per = spans[0][1]
    assert per % max(64, page) == 0
    covered = 0
    for r, (off, span) in enumerate(spans):
        assert off == r * per and span >= page
        if off < max_kv:
            assert off == covered
            covered = min(max_kv, off + span)
    assert covered == max_kv


def test_sub_blocks_tile_the_segment():
    for lo, hi, kv in [(0, 65536, 65536), (5, 7000, 180224), (0, 100, 64)]:
        blocks = list(sai.sub_blocks(lo, hi, kv))
        assert blocks[0][0] == lo and blocks[-1][1] == hi
        assert all(a2 == b1 for (_, b1), (a2, _) in zip(blocks, blocks[1:]))
        rows = blocks[0][1] - blocks[0][0]
        assert rows >= min(128, hi - lo)
        assert rows * kv * 4 <= max(sai.SCORE_BUDGET_BYTES, 128 * kv * 4)


def test_request_bounds():
    c1 = sai.PrefillChunk(0, torch.zeros(5), torch.zeros(5), torch.zeros(1, 4), 1)
    assert sai.request_bounds(c1, 5) == [0, 5]
    c2 = sai.PrefillChunk(0, torch.zeros(9), torch.zeros(9), torch.zeros(2, 4), 2, query_start_loc_cpu=[0, 4, 9])
    assert sai.request_bounds(c2, 9) == [0, 4, 9]
    c3 = sai.PrefillChunk(0, torch.zeros(9), torch.zeros(9), torch.zeros(2, 4), 2)
    with pytest.raises(RuntimeError):
        sai.request_bounds(c3, 9)


def test_pack_payload_and_destination():
    K = 4
    pend = [(10, 2, torch.arange(8, dtype=torch.float32).view(2, 4), torch.arange(100, 108, dtype=torch.int32).view(2, 4)),
            (12, 1, torch.full((1, 4), 5.0), torch.full((1, 4), 7, dtype=torch.int32))]
    f = sai.pack_payload(pend, K, "cpu")
    assert f.shape == (3, 8)
    assert torch.equal(f[:2, :4], pend[0][2])
    assert torch.equal(f[:2, 4:].contiguous().view(torch.int32), pend[0][3])
    dst, base = sai.destination(pend, "cpu")
    assert dst.numel() == 0 and base == 10
    pend2 = [pend[0], (20, 1, pend[1][2], pend[1][3])]
    dst, base = sai.destination(pend2, "cpu")
    assert base == -1 and dst.tolist() == [10, 11, 20]


def test_torch_merge_epilogue_matches_reference_restatement():
    rng = np.random.default_rng(3)
    tp, R, K = 3, 5, 16
    vals = rng.standard_normal((tp, R, K)).astype(np.float32)
    vals[1, 2, :5] = -np.inf
    pos = np.stack([rng.permutation(1000)[:K] + 1000 * s for s in range(tp) for _ in range(R)]).reshape(tp, R, K)
    allf = np.concatenate([vals, pos.astype(np.int32).view(np.float32)], axis=2)
    got = sai.torch_merge_epilogue(torch.from_numpy(allf), K).numpy()
    np.testing.assert_array_equal(np.sort(got, axis=1), O.shard_merge_torch_epilogue(allf, K))
    np.testing.assert_array_equal(np.sort(got, axis=1), O.shard_merge(allf, K))


def test_expand_spec_rows():
    seq = torch.tensor([10, 20], dtype=torch.int32)
    bt = torch.tensor([[1, 2], [3, 4]], dtype=torch.int32)
    s, b = mla.expand_spec_rows(seq, bt, 2)
    assert torch.equal(s, seq) and torch.equal(b, bt)
    s, b = mla.expand_spec_rows(seq, bt, 6)  # next_n = 3 verify tokens per request
    assert s.tolist() == [8, 9, 10, 18, 19, 20]
    assert b.tolist() == [[1, 2]] * 3 + [[3, 4]] * 3
    with pytest.raises(RuntimeError):
        mla.expand_spec_rows(seq, bt, 5)


def test_per_token_metadata():
    qsl = torch.tensor([0, 3, 7], dtype=torch.int32)
    bt = torch.tensor([[5, 6], [7, 8]], dtype=torch.int32)
    chunks = [(2, 4, torch.tensor([1, 2, 3, 1])), (6, 3, torch.tensor([2, 3, 4]))]
    seq, rows = mla.per_token_metadata(chunks, 2, 7, qsl, bt)
    assert seq.tolist() == [1, 2, 3, 1, 2, 3, 4]
    assert rows.tolist() == [[5, 6]] * 3 + [[7, 8]] * 4
    with pytest.raises(RuntimeError):
        mla.per_token_metadata(chunks, 2, 8, qsl, bt)  # chunks do not tile [2, 10)
    with pytest.raises(RuntimeError):
        mla.per_token_metadata(None, 0, 1, qsl, bt)


# ------------------------------------------- P2P exchange, fake IPC backend
class FakeIPC:
    """CPU stand-in for the IPC ops of ops.py: buffers in a shared registry,
    device waits as bounded host polls that set an error word on expiry (as
    the device waits do), the merges by the oracle. A rank built with
    stall_staged=True never publishes its staged flag (a stuck peer)."""

    registry: dict = {}
    lock = threading.Lock()

    def __init__(self, rank, timeout_s=5.0, stage_delay_s=0.0):
        self.rank, self.n_alloc, self.timeout_s = rank, 0, timeout_s
        self.stage_delay_s = stage_delay_s
        self.err = 0
        self.merges_p2p = 0

    @staticmethod
    def key(rank, i):
        return 1000 * (rank + 1) + i

    def sm70_ipc_alloc(self, nbytes):
        k = self.key(self.rank, self.n_alloc)
        self.n_alloc += 1
        buf = torch.zeros(nbytes, dtype=torch.uint8)
        with self.lock:
            self.registry[k] = buf
            self.registry[buf.data_ptr()] = buf
        return buf, torch.tensor(list(k.to_bytes(64, "little")), dtype=torch.uint8)

    def sm70_ipc_open(self, handle):
        return int.from_bytes(bytes(handle.numpy().tolist()), "little")

    def _buf(self, ptr):
        return self.registry[int(ptr)]

    def _flags(self, ptr):
        return self._buf(ptr).view(torch.int32)

    def _poll(self, cond):
        t0 = time.monotonic()
        while not cond():
            if self.err or time.monotonic() - t0 > self.timeout_s:
                self.err = 3  # DSA_ERR_TIMEOUT
                return False
            time.sleep(0.001)
        return True

    def sm70_ipc_flag_set(self, flag_ptr, which, seq):
        if which == 0 and self.stage_delay_s:
            time.sleep(self.stage_delay_s)
        if self.err:
            return
        self._flags(flag_ptr)[which] = seq

    def sm70_ipc_slot_wait(self, flag_ptrs, tp, min_seq):
        self._poll(lambda: all(int(self._flags(p)[1]) >= min_seq for p in flag_ptrs[:tp].tolist()))

    def shard_stage(self, slot_rows, vals, idx):
        if self.err:
            return
        K = vals.shape[1]
        slot_rows[:, :K] = vals
        slot_rows[:, K:] = idx.view(torch.float32)

    def sm70_indexer_shard_merge_p2p(self, out, data_ptrs, flag_ptrs, dst_rows, dst_base, topk, tp, R, seq, slot_off):
        if self.err or not self._poll(lambda: all(int(self._flags(p)[0]) >= seq for p in flag_ptrs[:tp].tolist())):
            return
        self.merges_p2p += 1
        allf = np.stack([self._buf(p)[slot_off:slot_off + R * 2 * topk * 4].view(torch.float32).view(R, 2 * topk)
                         .numpy() for p in data_ptrs[:tp].tolist()])
        self._write(out, O.shard_merge(allf, topk), dst_rows, dst_base, R, topk)

    def sm70_indexer_shard_merge(self, out, allf, dst_rows, dst_base, topk):
        self._write(out, O.shard_merge(allf.numpy(), topk), dst_rows, dst_base, allf.shape[1], topk)

    @staticmethod
    def _write(out, merged, dst_rows, dst_base, R, topk):
        rows = dst_rows.tolist() if dst_base < 0 else list(range(dst_base, dst_base + R))
        for i, r in enumerate(rows):
            out[r, :topk] = torch.from_numpy(merged[i])

    def p2p_failed(self, device):
        failed, self.err = self.err != 0, 0
        return failed


class HostGroup:
    """Ranks as threads: the host AND and the all-gather of merge_shards."""

    def __init__(self, n):
        self.n = n
        self.barrier = threading.Barrier(n, timeout=30)
        self.slots = [None] * n

    def _exchange(self, rank, v):
        self.slots[rank] = v
        self.barrier.wait()
        got = list(self.slots)
        self.barrier.wait()
        return got

    def agree(self, rank, ok):
        return all(self._exchange(rank, bool(ok)))

    def gather(self, rank, t):
        return torch.cat(self._exchange(rank, t.clone()), dim=0)


def _handles(tp):
    return [[FakeIPC.key(r, 0).to_bytes(64, "little"), FakeIPC.key(r, 1).to_bytes(64, "little")] for r in range(tp)]


def _payloads(seed, tp, R, K, rounds):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(rounds):
        vals = rng.standard_normal((tp, R, K)).astype(np.float32)
        pos = (rng.permutation(50000)[:tp * R * K].reshape(tp, R, K)).astype(np.int32)
        out.append((vals, pos))
    return out


def _run_ranks(tp, fn):
    errors = []

    def run(r):
        try:
            fn(r)
        except Exception as e:  # surfaced below
            errors.append(e)

    threads = [threading.Thread(target=run, args=(r,)) for r in range(tp)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(60)
    assert not errors, errors


def test_p2p_exchange_protocol_two_ranks():
    """Two ranks (threads) merge three times: the slots alternate (seq & 1)
    and the third merge waits until every rank merged the first."""
    tp, R, K, rounds = 2, 6, 8, 3
    FakeIPC.registry.clear()
    handles = _handles(tp)

    def gather(objs, payload):
        objs[:] = [tuple(h) for h in handles]

    ex = [sai.P2PExchange("cpu", tp, r, K, rows_cap=16, all_gather_object=gather, backend=FakeIPC(r))
          for r in range(tp)]
    data = _payloads(11, tp, R, K, rounds)
    outs = [[torch.full((R, K), -9, dtype=torch.int32) for _ in range(rounds)] for _ in range(tp)]

    def run(r):
        for i, (vals, pos) in enumerate(data):
            pend = [(0, R, torch.from_numpy(vals[r]), torch.from_numpy(pos[r]))]
            ex[r].merge(pend, outs[r][i])
            assert not ex[r].backend.p2p_failed("cpu")

    _run_ranks(tp, run)
    for i, (vals, pos) in enumerate(data):
        allf = np.concatenate([vals, pos.view(np.float32)], axis=2)
        exp = O.shard_merge(allf, K)
        for r in range(tp):
            np.testing.assert_array_equal(outs[r][i].numpy(), exp)
    assert [e.seq for e in ex] == [rounds, rounds]


def test_p2p_exchange_wait_expires_without_staging():
    """A peer that never stages: the merge wait expires, the error word is
    set, and nothing after it runs (no merged flag, no output write)."""
    tp, R, K = 2, 2, 4
    FakeIPC.registry.clear()
    handles = _handles(tp)
    ex = [sai.P2PExchange("cpu", tp, r, K, rows_cap=4, all_gather_object=lambda o, p: o.__setitem__(
        slice(None), [tuple(h) for h in handles]), backend=FakeIPC(r, timeout_s=0.2)) for r in range(tp)]
    out = torch.full((R, K), -9, dtype=torch.int32)
    ex[0].merge([(0, R, torch.zeros(R, K), torch.zeros(R, K, dtype=torch.int32))], out)
    assert ex[0].backend.p2p_failed("cpu")
    assert int(ex[0].fbuf.view(torch.int32)[1]) == 0  # merged flag never published
    assert (out == -9).all()


def test_p2p_failure_on_one_rank_moves_every_rank_to_the_all_gather_path():
    """Rank 1 publishes its staged flag late, so rank 0's merge wait expires
    while rank 1's merge succeeds. The ranks agree over the host: BOTH redo
    the step through the all-gather path (same collectives on every rank),
    both results are exact, and both stay off P2P for the next step."""
    tp, R, K = 2, 5, 16
    FakeIPC.registry.clear()
    handles = _handles(tp)
    group = HostGroup(tp)
    backends = [FakeIPC(0, timeout_s=0.3), FakeIPC(1, timeout_s=5.0, stage_delay_s=0.8)]
    shards = [sai.ShardConfig(tp=tp, rank=r, merge="p2p", rows_cap=8, backend=backends[r],
                              agree=lambda ok, r=r: group.agree(r, ok), gather=lambda t, r=r: group.gather(r, t))
              for r in range(tp)]
    for r in range(tp):  # exchanges built up front (stand-in IPC handle exchange)
        shards[r].p2p = sai.P2PExchange("cpu", tp, r, K, rows_cap=8, all_gather_object=lambda o, p: o.__setitem__(
            slice(None), [tuple(h) for h in handles]), backend=backends[r])
    data = _payloads(5, tp, R, K, 2)
    outs = [[torch.full((R, K), -9, dtype=torch.int32) for _ in range(2)] for _ in range(tp)]

    def run(r):
        for i, (vals, pos) in enumerate(data):
            pend = [(0, R, torch.from_numpy(vals[r]), torch.from_numpy(pos[r]))]
            sai.merge_shards(pend, outs[r][i], K, shards[r])

    _run_ranks(tp, run)
    assert [s.p2p_failed for s in shards] == [True, True]
    assert backends[0].merges_p2p == 0 and backends[1].merges_p2p == 1  # step 2 never tried P2P
    for i, (vals, pos) in enumerate(data):
        exp = O.shard_merge(np.concatenate([vals, pos.view(np.float32)], axis=2), K)
        for r in range(tp):
            np.testing.assert_array_equal(outs[r][i].numpy(), exp)


# ------------------------------------------------ key-sharded merge, gloo
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sharded_worker(rank, world, port, seed, result_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sai_w = importlib.import_module("glm5-on-v100_b200.sparse_attn_indexer")
        rng = np.random.default_rng(seed)
        R, max_kv, K, page = 7, 3000, 64, 64
        score = rng.standard_normal((R, max_kv)).astype(np.float32)  # distinct with probability 1
        lens = np.array([3000, 2999, 1500, 900, 100, 64, 2048], np.int32)
        off, span = sai_w.shard_span(max_kv, world, rank, page)
        vals, gidx = O.sharded_local_candidates(score, lens, K, off, span, rank)
        buf = torch.full((R, K), -9, dtype=torch.int32)
        shard = sai_w.ShardConfig(tp=world, rank=rank, merge="torch")
        sai_w.merge_shards([(0, R, torch.from_numpy(vals), torch.from_numpy(gidx))], buf, K, shard)
        result_q.put((rank, buf.numpy(), O.topk_rows(score, lens, K)))
    finally:
        dist.destroy_process_group()


def test_key_sharded_merge_two_gloo_ranks():
    """Each rank selects local top-K on its key span, then the all-gather +
    torch epilogue path of merge_shards yields the exact global top-K on every
    rank (the reference's global-subset-of-shard-union property)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, 21, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for rank, got, exp in res:
        np.testing.assert_array_equal(np.sort(got, axis=1), np.sort(exp, axis=1))


# ------------------------------------------- decode exchange slot reuse
def _run_decode_exchange_schedule(tp, steps, rng, merge_waits=True):
    """Random interleaving of tp ranks running the device-sequenced decode
    exchange (csrc/topk.cu exchange staging, csrc/shard_merge.cu exchange
    merge), each rank's kernels in stream order: stage(seq) writes this rank's
    slot seq & 1 and then publishes staged = seq; merge(seq) waits until every
    rank's staged >= seq, then reads every rank's slot seq & 1 (the reads may
    stay in flight across other ranks' events) and completes. Stage(seq + 1)
    of a rank starts only after its merge(seq) completed. Returns the slot
    conflicts seen: a stage writing a slot that some rank is still reading,
    or will still read, for an older step. merge_waits=False drops the
    merge's wait on the staged flags (the check must then find conflicts)."""
    staged = [0] * tp
    seq = [1] * tp                 # next step of each rank
    phase = ["stage"] * tp         # stage -> merge_wait -> merge_read -> done
    reading = {}                   # (reader, owner) -> step whose slot is being read
    reads_left = [set() for _ in range(tp)]
    conflicts = []
    while min(seq) <= steps or any(p != "stage" for p in phase):
        r = int(rng.integers(tp))
        s = seq[r]
        if phase[r] == "stage":
            if s > steps:
                continue
            slot = s & 1
            for (reader, owner), rs in reading.items():
                if owner == r and (rs & 1) == slot and rs < s:
                    conflicts.append((r, s, reader, rs))
            staged[r] = s
            phase[r] = "merge_wait"
        elif phase[r] == "merge_wait":
            if not merge_waits or all(x >= s for x in staged):
                phase[r] = "merge_read"
                reads_left[r] = set(range(tp))
                for q in range(tp):
                    reading[(r, q)] = s
        elif phase[r] == "merge_read":
            q = int(rng.choice(sorted(reads_left[r])))
            reads_left[r].discard(q)
            del reading[(r, q)]
            if not reads_left[r]:
                phase[r] = "stage"
                seq[r] += 1
    return conflicts


@pytest.mark.parametrize("tp", [2, 3, 8])
def test_decode_exchange_slot_reuse_needs_no_wait(tp):
    """The exchange top-k writes its slot seq & 1 without waiting on the
    peers' merged flags: over many random interleavings of the ranks, no
    stage ever overwrites a slot a peer is still reading (the peer's staged
    flag of the previous step, which this rank's merge waited for, is only
    published after that peer finished reading the slot)."""
    rng = np.random.default_rng(tp)
    for _ in range(200):
        assert _run_decode_exchange_schedule(tp, steps=6, rng=rng) == []


def test_decode_exchange_model_detects_a_missing_wait():
    """The same model with the merge's staged-flag wait removed does see
    conflicts, so the check above can fail."""
    rng = np.random.default_rng(5)
    assert any(_run_decode_exchange_schedule(2, steps=6, rng=rng, merge_waits=False) for _ in range(200))
