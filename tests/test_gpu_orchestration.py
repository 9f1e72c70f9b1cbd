"""GPU tests of the callers around the kernels: the indexer orchestration
(sparse_attn_indexer.sparse_indexer: K store, decode and prefill top-k) and
the MLA glue (mla_sparse.forward_mqa_sparse with spec-as-decode rows,
forward_mha_sparse with its projections), against the CPU oracle on the same
inputs.

Tolerances: indexer scores within 1e-4 of the row's max |score| of the fp64
oracle; top-k sets equal to the exact top-K of the kernel's own f32 scores
except at positions within 1 ulp of the K-th score; attention outputs as in
the kernel tests (2e-3 relative per row and head beyond the output dtype's
rounding, lse 2e-3 absolute).
"""
import importlib

import numpy as np
import pytest
import torch

import cases
from oracle import dsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
sai = importlib.import_module("glm5-on-v100_b200.sparse_attn_indexer")
mla = importlib.import_module("glm5-on-v100_b200.mla_sparse")
ops = importlib.import_module("glm5-on-v100_b200.ops")


def assert_topk_1ulp(got, scores, lens, K):
    """got [n, K] positions (ascending, -1 padded) against the exact top-K of
    the kernel's own f32 scores: the index sets may differ only at positions
    whose score lies within 1 ulp of the K-th score (the north-star rule)."""
    exp = O.topk_rows(scores, lens, K)
    for r in range(got.shape[0]):
        n = int(min(lens[r], scores.shape[1]))
        g = got[r]
        assert (g[: min(n, K)] >= 0).all() and (g[min(n, K):] == -1).all(), r
        assert np.all(np.diff(g[g >= 0]) > 0), r  # ascending, distinct
        if n <= K:
            np.testing.assert_array_equal(g[:n], np.arange(n))
            continue
        kth = np.float32(np.sort(scores[r, :n])[::-1][K - 1])
        ulp = np.spacing(np.abs(kth))
        diff = set(g.tolist()) ^ set(exp[r].tolist())
        assert all(abs(np.float32(scores[r, p]) - kth) <= ulp for p in diff), r


def assert_scores_close(s, ref, lens):
    """Kernel scores within 1e-4 of the row's max |score| of the fp64 oracle."""
    for r in range(s.shape[0]):
        n = int(min(lens[r], s.shape[1]))
        if n:
            assert np.abs(s[r, :n] - ref[r, :n]).max() <= 1e-4 * max(np.abs(ref[r, :n]).max(), 1e-6), r


def indexer_inputs(seed, T, Hi, n_blocks, page):
    rng = np.random.default_rng(seed)
    k_rows = cases.f16_exact(rng.standard_normal((n_blocks * page, 128)))
    q = cases.f16_exact(rng.standard_normal((T, Hi, 128)))
    w = cases.f16_exact(rng.standard_normal((T, Hi)) / np.sqrt(Hi))
    return rng, k_rows, q, w


@pytest.mark.parametrize("fused", [True, False])
def test_sparse_indexer_decode(dsa, fused):
    page, Hi, K, nd = 64, 32, 512, 5
    seq = np.array([4000, 3100, 600, 511, 2000], np.int32)
    bps = 64
    rng, k_rows, q, w = indexer_inputs(5, nd, Hi, nd * bps + 2, page)
    bt = rng.permutation(nd * bps + 2)[: nd * bps].reshape(nd, bps).astype(np.int32)
    cache = torch.from_numpy(k_rows.reshape(-1, page, 128)).to(torch.bfloat16).to(DEV)
    # this step's keys: each decode token's own (last) position, already holding its key
    slots = np.array([bt[b, (seq[b] - 1) // page] * page + (seq[b] - 1) % page for b in range(nd)], np.int32)
    k_new = torch.from_numpy(k_rows[slots]).to(torch.bfloat16).to(DEV)
    meta = sai.IndexerMeta(slot_mapping=torch.from_numpy(slots).to(DEV), num_decode_tokens=nd,
                           decode=sai.DecodeMeta(torch.from_numpy(bt).to(DEV), torch.from_numpy(seq).to(DEV)))
    buf = torch.full((nd, K), -7, dtype=torch.int32, device=DEV)
    qd = torch.from_numpy(q).to(torch.bfloat16).to(DEV)
    sai.sparse_indexer(meta, cache, qd, k_new, torch.from_numpy(w).to(DEV), K, buf, fused_decode_topk=fused)
    torch.cuda.synchronize()
    # the kernel's own scores (same launch as inside sparse_indexer), and the
    # fp64 oracle on q and the keys as the device holds them (bf16)
    score = torch.empty(nd, bps * page, device=DEV)
    h = torch.zeros(nd, 4096, dtype=torch.int32, device=DEV) if fused else None
    ops.sm70_indexer_logits(score, qd, cache, torch.from_numpy(w).to(DEV), torch.from_numpy(bt).to(DEV),
                            torch.from_numpy(seq).to(DEV), h)
    s = score.cpu().numpy()
    ref = O.indexer_logits(qd.float().cpu().numpy(), cache.float().cpu().numpy().reshape(-1, 128), w, bt, seq, page,
                           bps * page)
    assert_scores_close(s, ref, seq)
    assert_topk_1ulp(buf.cpu().numpy(), s, seq, K)


def test_sparse_indexer_prefill_two_requests(dsa):
    """One prefill chunk holding two requests (300 and 70 new tokens at the
    end of 2000- and 900-token contexts): per-request sub-blocks, causal
    lengths from cu_seqlen_ke - cu_seqlen_ks, and the chunk bridge entry."""
    page, Hi, K = 64, 32, 256
    ctx = [2000, 900]
    new = [300, 70]
    bps = 32
    T = sum(new)
    rng, k_rows, q, w = indexer_inputs(9, T, Hi, 2 * bps + 1, page)
    bt = rng.permutation(2 * bps + 1)[: 2 * bps].reshape(2, bps).astype(np.int32)
    ke = np.concatenate([np.arange(c - n + 1, c + 1) for c, n in zip(ctx, new)]).astype(np.int32)
    ks = np.zeros(T, np.int32)
    req = np.repeat([0, 1], new)
    pos = ke - 1
    slots = (bt[req, pos // page] * page + pos % page).astype(np.int32)
    cache = torch.from_numpy(k_rows.reshape(-1, page, 128)).to(torch.bfloat16).to(DEV)
    chunk = sai.PrefillChunk(token_start=0, cu_seqlen_ks=torch.from_numpy(ks).to(DEV),
                             cu_seqlen_ke=torch.from_numpy(ke).to(DEV), block_table=torch.from_numpy(bt).to(DEV),
                             num_reqs=2, query_start_loc_cpu=[0, new[0], T])
    meta = sai.IndexerMeta(slot_mapping=torch.from_numpy(slots).to(DEV), prefill_chunks=[chunk])
    buf = torch.full((T, K), -7, dtype=torch.int32, device=DEV)
    qd = torch.from_numpy(q).to(torch.bfloat16).to(DEV)
    sai.sparse_indexer(meta, cache, qd, torch.from_numpy(k_rows[slots]).to(torch.bfloat16).to(DEV),
                       torch.from_numpy(w).to(DEV), K, buf)
    torch.cuda.synchronize()
    ref = O.indexer_logits(qd.float().cpu().numpy(), cache.float().cpu().numpy().reshape(-1, 128), w, bt[req], ke,
                           page, bps * page)
    # the kernel's own scores, one launch per request segment as sparse_indexer makes them
    s = np.full((T, bps * page), -np.inf, np.float32)
    wd = torch.from_numpy(w).to(DEV)
    for r, (lo, hi) in enumerate([(0, new[0]), (new[0], T)]):
        mk = int((ke[lo:hi].max() + 63) // 64 * 64)
        sc = torch.empty(hi - lo, mk, device=DEV)
        seg_bt = torch.from_numpy(bt[r:r + 1, : (mk + page - 1) // page]).to(DEV).expand(hi - lo, -1).contiguous()
        ops.sm70_indexer_logits(sc, qd[lo:hi].contiguous(), cache, wd[lo:hi].contiguous(), seg_bt,
                                torch.from_numpy(ke[lo:hi]).to(DEV))
        s[lo:hi, :mk] = sc.cpu().numpy()
    assert_scores_close(s, ref, ke)
    assert_topk_1ulp(buf.cpu().numpy(), s, ke, K)
    (tok_lo, n_q, ke_out), = sai.PREFILL_META["chunks"]
    assert tok_lo == 0 and n_q == T and ke_out.cpu().tolist() == ke.tolist()


def test_sparse_indexer_custom_op_matches_direct_call(dsa):
    """torch.ops.dsa_b200.sm70_sparse_indexer (the reference's custom op
    schema, metadata looked up by layer name in the forward context) writes
    the same buffer as a direct sparse_indexer call, and returns it."""
    page, Hi, K, nd = 64, 32, 256, 3
    seq = np.array([3000, 700, 256], np.int32)
    bps = 48
    rng, k_rows, q, w = indexer_inputs(15, nd, Hi, nd * bps + 1, page)
    bt = rng.permutation(nd * bps + 1)[: nd * bps].reshape(nd, bps).astype(np.int32)
    slots = np.array([bt[b, (seq[b] - 1) // page] * page + (seq[b] - 1) % page for b in range(nd)], np.int32)
    qd = torch.from_numpy(q).to(torch.bfloat16).to(DEV)
    kn = torch.from_numpy(k_rows[slots]).to(torch.bfloat16).to(DEV)
    wd = torch.from_numpy(w).to(DEV)
    meta = sai.IndexerMeta(slot_mapping=torch.from_numpy(slots).to(DEV), num_decode_tokens=nd,
                           decode=sai.DecodeMeta(torch.from_numpy(bt).to(DEV), torch.from_numpy(seq).to(DEV)))
    outs = []
    for via_op in (False, True):
        cache = torch.from_numpy(k_rows.reshape(-1, page, 128)).to(torch.bfloat16).to(DEV)
        buf = torch.full((nd, K), -7, dtype=torch.int32, device=DEV)
        if via_op:
            with sai.forward_context({"model.layers.3.self_attn.indexer.k_cache": meta}):
                ret = dsa.sm70_sparse_indexer("model.layers.3.self_attn.indexer.k_cache", cache, qd, kn, wd, K, 128,
                                              4096, buf)
            assert ret.data_ptr() == buf.data_ptr()
        else:
            sai.sparse_indexer(meta, cache, qd, kn, wd, K, buf)
        torch.cuda.synchronize()
        outs.append(buf.cpu().numpy())
    np.testing.assert_array_equal(outs[0], outs[1])
    assert (outs[1] != -7).all()


def _attn_ref(q, kv_rows, idx, bt, seq, page, scale):
    return O.sparse_mla_decode(q, kv_rows, idx, bt, seq, page, scale)


def test_forward_mqa_sparse_spec_rows(dsa):
    """Two verify tokens per request read their rows from the top-k buffer
    and use causal lengths seq - 1 and seq (triton_mla.py:261-279)."""
    page, H, K, n_req, next_n = 64, 64, 512, 3, 2
    seq = np.array([1500, 700, 2048], np.int32)
    c = cases.decode_case(17, B=n_req, H=H, page=page, seq_lens=seq, topk=K, blocks_per_seq=32)
    rows = O.dsmla_encode_rows(c["kv"])
    kv_ref = O.dsmla_decode_rows(rows)
    nb = c["kv"].shape[0] // page
    cache = torch.from_numpy(rows.reshape(nb, page, 656)).to(DEV)
    rng = np.random.default_rng(4)
    B = n_req * next_n
    q = cases.f16_exact(rng.standard_normal((B, H, 576)))
    tok_seq = np.repeat(seq, next_n) - np.tile([1, 0], n_req)
    idx = np.stack([np.sort(rng.choice(int(s), size=K, replace=False)) for s in tok_seq]).astype(np.int32)
    buf = torch.full((B + 4, K), -1, dtype=torch.int32, device=DEV)
    buf[:B] = torch.from_numpy(idx).to(DEV)
    scale = 1.0 / np.sqrt(192.0)
    o, lse = mla.forward_mqa_sparse(torch.from_numpy(q).to(torch.bfloat16).to(DEV), cache, buf, K,
                                    torch.from_numpy(c["block_table"]).to(DEV), torch.from_numpy(seq).to(DEV), scale)
    torch.cuda.synchronize()
    bt_tok = np.repeat(c["block_table"], next_n, axis=0)
    qb = torch.from_numpy(q).to(torch.bfloat16).float().numpy()
    o_ref, lse_ref = _attn_ref(qb, kv_ref, idx, bt_tok, tok_seq, page, scale)
    rel = np.linalg.norm(o.float().cpu().numpy() - o_ref, axis=-1) / np.linalg.norm(o_ref, axis=-1)
    rnd = torch.from_numpy(o_ref.astype(np.float32)).to(torch.bfloat16).float().numpy()
    floor = np.linalg.norm(rnd - o_ref, axis=-1) / np.linalg.norm(o_ref, axis=-1)
    assert (rel - floor).max() <= 2e-3
    np.testing.assert_allclose(lse.cpu().numpy(), lse_ref, atol=2e-3, rtol=0)


def test_forward_mha_sparse_projections(dsa):
    """Sparse prefill glue: q_nope . W_UK_T -> latent, sparse attention over
    each token's top-k causal keys, then . W_UV; the per-token lengths and
    block-table rows come from the indexer's chunk entries."""
    page, H, K = 64, 16, 256
    nope, rope, V = 128, 64, 128
    ctx = 1200
    new = 40
    c = cases.decode_case(23, B=1, H=H, page=page, seq_lens=[ctx], topk=K, blocks_per_seq=ctx // page + 1)
    rows = O.dsmla_encode_rows(c["kv"])
    kv_ref = O.dsmla_decode_rows(rows)
    nb = c["kv"].shape[0] // page
    cache = torch.from_numpy(rows.reshape(nb, page, 656)).to(DEV)
    rng = np.random.default_rng(8)
    q = torch.from_numpy(rng.standard_normal((new, H, nope + rope)).astype(np.float32) * 0.5).to(torch.bfloat16)
    W_UK_T = torch.from_numpy(rng.standard_normal((H, nope, 512)).astype(np.float32) / np.sqrt(nope)).to(torch.bfloat16)
    W_UV = torch.from_numpy(rng.standard_normal((H, 512, V)).astype(np.float32) / np.sqrt(512)).to(torch.bfloat16)
    ke = np.arange(ctx - new + 1, ctx + 1).astype(np.int32)
    idx = np.stack([np.sort(rng.choice(int(s), size=min(K, int(s)), replace=False)) for s in ke]).astype(np.int32)
    nd0 = 3  # decode tokens ahead of the prefill rows in the buffer
    buf = torch.full((nd0 + new, K), -1, dtype=torch.int32, device=DEV)
    buf[nd0:] = torch.from_numpy(idx).to(DEV)
    chunks = [(nd0, new, torch.from_numpy(ke).to(DEV))]
    qsl = torch.tensor([0, new], dtype=torch.int32, device=DEV)
    bt = torch.from_numpy(c["block_table"]).to(DEV)
    scale = 1.0 / np.sqrt(192.0)
    out = mla.forward_mha_sparse(q.to(DEV), cache, buf, K, nd0, chunks, qsl, bt, W_UK_T.to(DEV), W_UV.to(DEV), scale,
                                 qk_nope_head_dim=nope, qk_rope_head_dim=rope)
    torch.cuda.synchronize()
    # reference: the same projections in fp32 from the same bf16 operands
    qf, wk, wv = q.float(), W_UK_T.float(), W_UV.float()
    ql = torch.cat([torch.bmm(qf[..., :nope].transpose(0, 1), wk).transpose(0, 1), qf[..., nope:]], dim=-1)
    ql = ql.to(torch.bfloat16).float().numpy()
    o_ref, _ = _attn_ref(ql, kv_ref, idx, np.repeat(c["block_table"], new, axis=0), ke, page, scale)
    o_ref = torch.from_numpy(o_ref.astype(np.float32)).to(torch.bfloat16).float()
    out_ref = torch.bmm(o_ref.transpose(0, 1), wv).transpose(0, 1).reshape(new, H * V).numpy()
    got = out.float().cpu().numpy()
    err = np.linalg.norm(got - out_ref, axis=-1) / np.linalg.norm(out_ref, axis=-1)
    assert err.max() <= 1e-2  # two bf16 roundings (latent q, attention output) feed the bf16 bmm
