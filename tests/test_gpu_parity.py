"""GPU parity: every kernel of the DSA path against the CPU oracle (and the
reference-generated golden fixtures) on identical seeded inputs, called through
the C ABI via the torch-op wrappers.

Tolerances: attention outputs within 2e-3 relative error per (row, head)
(||o - o_ref||_2 / ||o_ref||_2, fp16/bf16 out, fp32 accumulate) beyond the
error that rounding the exact result to the output dtype alone causes (see
assert_attn_close), and lse within 2e-3 absolute; indexer scores within 1e-4
of the row's max |score| (inputs are
exactly representable, accumulation is fp32); integer and byte outputs
(top-k positions, cache rows, histograms, merges) bit-exact.
"""
import os

import numpy as np
import pytest
import torch

import cases
from oracle import dsa_oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"
ATTN_RTOL = 2e-3


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


def kv_tensor(kv_f32, page, fmt):
    """(device cache tensor, dequantised rows the oracle should see)."""
    nb = kv_f32.shape[0] // page
    if fmt == "fp8":
        rows = O.dsmla_encode_rows(kv_f32)
        return to_dev(rows.reshape(nb, page, 656)), O.dsmla_decode_rows(rows)
    if fmt == "f16":
        return to_dev(kv_f32.reshape(nb, page, 576), torch.float16), kv_f32.astype(np.float16).astype(np.float64)
    t = torch.from_numpy(kv_f32.reshape(nb, page, 576)).to(torch.bfloat16)
    return t.to(DEV), t.float().numpy().reshape(-1, 576).astype(np.float64)


def run_decode(dsa, c, fmt="fp8", q_dtype=torch.bfloat16, o_dtype=torch.bfloat16, scale=1.0 / np.sqrt(192.0)):
    kv_t, kv_ref = kv_tensor(c["kv"], c["page"], fmt)
    q = to_dev(c["q"], q_dtype)
    B, H = c["q"].shape[:2]
    o = torch.full((B, H, 512), float("nan"), dtype=o_dtype, device=DEV)
    lse = torch.full((B, H), float("nan"), dtype=torch.float32, device=DEV)
    dsa.sm70_sparse_mla_decode(o, lse, q, kv_t, to_dev(c["idx"]), to_dev(c["block_table"]), to_dev(c["seq_lens"]),
                               scale)
    torch.cuda.synchronize()
    o_ref, lse_ref = O.sparse_mla_decode(q.float().cpu().numpy(), kv_ref, c["idx"], c["block_table"], c["seq_lens"],
                                         c["page"], scale)
    return o.float().cpu().numpy(), lse.cpu().numpy(), o_ref, lse_ref


def random_dsmla_cache(nb, page, seed):
    """A device fp8_ds_mla cache of random valid rows, built on the GPU
    (uniform e4m3 codes except NaN, scales in [0.5, 1.5)/448, N(0,1) rope)."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    kv = torch.randint(0, 256, (nb, page, 656), dtype=torch.uint8, device=DEV, generator=g)
    codes = kv[..., :512]
    codes[(codes & 0x7F) == 0x7F] = 0x7E
    sc = (torch.rand(nb, page, 4, device=DEV, generator=g) + 0.5) / 448.0
    kv[..., 512:528] = sc.contiguous().view(torch.uint8).view(nb, page, 16)
    rope = torch.randn(nb, page, 64, device=DEV, generator=g).to(torch.float16)
    kv[..., 528:656] = rope.view(torch.uint8).view(nb, page, 128)
    return kv


def assert_attn_close(o, lse, o_ref, lse_ref, rtol=ATTN_RTOL, out_dtype=None):
    """Per (row, head): ||o - o_ref|| <= rtol * ||o_ref|| + ||rnd(o_ref) - o_ref||.

    The second term is the error of a perfect kernel whose fp32 result is
    rounded to the output dtype (for bf16 it alone is ~1.7e-3 relative), so
    the bound is 2e-3 relative error beyond the output format's own rounding.
    """
    assert np.isfinite(o).all()
    empty = np.isneginf(lse_ref)
    np.testing.assert_array_equal(np.isneginf(lse), empty)
    assert np.all(o[empty] == 0)
    num = np.linalg.norm(o - o_ref, axis=-1)
    den = np.maximum(np.linalg.norm(o_ref, axis=-1), 1e-30)
    floor = 0.0
    if out_dtype is not None:
        rnd = torch.from_numpy(o_ref.astype(np.float32)).to(out_dtype).float().numpy()
        floor = np.linalg.norm(rnd - o_ref, axis=-1) / den
    excess = np.where(empty, 0.0, num / den - floor)
    assert excess.max() <= rtol, f"max per-row relative error beyond output rounding {excess.max():.3e}"
    np.testing.assert_allclose(lse[~empty], lse_ref[~empty], atol=2e-3, rtol=0)


# ---------------------------------------------------------- sparse decode
@pytest.mark.parametrize("name", ["config1", "ragged"])
def test_decode_matches_reference_golden(dsa, name):
    f = np.load(os.path.join(GOLD, f"mqa_decode_{name}.npz"))
    c = cases.decode_case(int(f["seed"]), int(f["B"]), int(f["H"]), int(f["page"]), f["seq_lens"], int(f["topk"]),
                          int(f["bps"]))
    o, lse, o_ref, lse_ref = run_decode(dsa, c, "f16", torch.float16, torch.float16, float(f["scale"]))
    assert_attn_close(o, lse, o_ref, lse_ref)
    # and directly against the reference's own torch output
    assert_attn_close(o, lse, f["o"].astype(np.float64), f["lse"].astype(np.float64))


@pytest.mark.parametrize("fmt", ["fp8", "f16", "bf16"])
@pytest.mark.parametrize("q_dtype,o_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float16),
                                             (torch.bfloat16, torch.float16)])
def test_decode_formats(dsa, fmt, q_dtype, o_dtype):
    c = cases.decode_case(21, B=4, H=64, page=64, seq_lens=[2048, 5000, 100, 9000], topk=2048, blocks_per_seq=160)
    assert_attn_close(*run_decode(dsa, c, fmt, q_dtype, o_dtype), out_dtype=o_dtype)


@pytest.mark.parametrize("B,H,topk", [(1, 8, 2048), (2, 16, 512), (3, 128, 256), (6, 72, 64), (200, 64, 96),
                                      (64, 64, 2048), (8, 64, 2048), (16, 64, 2048)])
def test_decode_shapes_and_splits(dsa, B, H, topk):
    """Shapes across the slice plans: 32, 16 and 8 slices with partial
    states and the slice merge (B = 1, 8, 16 at top-2048), two slices merged
    in a cluster (B = 64), one slice (B = 200)."""
    rng = np.random.default_rng(B * 1000 + H)
    seq = rng.integers(1, 6000, size=B)
    c = cases.decode_case(31 + B, B=B, H=H, page=64, seq_lens=seq, topk=topk, blocks_per_seq=94)
    assert_attn_close(*run_decode(dsa, c, "fp8"), out_dtype=torch.bfloat16)


@pytest.mark.parametrize("fmt", ["fp8", "f16"])
def test_decode_growing_scores_rescale_path(dsa, fmt):
    """Later tiles hold ever larger scores, so the running max grows by more
    than 2^8 several times and the in-TMEM rescale of O is exercised."""
    # 40 rows keep several 128-row tiles per CTA (few slices), so the running
    # max must move inside a CTA; logits stay at realistic magnitudes (the max
    # grows from ~2 to ~30 in log2 units along the sequence).
    B, S = 40, 4096
    c = cases.decode_case(71, B=B, H=64, page=64, seq_lens=[S] * B, topk=2048, blocks_per_seq=S // 64)
    grow = np.linspace(0.2, 4.0, S).astype(np.float32)[:, None]
    for b in range(B):  # rows of each sequence grow with position
        rows = c["block_table"][b][np.arange(S) // 64].astype(np.int64) * 64 + np.arange(S) % 64
        c["kv"][rows] = cases.f16_exact(c["kv"][rows] * grow)
    assert_attn_close(*run_decode(dsa, c, fmt, torch.bfloat16, torch.bfloat16), out_dtype=torch.bfloat16)


def test_decode_invalid_entries_and_empty_rows(dsa):
    c = cases.decode_case(41, B=6, H=64, page=16, seq_lens=[300, 300, 0, 50, 300, 300], topk=128, blocks_per_seq=20)
    idx = c["idx"]
    idx[0, ::3] = -1                       # unused slots
    idx[1, 5:40] = 299                     # duplicates count separately
    idx[3, :] = np.arange(128) - 40        # negatives and >= seq_len mixed
    idx[4, :] = -1                         # empty row -> o = 0, lse = -inf
    c["block_table"][5, 2] = 10 ** 6       # resolves past the cache: zero row, still counted
    c["block_table"][5, 3] = -7            # negative block id: zero row, still counted
    o, lse, o_ref, lse_ref = run_decode(dsa, c, "fp8")
    assert np.isneginf(lse[2]).all() and np.isneginf(lse[4]).all()
    assert_attn_close(o, lse, o_ref, lse_ref, out_dtype=torch.bfloat16)


def test_decode_topk_zero(dsa):
    B, H = 2, 64
    q = torch.randn(B, H, 576, device=DEV, dtype=torch.bfloat16)
    kv = torch.zeros(4, 64, 656, dtype=torch.uint8, device=DEV)
    o = torch.full((B, H, 512), 7.0, dtype=torch.bfloat16, device=DEV)
    lse = torch.zeros(B, H, device=DEV)
    dsa.sm70_sparse_mla_decode(o, lse, q, kv, torch.zeros(B, 0, dtype=torch.int32, device=DEV),
                               torch.zeros(B, 4, dtype=torch.int32, device=DEV),
                               torch.full((B,), 100, dtype=torch.int32, device=DEV), 0.1)
    torch.cuda.synchronize()
    assert (o == 0).all() and torch.isneginf(lse).all()


def test_decode_mtp_rows_and_sparse_equals_dense(dsa):
    """Spec-as-decode: two query rows per sequence (tmla.py:261-279); with
    seq_len <= topk the sparse op equals dense attention (the reference's
    docs/INTEGRATION.md:124-128)."""
    rng = np.random.default_rng(51)
    n_req, next_n, H, page, topk = 3, 2, 64, 64, 2048
    seq_req = np.array([700, 2048, 1500])
    seq = (seq_req[:, None] - (next_n - 1) + np.arange(next_n)).reshape(-1).astype(np.int32)
    c = cases.decode_case(52, B=n_req * next_n, H=H, page=page, seq_lens=seq, topk=topk, blocks_per_seq=32)
    c["block_table"] = np.repeat(c["block_table"][::next_n], next_n, axis=0)  # rows of a request share blocks
    c["idx"] = np.stack([np.where(np.arange(topk) < s, np.arange(topk), -1) for s in seq]).astype(np.int32)
    o, lse, o_ref, lse_ref = run_decode(dsa, c, "f16", torch.float16, torch.float16)
    assert_attn_close(o, lse, o_ref, lse_ref)


def test_decode_plan_cluster_and_partial_paths(dsa):
    """The fp8 path merges the slices of a row inside a thread-block cluster
    (no workspace, one launch) when the split count is 2 or 4, and falls back
    to partial states + the merge kernel otherwise; the shapes of
    test_decode_shapes_and_splits reach both."""
    from importlib import import_module

    ops = import_module("glm5-on-v100_b200.ops")
    L = import_module("glm5-on-v100_b200._lib")
    big = ops.decode_plan(64, 64, 2048, L.DSA_FP8_DS_MLA)
    assert big["n_splits"] == 2 and big["cluster_size"] == 2
    assert big["workspace_bytes"] == 0 and big["launches"] == 1
    seen = set()
    for B, H, topk in [(1, 8, 2048), (2, 16, 512), (3, 128, 256), (6, 72, 64), (200, 64, 96), (64, 64, 2048)]:
        pl = ops.decode_plan(B, H, topk, L.DSA_FP8_DS_MLA)
        assert (pl["cluster_size"] > 1) == (pl["n_splits"] in (2, 4))
        assert (pl["launches"] == 2) == (pl["n_splits"] > 1 and pl["cluster_size"] == 1)
        assert (pl["workspace_bytes"] > 0) == (pl["launches"] == 2)
        seen.add("cluster" if pl["cluster_size"] > 1 else ("partial" if pl["n_splits"] > 1 else "single"))
    assert seen == {"cluster", "partial", "single"}, seen
    empty = ops.decode_plan(4, 64, 0, L.DSA_FP8_DS_MLA)
    assert empty["n_splits"] == 1 and empty["launches"] == 1


def test_decode_full_size_sampled_rows(dsa):
    """The headline decode shape at 128k context: B=64, H=64, topk=2048, fp8 cache."""
    B, H, S, page, topk = 64, 64, 131072, 64, 2048
    rng = np.random.default_rng(61)
    nb = B * (S // page)
    kv = random_dsmla_cache(nb, page, seed=61)
    bt = rng.permutation(nb).reshape(B, S // page).astype(np.int32)
    idx = np.stack([np.sort(rng.choice(S, topk, replace=False)) for _ in range(B)]).astype(np.int32)
    seq = np.full(B, S, np.int32)
    q = rng.standard_normal((B, H, 576)).astype(np.float32)
    qt = to_dev(q, torch.bfloat16)
    o = torch.empty(B, H, 512, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(B, H, device=DEV)
    scale = 1.0 / np.sqrt(192.0)
    dsa.sm70_sparse_mla_decode(o, lse, qt, kv, to_dev(idx), to_dev(bt), to_dev(seq), scale)
    torch.cuda.synchronize()
    sample = [0, 17, 38, 63]
    flat = kv.view(-1, 656)
    for b in sample:
        rows = bt[b][idx[b] // page].astype(np.int64) * page + idx[b] % page
        kv_rows = O.dsmla_decode_rows(flat[torch.from_numpy(rows).to(DEV)].cpu().numpy())
        local_bt = np.arange(topk // page + 1, dtype=np.int32)[None]
        o_ref, lse_ref = O.sparse_mla_decode(qt[b:b + 1].float().cpu().numpy(),
                                             np.concatenate([kv_rows, np.zeros((page, 576))]),
                                             np.arange(topk, dtype=np.int32)[None], local_bt,
                                             np.array([topk], np.int32), page, scale)
        assert_attn_close(o[b:b + 1].float().cpu().numpy(), lse[b:b + 1].cpu().numpy(), o_ref, lse_ref,
                          out_dtype=torch.bfloat16)


def test_sparse_prefill_full_size_sampled_rows(dsa):
    """Sparse prefill at its full size: 16,384 query tokens x 64 heads at the
    end of a 180,224-token fp8_ds_mla cache, each attending to 2,048 sorted
    uniform-random causal positions, in one call; sampled tokens (first,
    last and spread between) against the oracle."""
    T, H, S, page, topk = 16384, 64, 180224, 64, 2048
    nb = S // page
    kv = random_dsmla_cache(nb, page, seed=83)
    g = torch.Generator(device=DEV).manual_seed(83)
    perm = torch.randperm(nb, device=DEV, generator=g).to(torch.int32)
    bt = perm.view(1, nb).expand(T, nb).contiguous()
    seq = torch.arange(S - T + 1, S + 1, device=DEV, dtype=torch.int32)
    idx = torch.empty(T, topk, dtype=torch.int32, device=DEV)
    pos = torch.arange(S, device=DEV)
    for r0 in range(0, T, 256):
        u = torch.rand(256, S, device=DEV, generator=g)
        u.masked_fill_(pos.view(1, S) >= seq[r0:r0 + 256].view(-1, 1), -1.0)
        idx[r0:r0 + 256] = torch.sort(u.topk(topk, dim=1).indices, dim=1).values.to(torch.int32)
        del u
    q = torch.randn(T, H, 576, device=DEV, generator=g).to(torch.bfloat16)
    o = torch.empty(T, H, 512, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(T, H, device=DEV)
    scale = 1.0 / np.sqrt(192.0)
    dsa.sm70_sparse_mla_decode(o, lse, q, kv, idx, bt, seq, scale)
    torch.cuda.synchronize()
    flat = kv.view(-1, 656)
    btn = perm.cpu().numpy()
    for t in [0, 1, 2047, 5000, 9999, 12288, 16382, 16383]:
        ix = idx[t].cpu().numpy()
        assert ix.max() < S - T + 1 + t and np.all(np.diff(ix) > 0)
        rows = btn[ix // page].astype(np.int64) * page + ix % page
        kv_rows = O.dsmla_decode_rows(flat[torch.from_numpy(rows).to(DEV)].cpu().numpy())
        o_ref, lse_ref = O.sparse_mla_decode(q[t:t + 1].float().cpu().numpy(),
                                             np.concatenate([kv_rows, np.zeros((page, 576))]),
                                             np.arange(topk, dtype=np.int32)[None],
                                             np.arange(topk // page + 1, dtype=np.int32)[None],
                                             np.array([topk], np.int32), page, scale)
        assert_attn_close(o[t:t + 1].float().cpu().numpy(), lse[t:t + 1].cpu().numpy(), o_ref, lse_ref,
                          out_dtype=torch.bfloat16)


def test_sparse_prefill_equals_reference_dense_prefill(dsa):
    """Selecting every causal position, the CUDA sparse path reproduces the
    reference's own dense varlen prefill (_varlen_attention output committed
    in tests/golden/varlen_prefill.npz by tests/golden/make_golden.py)."""
    f = np.load(os.path.join(GOLD, "varlen_prefill.npz"))
    S, T, H = int(f["S"]), int(f["T"]), int(f["H"])
    rng = np.random.default_rng(int(f["seed"]))
    q = cases.f16_exact(rng.standard_normal((T, H, 576)))
    kv = cases.f16_exact(rng.standard_normal((S, 576)))
    assert cases.digest(q, kv) == str(f["digest"])
    idx = np.full((T, S), -1, np.int32)
    for i in range(T):
        n = S - T + i + 1
        idx[i, :n] = np.arange(n)
    page = 16
    bt = np.tile(np.arange(S // page, dtype=np.int32), (T, 1))
    o = torch.empty(T, H, 512, dtype=torch.float16, device=DEV)
    lse = torch.empty(T, H, device=DEV)
    dsa.sm70_sparse_mla_decode(o, lse, to_dev(q, torch.float16), to_dev(kv.reshape(S // page, page, 576),
                                                                       torch.float16),
                               to_dev(idx), to_dev(bt), to_dev(np.full(T, S, np.int32)), float(f["scale"]))
    torch.cuda.synchronize()
    assert_attn_close(o.float().cpu().numpy(), lse.cpu().numpy(), f["o"].astype(np.float64),
                      f["lse"].T.astype(np.float64), out_dtype=torch.float16)


# ---------------------------------------------------------- indexer logits
def idx_cache(k_rows_f32, page, fmt):
    nb = k_rows_f32.shape[0] // page
    if fmt == "fp8":
        rows = O.idxk_encode_rows(k_rows_f32)
        return to_dev(rows.reshape(nb, page, 132)), O.idxk_decode_rows(rows)
    dt = torch.float16 if fmt == "f16" else torch.bfloat16
    t = torch.from_numpy(k_rows_f32.reshape(nb, page, 128)).to(dt)
    return t.to(DEV), t.float().numpy().reshape(-1, 128).astype(np.float64)


def logits_case(seed, B, Hi, S, page, shared_bt=False, causal=False):
    rng = np.random.default_rng(seed)
    bps = (S + page - 1) // page
    nb = (1 if shared_bt else B) * bps + 2
    k = cases.f16_exact(rng.standard_normal((nb * page, 128)))
    q = cases.f16_exact(rng.standard_normal((B, Hi, 128)))
    w = cases.f16_exact(rng.standard_normal((B, Hi)) / np.sqrt(Hi))
    if shared_bt:
        bt = np.tile(rng.permutation(nb)[:bps], (B, 1)).astype(np.int32)
    else:
        bt = rng.permutation(nb)[:B * bps].reshape(B, bps).astype(np.int32)
    if causal:
        seq = (S - B + 1 + np.arange(B)).astype(np.int32)
    else:
        seq = rng.integers(1, S + 1, size=B).astype(np.int32)
    return dict(k=k, q=q, w=w, bt=bt, seq=seq, page=page, max_kv=bps * page)


def run_logits(dsa, c, fmt="f16", q_dtype=torch.float16, w_dtype=torch.float16, hist=False, packed=False):
    kc, k_ref = idx_cache(c["k"], c["page"], fmt)
    B = c["q"].shape[0]
    q = to_dev(c["q"], q_dtype)
    w = to_dev(c["w"], w_dtype)
    score = torch.full((B, c["max_kv"]), float("nan"), device=DEV)
    h = torch.zeros(B, 4096, dtype=torch.int32, device=DEV) if hist else None
    if packed:
        n16 = (B + 15) // 16 * 16
        qp = torch.nn.functional.pad(q, (0, 0, 0, 0, 0, n16 - B))
        qp = qp.view(n16 // 16, 16, 32, 8, 16).permute(2, 0, 3, 1, 4).contiguous()
        dsa.sm70_indexer_logits_packed(score, qp, kc, w, to_dev(c["bt"]), to_dev(c["seq"]))
    else:
        dsa.sm70_indexer_logits(score, q, kc, w, to_dev(c["bt"]), to_dev(c["seq"]), h)
    torch.cuda.synchronize()
    ref = O.indexer_logits(q.float().cpu().numpy(), k_ref, w.float().cpu().numpy(), c["bt"], c["seq"], c["page"],
                           c["max_kv"])
    return score.cpu().numpy(), ref, (h.cpu().numpy() if hist else None)


def assert_scores_close(s, ref):
    inf = np.isneginf(ref)
    np.testing.assert_array_equal(np.isneginf(s), inf)
    for b in range(s.shape[0]):
        fin = ~inf[b]
        if fin.any():
            scale = max(np.abs(ref[b, fin]).max(), 1e-6)
            assert np.abs(s[b, fin] - ref[b, fin]).max() <= 1e-4 * scale, b


@pytest.mark.parametrize("fmt", ["f16", "bf16", "fp8"])
@pytest.mark.parametrize("Hi", [8, 32, 64])
def test_indexer_rows_kernel(dsa, fmt, Hi):
    c = logits_case(100 + Hi, B=3, Hi=Hi, S=5000, page=64)
    qd = torch.bfloat16 if fmt == "bf16" else torch.float16
    s, ref, h = run_logits(dsa, c, fmt, qd, torch.float32, hist=True)
    assert_scores_close(s, ref)
    np.testing.assert_array_equal(h, O.level1_hist(s, c["seq"]))


def _logits_cabi(dsa, score, q, kc_ptr, n_kv_rows, page, w, bt, seq, B, Hi, hist):
    L = dsa._lib
    L.call("dsa_indexer_logits", score.data_ptr(), score.stride(0), score.size(1), q.data_ptr(), L.DSA_F16,
           kc_ptr, L.DSA_FP8_IDXK, n_kv_rows, page, w.data_ptr(), L.DSA_F32, bt.data_ptr(), bt.stride(0),
           bt.size(1), seq.data_ptr(), B, Hi, hist.data_ptr(), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("Hi", [8, 32, 64])
def test_indexer_paged_rows_kernel_edges(dsa, Hi):
    """The tcgen05 decode kernel for fp8 caches with 64-token pages (bulk page
    copies, 4096 positions per CTA): missing blocks, a last page partly past
    the cache, a row of length 0, a row longer than max_kv, a row ending on a
    CTA boundary and an unaligned score stride. Scores match the mma.sync
    rows kernel on the same bytes viewed as 32-token pages and the oracle
    (within the logits tolerance: the two kernels sum in different orders),
    the histogram is exact on the kernel's own scores, and nothing is written
    past max_kv."""
    B, S = 6, 4500
    c = logits_case(700 + Hi, B=B, Hi=Hi, S=S, page=64)
    nb = c["k"].shape[0] // 64
    n_kv_rows = nb * 64 - 10  # the last page is only partly inside the cache
    bt = c["bt"].copy()
    bt[2, 5], bt[2, 9] = -1, nb + 7
    bt[4, 3] = nb - 1
    seq = c["seq"].copy()
    seq[0], seq[1], seq[3], seq[5] = 4500, 0, c["max_kv"] + 50, 4096  # 4096 = one CTA's positions
    rows = O.idxk_encode_rows(c["k"])
    kc = to_dev(rows.reshape(nb, 64, 132))
    q = to_dev(c["q"], torch.float16)
    w = to_dev(c["w"], torch.float32)
    pad = 3
    out = {}
    for page in (64, 32):
        btp = bt if page == 64 else np.stack([2 * bt, 2 * bt + 1], axis=2).reshape(B, -1)
        btp = np.where((bt if page == 64 else np.repeat(bt, 2, axis=1)) < 0, -1, btp).astype(np.int32)
        buf = torch.full((B, c["max_kv"] + pad), float("nan"), device=DEV)
        hist = torch.zeros(B, 4096, dtype=torch.int32, device=DEV)
        _logits_cabi(dsa, buf[:, : c["max_kv"]], q, kc.data_ptr(), n_kv_rows, page, w, to_dev(btp), to_dev(seq),
                     B, Hi, hist)
        torch.cuda.synchronize()
        assert torch.isnan(buf[:, c["max_kv"]:]).all()
        out[page] = (buf[:, : c["max_kv"]].cpu().numpy(), hist.cpu().numpy())
    s64, h64 = out[64]
    s32, h32 = out[32]
    assert_scores_close(s64, s32.astype(np.float64))
    np.testing.assert_array_equal(h32, O.level1_hist(s32, seq))
    k_ref = O.idxk_decode_rows(rows)[:n_kv_rows]
    ref = O.indexer_logits(c["q"], k_ref, c["w"], bt, seq, 64, c["max_kv"])
    assert_scores_close(s64, ref)
    np.testing.assert_array_equal(h64, O.level1_hist(s64, seq))


@pytest.mark.parametrize("fmt", ["f16", "bf16", "fp8"])
def test_indexer_tiles_kernel_causal(dsa, fmt):
    c = logits_case(200, B=150, Hi=32, S=3000, page=64, shared_bt=True, causal=True)
    qd = torch.bfloat16 if fmt == "bf16" else torch.float16
    s, ref, _ = run_logits(dsa, c, fmt, qd, torch.float16)
    assert_scores_close(s, ref)


@pytest.mark.parametrize("fmt,Hi,page,B,S,pad,holes", [
    ("bf16", 32, 64, 300, 5000, 0, False),
    ("f16", 64, 8, 130, 777, 3, True),
    ("bf16", 1, 512, 129, 1300, 1, True),
    ("f16", 17, 16, 67, 2100, 0, False),
])
def test_indexer_tc_kernel_edges(dsa, fmt, Hi, page, B, S, pad, holes):
    """The tcgen05 prefill kernel (16-bit cache of q's type, rows sharing one
    block table): partial query and key tiles, pages shorter and longer than
    its 256-key tile, missing blocks (negative and past the cache), an
    unaligned score row stride, a row of length 0 and a row longer than
    max_kv. Nothing is written past max_kv."""
    c = logits_case(500 + B, B=B, Hi=Hi, S=S, page=page, shared_bt=True)
    if holes:
        nb = c["k"].shape[0] // page
        bt = c["bt"].copy()
        bt[:, 1] = -1
        bt[:, 3 % bt.shape[1]] = nb + 5
        c["bt"] = bt
    c["seq"][0] = 0
    c["seq"][1] = c["max_kv"] + 100
    kc, k_ref = idx_cache(c["k"], page, fmt)
    q = to_dev(c["q"], torch.bfloat16 if fmt == "bf16" else torch.float16)
    w = to_dev(c["w"], torch.float32)
    buf = torch.full((B, c["max_kv"] + pad), float("nan"), device=DEV)
    score = buf[:, : c["max_kv"]]
    dsa.sm70_indexer_logits(score, q, kc, w, to_dev(c["bt"]), to_dev(c["seq"]), None)
    torch.cuda.synchronize()
    ref = O.indexer_logits(q.float().cpu().numpy(), k_ref, c["w"], c["bt"], c["seq"], page, c["max_kv"])
    assert_scores_close(score.cpu().numpy(), ref)
    if pad:
        assert torch.isnan(buf[:, c["max_kv"]:]).all()


@pytest.mark.parametrize("B", [70, 300])
def test_indexer_packed_equals_unpacked(dsa, B):
    # the fp8 cache runs the same mma.sync kernel for both q layouts: bit-identical
    c = logits_case(300 + B, B=B, Hi=32, S=1500, page=64, shared_bt=True, causal=True)
    s1, ref, _ = run_logits(dsa, c, "fp8")
    s2, _, _ = run_logits(dsa, c, "fp8", packed=True)
    np.testing.assert_array_equal(s1, s2)
    assert_scores_close(s2, ref)
    # with a 16-bit cache both layouts run the tcgen05 kernel (packed q through
    # 32-byte-swizzled boxes of a 5-D tensor map, one per MMA K-step): the
    # same products in the same order, bit-identical
    for fmt, qd in (("f16", torch.float16), ("bf16", torch.bfloat16)):
        s3, ref3, _ = run_logits(dsa, c, fmt, qd)
        s4, _, _ = run_logits(dsa, c, fmt, qd, packed=True)
        assert_scores_close(s3, ref3)
        np.testing.assert_array_equal(s3, s4)


def test_indexer_prefill_full_size_sampled_rows(dsa):
    """The indexer prefill shapes (65,536 keys, 32 heads, bf16): the last
    4,096-row sub-block of the causal chunk through logits + top-2048; sampled
    rows against the oracle, and every row's selection exact on the kernel's
    own scores for 64 rows spread over the sub-block."""
    N, Hi, page, K, R = 65536, 32, 64, 2048, 4096
    g = torch.Generator(device=DEV).manual_seed(77)
    nb = N // page
    kc = torch.randn(nb, page, 128, device=DEV, generator=g).to(torch.bfloat16)
    bt_row = torch.randperm(nb, device=DEV, generator=g).to(torch.int32)
    bt = bt_row.view(1, nb).expand(R, nb).contiguous()
    q = torch.randn(R, Hi, 128, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(R, Hi, device=DEV, generator=g) / Hi ** 0.5).to(torch.float16)
    lens = torch.arange(N - R + 1, N + 1, dtype=torch.int32, device=DEV)
    score = torch.empty(R, N, device=DEV)
    idx = torch.empty(R, K, dtype=torch.int32, device=DEV)
    dsa.sm70_indexer_logits(score, q, kc, w, bt, lens, None)
    dsa.persistent_topk(score, lens, idx, torch.empty(0, device=DEV), K, N)
    torch.cuda.synchronize()
    k_ref = kc.float().cpu().numpy().reshape(-1, 128).astype(np.float64)
    rows = [0, 1, 2047, R - 1]
    s_rows = score[rows].cpu().numpy()
    ref = O.indexer_logits(q[rows].float().cpu().numpy(), k_ref, w[rows].float().cpu().numpy(),
                           bt[rows].cpu().numpy(), lens[rows].cpu().numpy(), page, N)
    assert_scores_close(s_rows, ref)
    sample = torch.arange(0, R, R // 64, device=DEV)
    np.testing.assert_array_equal(idx[sample].cpu().numpy(),
                                  O.topk_rows(score[sample].cpu().numpy(), lens[sample].cpu().numpy(), K))


@pytest.mark.parametrize("mult", [2.0 ** 20, 2.0 ** 100, 2.0 ** -30])
def test_decode_bf16_q_outside_fp16_range(dsa, mult):
    """bf16 q far outside fp16's normal range (2^20, 2^100 above it; 2^-30,
    deep in its subnormals): the tcgen05 kernel shifts each CTA's Q by a power
    of two for the fp16 MMA and undoes it in the softmax scale, so o and lse
    match the oracle as for N(0,1) q (scale divided by mult keeps the scores
    O(1))."""
    c = cases.decode_case(91, B=4, H=64, page=64, seq_lens=[2048, 3000, 700, 4000], topk=512, blocks_per_seq=64)
    c["q"] = (c["q"].astype(np.float64) * mult).astype(np.float32)
    assert_attn_close(*run_decode(dsa, c, "fp8", torch.bfloat16, torch.bfloat16, 1.0 / np.sqrt(192.0) / mult),
                      out_dtype=torch.bfloat16)


@pytest.mark.parametrize("mult", [2.0 ** 20, 2.0 ** -30])
def test_indexer_decode_bf16_q_outside_fp16_range(dsa, mult):
    """The tcgen05 decode indexer (fp8 cache) with bf16 q scaled far outside
    fp16's normal range: scores within 1e-4 of the oracle's, histogram exact."""
    c = logits_case(515, B=3, Hi=32, S=5000, page=64)
    c["q"] = (c["q"].astype(np.float64) * mult).astype(np.float32)
    s, ref, h = run_logits(dsa, c, "fp8", torch.bfloat16, torch.float32, hist=True)
    assert_scores_close(s, ref)
    np.testing.assert_array_equal(h, O.level1_hist(s, c["seq"]))


def test_indexer_q_bf16_with_fp16_cache(dsa):
    c = logits_case(310, B=5, Hi=32, S=700, page=16)
    s, ref, _ = run_logits(dsa, c, "f16", torch.bfloat16, torch.bfloat16)
    assert_scores_close(s, ref)


# ------------------------------------------------------------------- top-k
@pytest.mark.parametrize("K", [1, 7, 512, 2048, 4096])
def test_topk_rows_exact_with_ties(dsa, K):
    rng = np.random.default_rng(K)
    B, S = 9, 9000
    score = (np.round(rng.standard_normal((B, S)) * 8) / 8).astype(np.float32)  # heavy ties
    score[2, :] = 1.5                                                              # all tied
    score[3, 100:] = -np.inf
    lens = np.array([S, S - 1, S, S, K, K - 1 if K > 1 else 0, 0, 2 * K + 1, S // 3], np.int32)
    out = torch.full((B, K), -7, dtype=torch.int32, device=DEV)
    dsa.persistent_topk(to_dev(score), to_dev(lens.reshape(-1, 1)), out, torch.empty(0, device=DEV), K, S)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.topk_rows(score, lens, K))


def test_topk_adversarial_rows_and_boundaries(dsa):
    """persistent_topk on rows that defeat shortcuts: large scores only at
    512 evenly spaced runs of 8 positions (what a strided sample would see),
    rows of 8192 and 8193 keys (power-of-two edges), and heavy ties from
    quarter-step rounding; every row exact against the oracle."""
    rng = np.random.default_rng(5)
    K, S = 2048, 60000
    score = rng.standard_normal((4, S)).astype(np.float32)
    n = S
    starts = (np.arange(512, dtype=np.int64) * (n - 8) // 511) & ~3
    sampled = (starts[:, None] + np.arange(8)).reshape(-1)
    score[0, sampled] = 1000.0 + rng.random(sampled.size).astype(np.float32)
    score[2, :] = np.round(score[2, :] * 4) / 4
    lens = np.array([S, 8192, 8193, S], np.int32)
    out = torch.full((4, K), -7, dtype=torch.int32, device=DEV)
    dsa.persistent_topk(to_dev(score), to_dev(lens.reshape(-1, 1)), out, torch.empty(0, device=DEV), K, S)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.topk_rows(score, lens, K))


def test_decode_topk_with_fused_histogram_end_to_end(dsa):
    """indexer logits (+hist) -> decode top-k: the kernel's scores within
    1e-4 of the fp64 oracle, and the selected set exact on those f32 scores
    (so no member differs, not even among ties within 1 ulp of the K-th)."""
    c = logits_case(400, B=4, Hi=32, S=20000, page=64)
    c["seq"] = np.array([20000, 15000, 2048, 1000], np.int32)
    kc, k_ref = idx_cache(c["k"], c["page"], "f16")
    B, K = 4, 2048
    score = torch.empty(B, c["max_kv"], device=DEV)
    hist = torch.zeros(B, 4096, dtype=torch.int32, device=DEV)
    q, w = to_dev(c["q"], torch.float16), to_dev(c["w"], torch.float16)
    dsa.sm70_indexer_logits(score, q, kc, w, to_dev(c["bt"]), to_dev(c["seq"]), hist)
    idx = torch.empty(B, K, dtype=torch.int32, device=DEV)
    dsa.sm70_decode_topk(idx, score, to_dev(c["seq"]), hist, K)
    torch.cuda.synchronize()
    s = score.cpu().numpy()
    got = idx.cpu().numpy()
    np.testing.assert_array_equal(got, O.topk_rows(s, c["seq"], K))
    ref = O.indexer_logits(c["q"], k_ref, c["w"], c["bt"], c["seq"], c["page"], c["max_kv"])
    assert_scores_close(s, ref)


def test_topk_long_decode_row(dsa):
    rng = np.random.default_rng(77)
    S, K = 180224, 2048
    score = rng.standard_normal((2, S)).astype(np.float32)
    lens = np.array([S, 100000], np.int32)
    out = torch.empty(2, K, dtype=torch.int32, device=DEV)
    dsa.persistent_topk(to_dev(score), to_dev(lens), out, torch.empty(0, device=DEV), K, S)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.topk_rows(score, lens, K))


def cluster_topk_rows(rng, S):
    """Rows for the cluster top-k (few rows of >= 8192 keys with a histogram):
    a long row, a short one (< K), one just above K, one with a long run of
    values equal to the K-th, and one whose threshold bin holds more keys
    than the candidate buffer (the one-CTA fallback inside the cluster)."""
    B = 6
    s = rng.standard_normal((B, S)).astype(np.float32)
    s[3] = np.round(s[3] * 2) / 2             # few distinct values: huge ties at the K-th
    n_eq = min(30000, S - 100)                # more equal keys than the candidate buffer holds
    s[4, :n_eq] = 1.0
    s[4, n_eq:] = rng.standard_normal(S - n_eq).astype(np.float32) - 5.0
    s[5] = np.arange(S, dtype=np.float32)[::-1] * 1e-3  # strictly decreasing
    lens = np.array([S, 1500, 2049, S, S, S - 7], np.int32)
    for b in range(B):
        s[b, lens[b]:] = -np.inf
    return s, lens


@pytest.mark.parametrize("S", [9000, 9001, 70000, 180224, 240000])
def test_decode_topk_cluster_mode_exact(dsa, S):
    """Few long rows with the fused histogram run as a cluster of CTAs per row;
    exact (lowest-position ties, ascending, -1 padded) and the histogram is
    left as given (sm70_decode_topk does not clear it). S = 9001 leaves most
    rows off 16-byte alignment and 240000 gives each CTA more scores than it
    stages in shared memory: both read the scores from global memory."""
    rng = np.random.default_rng(S)
    s, lens = cluster_topk_rows(rng, S)
    K = 2048
    hist = to_dev(O.level1_hist(s, lens))
    out = torch.full((s.shape[0], K), -9, dtype=torch.int32, device=DEV)
    dsa.sm70_decode_topk(out, to_dev(s), to_dev(lens), hist, K)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.topk_rows(s, lens, K))
    np.testing.assert_array_equal(hist.cpu().numpy(), O.level1_hist(s, lens))


def test_topk_payload_cluster_mode_clears_hist(dsa):
    """Payload mode in cluster mode: values, shifted positions, pads, and the
    consumed histogram zeroed for the next step."""
    from importlib import import_module

    ops = import_module("glm5-on-v100_b200.ops")
    rng = np.random.default_rng(33)
    S, K, off = 40000, 2048, 90000
    s, lens = cluster_topk_rows(rng, S)
    hist = to_dev(O.level1_hist(s, lens))
    pay = torch.full((s.shape[0], 2 * K), 7.0, device=DEV)
    ops.topk_rows_payload(pay, to_dev(s), to_dev(lens), hist, K, off)
    torch.cuda.synchronize()
    exp = O.topk_rows(s, lens, K)
    p = pay.cpu().numpy()
    np.testing.assert_array_equal(p[:, K:].copy().view(np.int32), np.where(exp >= 0, exp + off, -1))
    np.testing.assert_array_equal(p[:, :K], np.where(exp >= 0, np.take_along_axis(s, np.maximum(exp, 0), axis=1),
                                                     -np.inf).astype(np.float32))
    assert int(hist.abs().sum()) == 0


# -------------------------------------------------------------- K scatter
@pytest.mark.parametrize("k_dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("fmt", ["fp8", "f16", "bf16"])
def test_indexer_k_store_bit_exact(dsa, k_dtype, fmt):
    rng = np.random.default_rng(5)
    n_tok, n_rows = 300, 1000
    k32 = (rng.standard_normal((n_tok, 128)) * np.exp2(rng.integers(-6, 6, (n_tok, 1)))).astype(np.float32)
    k32[3] = 0.0                      # all-zero row -> scale FLT_MIN
    k32[4, 7] = 1e4                   # large outlier
    kt = torch.from_numpy(k32).to(k_dtype)
    kin = kt.float().numpy()
    slot = rng.permutation(n_rows)[:n_tok].astype(np.int32)
    slot[::17] = -1
    slot[5] = n_rows + 3              # out of range: skipped
    if fmt == "fp8":
        cache = torch.zeros(n_rows // 10, 10, 132, dtype=torch.uint8, device=DEV)
        base = np.zeros((n_rows, 132), np.uint8)
    elif fmt == "f16":
        cache = torch.zeros(n_rows // 10, 10, 128, dtype=torch.float16, device=DEV)
        base = np.zeros((n_rows, 128), np.float16)
    else:
        cache = torch.zeros(n_rows // 10, 10, 128, dtype=torch.bfloat16, device=DEV)
        base = np.zeros((n_rows, 128), np.uint16)  # bf16 bit patterns
    dsa.sm70_indexer_k_store(cache, kt.to(DEV), to_dev(slot))
    torch.cuda.synchronize()
    exp = O.indexer_k_store(base, kin, slot, fmt)
    got = cache.cpu().view(torch.uint8).numpy().reshape(n_rows, -1)
    np.testing.assert_array_equal(got, exp.view(np.uint8).reshape(n_rows, -1))


# ------------------------------------------------------------ shard merge
def merge_payload(rng, tp, R, K, n_pos=10 ** 6):
    vals = (np.round(rng.standard_normal((tp, R, K)) * 4) / 4).astype(np.float32)
    vals[0, 0, :K // 3] = -np.inf
    if R > 1:
        vals[:, 1, :] = -np.inf
    pos = np.stack([rng.permutation(n_pos)[:tp * K].reshape(tp, K) for _ in range(R)], axis=1).astype(np.int32)
    pos[vals == -np.inf] = -1
    return np.concatenate([vals, pos.view(np.float32)], axis=2)


@pytest.mark.parametrize("R", [5, 37])  # a cluster of tp CTAs per row / one CTA per row
@pytest.mark.parametrize("tp,K", [(1, 64), (2, 2048), (3, 100), (4, 2048), (8, 2048), (8, 1)])
def test_shard_merge_exact(dsa, tp, K, R):
    rng = np.random.default_rng(tp * 31 + K + R)
    allf = merge_payload(rng, tp, R, K)
    out = torch.full((R + 3, K), -9, dtype=torch.int32, device=DEV)
    dsa.sm70_indexer_shard_merge(out, to_dev(allf), torch.empty(0, dtype=torch.int32, device=DEV), 2, K)
    dst = rng.permutation(R + 3)[:R].astype(np.int32)
    out2 = torch.full((R + 3, K), -9, dtype=torch.int32, device=DEV)
    dsa.sm70_indexer_shard_merge(out2, to_dev(allf), to_dev(dst), -1, K)
    torch.cuda.synchronize()
    exp = O.shard_merge(allf, K)
    np.testing.assert_array_equal(out.cpu().numpy()[2:2 + R], exp)
    np.testing.assert_array_equal(out2.cpu().numpy()[dst], exp)


def test_shard_merge_reference_fixture(dsa):
    f = np.load(os.path.join(GOLD, "shard_merge.npz"))
    allf, K = f["allf"], int(f["K"])
    R = allf.shape[1]
    out = torch.empty(R, K, dtype=torch.int32, device=DEV)
    dsa.sm70_indexer_shard_merge(out, to_dev(allf), torch.empty(0, dtype=torch.int32, device=DEV), 0, K)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.shard_merge(allf, K))


def test_bounded_mbarrier_wait_expiry_is_reported(dsa, monkeypatch):
    """An mbarrier wait that can never complete (one of two arrivals) runs out
    after 10 ms of device time: the status word reads TIMEOUT, the torch layer
    raises DsaDeviceError (and clears it), the debug mode raises at the next
    op call, and the context stays usable for real work."""
    from importlib import import_module

    L = import_module("glm5-on-v100_b200._lib")
    ops = dsa.ops
    ops.device_error(reset=True)
    ops.selftest_wait_timeout(0.01)
    torch.cuda.synchronize()
    assert ops.device_error() == L.DSA_ERR_TIMEOUT
    with pytest.raises(ops.DsaDeviceError):
        ops.check_device_status()
    assert ops.device_error() == 0
    # debug mode: the next op call synchronises and raises
    ops.selftest_wait_timeout(0.01)
    monkeypatch.setattr(L, "CHECK_DEVICE", True)
    rng = np.random.default_rng(4)
    s = rng.standard_normal((3, 5000)).astype(np.float32)
    lens = np.array([5000, 4000, 100], np.int32)
    out = torch.empty(3, 256, dtype=torch.int32, device=DEV)
    with pytest.raises(ops.DsaDeviceError):
        dsa.persistent_topk(to_dev(s), to_dev(lens), out, torch.empty(0, device=DEV), 256, 5000)
    # the same call again: clean status, exact result
    dsa.persistent_topk(to_dev(s), to_dev(lens), out, torch.empty(0, device=DEV), 256, 5000)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.topk_rows(s, lens, 256))
    assert ops.device_error() == 0


def test_shard_merge_p2p_local_slots_and_timeout(dsa):
    """The P2P merge over pointer arrays (two slabs on this GPU stand in for
    peers), then a bounded wait on a flag nothing sets: the kernel returns,
    reports TIMEOUT, and the context stays usable."""
    rng = np.random.default_rng(9)
    tp, R, K = 2, 4, 2048
    allf = merge_payload(rng, tp, R, K)
    slabs = [to_dev(allf[s]) for s in range(tp)]
    flags = [torch.zeros(2, dtype=torch.int32, device=DEV) for _ in range(tp)]
    for f in flags:
        f[0] = 5
    data_ptrs = torch.tensor([s.data_ptr() for s in slabs], dtype=torch.int64)
    flag_ptrs = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64)
    out = torch.empty(R, K, dtype=torch.int32, device=DEV)
    dsa.sm70_indexer_shard_merge_p2p(out, data_ptrs, flag_ptrs, torch.empty(0, dtype=torch.int32, device=DEV), 0, K,
                                     tp, R, 5, 0)
    torch.cuda.synchronize()
    dsa.ops.check_p2p_status(DEV)
    np.testing.assert_array_equal(out.cpu().numpy(), O.shard_merge(allf, K))
    # flag_set publishes, slot_wait sees it
    dsa.sm70_ipc_flag_set(flags[0].data_ptr(), 1, 11)
    dsa.sm70_ipc_flag_set(flags[1].data_ptr(), 1, 11)
    dsa.sm70_ipc_slot_wait(flag_ptrs, tp, 11)
    torch.cuda.synchronize()
    dsa.ops.check_p2p_status(DEV)
    # a wait that runs out: staged flag stays at 5 < 6
    old = dsa.ops.P2P_TIMEOUT_NS
    dsa.ops.P2P_TIMEOUT_NS = 50_000_000  # 50 ms
    try:
        dsa.sm70_indexer_shard_merge_p2p(out, data_ptrs, flag_ptrs, torch.empty(0, dtype=torch.int32, device=DEV),
                                         0, K, tp, 1, 6, 0)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="TIMEOUT"):
            dsa.ops.check_p2p_status(DEV)
    finally:
        dsa.ops.P2P_TIMEOUT_NS = old
    x = torch.ones(4, device=DEV) * 2
    assert float(x.sum()) == 8.0


def sharded_payload(rng, tp, R, K, span, overlap=False, ties=False):
    """Candidates shaped like the key-sharded pipeline's: shard s holds its
    local top-K as ascending positions of its own key span (shifted by s *
    span, or all in one span when overlap is set), -1 / -inf pads at the end
    of short rows."""
    vals = rng.standard_normal((tp, R, K)).astype(np.float32)
    if ties:
        vals = np.round(vals).astype(np.float32)  # few distinct values: long runs of equal keys
    pos = np.empty((tp, R, K), np.int32)
    for s in range(tp):
        for r in range(R):
            pos[s, r] = np.sort(rng.choice(span, K, replace=False)) + (0 if overlap else s * span)
    n_short = min(K, 3)
    vals[tp - 1, 0, K - n_short:] = -np.inf  # a shard with fewer than K keys in row 0
    pos[tp - 1, 0, K - n_short:] = -1
    if R > 2:
        vals[:, 2, :] = -np.inf  # a row no shard reaches
        pos[:, 2, :] = -1
    return np.concatenate([vals, pos.view(np.float32)], axis=2)


@pytest.mark.parametrize("tp,K,overlap,ties", [(2, 2048, False, False), (8, 2048, False, False),
                                               (4, 2048, True, False), (8, 2048, False, True),
                                               (3, 512, True, True), (5, 6, False, False)])
@pytest.mark.parametrize("R", [6, 33])  # a cluster of tp CTAs per row / one CTA per row
def test_shard_merge_sorted_runs(dsa, tp, K, overlap, ties, R):
    """The merge's ordered path (every shard's run ascending): disjoint key
    spans, overlapping spans (binary-searched ranks) and long runs of equal
    values (column-order tie ranks); bit-exact against the oracle."""
    rng = np.random.default_rng(tp * 7 + K + 3 * overlap + ties + R)
    allf = sharded_payload(rng, tp, R, K, span=max(4 * K, 64), overlap=overlap, ties=ties)
    out = torch.full((R, K), -9, dtype=torch.int32, device=DEV)
    dsa.sm70_indexer_shard_merge(out, to_dev(allf), torch.empty(0, dtype=torch.int32, device=DEV), 0, K)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.shard_merge(allf, K))


def test_shard_merge_all_equal_values(dsa):
    """Every candidate has the same value: the lower columns win (the first K
    columns of shard 0), whatever their positions."""
    tp, R, K = 4, 3, 2048
    rng = np.random.default_rng(5)
    vals = np.full((tp, R, K), 1.5, np.float32)
    pos = rng.permutation(tp * R * K).reshape(tp, R, K).astype(np.int32)
    allf = np.concatenate([vals, pos.view(np.float32)], axis=2)
    out = torch.empty(R, K, dtype=torch.int32, device=DEV)
    dsa.sm70_indexer_shard_merge(out, to_dev(allf), torch.empty(0, dtype=torch.int32, device=DEV), 0, K)
    torch.cuda.synchronize()
    exp = O.shard_merge(allf, K)
    np.testing.assert_array_equal(exp, np.sort(pos[0], axis=1))
    np.testing.assert_array_equal(out.cpu().numpy(), exp)


def test_topk_rows_payload_matches_topk(dsa):
    """The payload top-k (local top-K + value gather + global-id shift in one
    launch) against the index top-k on the same scores; its hist is zeroed."""
    from importlib import import_module

    ops = import_module("glm5-on-v100_b200.ops")
    rng = np.random.default_rng(12)
    B, S, K, off = 5, 9000, 2048, 40960
    s = rng.standard_normal((B, S)).astype(np.float32)
    lens = np.array([9000, 5000, 2048, 100, 0], np.int32)
    for b in range(B):
        s[b, lens[b]:] = -np.inf
    score, dl = to_dev(s), to_dev(lens)
    hist = to_dev(O.level1_hist(s, lens))
    pay = torch.full((B, 2 * K), 7.0, device=DEV)
    ops.topk_rows_payload(pay, score, dl, hist, K, off)
    torch.cuda.synchronize()
    exp = O.topk_rows(s, lens, K)
    p = pay.cpu().numpy()
    got_pos = p[:, K:].copy().view(np.int32)
    np.testing.assert_array_equal(got_pos, np.where(exp >= 0, exp + off, -1))
    exp_val = np.where(exp >= 0, np.take_along_axis(s, np.maximum(exp, 0), axis=1), -np.inf)
    np.testing.assert_array_equal(p[:, :K], exp_val)
    assert int(hist.abs().sum()) == 0


def test_decode_exchange_single_rank_steps_and_timeout(dsa):
    """The device-sequenced decode exchange with one rank (its own slots):
    five steps in a row (slots alternate, ctl[0] advances, staged/merged
    flags follow), each exact against the oracle; then the merge's wait on a
    staged flag that runs out (the flag forced back after the stage): TIMEOUT
    is reported, merged is not published, and the context stays usable."""
    from importlib import import_module

    ops = import_module("glm5-on-v100_b200.ops")
    sai = import_module("glm5-on-v100_b200.sparse_attn_indexer")
    rng = np.random.default_rng(21)
    B, S, K = 6, 12000, 2048
    ex = sai.DecodeExchange(torch.device(DEV), 1, 0, K, 8, all_gather_object=lambda o, p: o.__setitem__(0, p))
    lens = np.array([12000, 11000, 3000, 2048, 17, 0], np.int32)
    dl = to_dev(lens)
    for step in range(5):
        s = rng.standard_normal((B, S)).astype(np.float32)
        score = to_dev(s)
        out = torch.full((B, K), -9, dtype=torch.int32, device=DEV)
        # odd steps with the fused histogram (the cluster kernel, B < SMs and
        # S >= 8192), even steps without it (one CTA per row)
        hist = to_dev(O.level1_hist(s, lens)) if step % 2 else None
        ex.topk_stage(score, dl, hist, 0)
        ex.merge(out, B)
        torch.cuda.synchronize()
        assert not ops.p2p_failed(DEV)
        exp = np.sort(O.topk_rows(s, lens, K), axis=1)
        np.testing.assert_array_equal(out.cpu().numpy(), exp)
        assert int(ex.ctl[0]) == step + 1
        assert ex.fbuf.view(torch.int32)[:2].tolist() == [step + 1, step + 1]
    old = ops.P2P_TIMEOUT_NS
    ops.P2P_TIMEOUT_NS = 50_000_000  # 50 ms
    try:
        s = rng.standard_normal((B, S)).astype(np.float32)
        ex.topk_stage(to_dev(s), dl, to_dev(O.level1_hist(s, lens)), 0)
        ex.fbuf.view(torch.int32)[0] = 0  # staged flag forced back: the step-6 merge wait (staged >= 6) cannot finish
        ex.merge(torch.empty(B, K, dtype=torch.int32, device=DEV), B)
        torch.cuda.synchronize()
        assert ops.p2p_failed(DEV)
        assert ex.fbuf.view(torch.int32)[:2].tolist() == [0, 5]  # merged not published
    finally:
        ops.P2P_TIMEOUT_NS = old
    x = torch.ones(4, device=DEV) * 2
    assert float(x.sum()) == 8.0


def test_ipc_alloc_handle(dsa):
    buf, handle = dsa.sm70_ipc_alloc(4096)
    assert buf.is_cuda and buf.numel() == 4096 and handle.numel() == 64
    assert int(buf.sum()) == 0
    buf.fill_(3)
    torch.cuda.synchronize()
    assert int(buf.sum()) == 3 * 4096
