"""CPU: pin the oracle against fixtures produced by the reference's own code.

Fixtures are made by tests/golden/make_golden.py (which imports the reference);
here only the committed .npz files and the regenerated seeded inputs are used.
"""
import os

import numpy as np
import pytest
import torch

import cases
from oracle import dsa_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


@pytest.mark.parametrize("name", ["config1", "ragged"])
def test_sparse_decode_matches_reference_torch_path(name):
    f = _load(f"mqa_decode_{name}.npz")
    c = cases.decode_case(int(f["seed"]), int(f["B"]), int(f["H"]), int(f["page"]), f["seq_lens"], int(f["topk"]),
                          int(f["bps"]))
    assert cases.digest(c["q"], c["kv"], c["idx"], c["block_table"], c["seq_lens"]) == str(f["digest"])
    o, lse = O.sparse_mla_decode(c["q"], c["kv"].astype(np.float64), c["idx"], c["block_table"], c["seq_lens"],
                                 c["page"], float(f["scale"]))
    # reference computes in fp32; the oracle in fp64
    np.testing.assert_allclose(o, f["o"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(lse, f["lse"], atol=2e-6, rtol=0)


def test_sparse_equals_dense_prefill_reference():
    """Selecting every causal position reproduces the reference's dense varlen prefill."""
    f = _load("varlen_prefill.npz")
    S, T, H = int(f["S"]), int(f["T"]), int(f["H"])
    rng = np.random.default_rng(int(f["seed"]))
    q = cases.f16_exact(rng.standard_normal((T, H, 576)))
    kv = cases.f16_exact(rng.standard_normal((S, 576)))
    assert cases.digest(q, kv) == str(f["digest"])
    idx = np.full((T, S), -1, np.int32)
    for i in range(T):
        n = S - T + i + 1
        idx[i, :n] = np.arange(n)
    bt = np.tile(np.arange(S // 16, dtype=np.int32), (T, 1))
    o, lse = O.sparse_mla_decode(q, kv.astype(np.float64), idx, bt, np.full(T, S, np.int32), 16, float(f["scale"]))
    np.testing.assert_allclose(o, f["o"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(lse.T, f["lse"], atol=2e-6, rtol=0)


def tie_aware_equal(a_row, b_row, vals_of):
    """Equal selections up to members tied at the K-th value: the multisets of
    selected values agree and every differing member carries the K-th value
    (torch.topk's tie order is unspecified; sai.py:969-976 claims set equality)."""
    va = sorted(vals_of(x) for x in a_row.tolist())
    vb = sorted(vals_of(x) for x in b_row.tolist())
    if va != vb:
        return False
    kth = va[0]
    diff = set(a_row.tolist()) ^ set(b_row.tolist())
    return all(vals_of(x) == kth for x in diff)


def test_shard_merge_matches_reference_epilogue():
    f = _load("shard_merge.npz")
    allf, K = f["allf"], int(f["K"])
    ours = O.shard_merge(allf, K)
    ref = f["mi_sorted"]
    tp, R, _ = allf.shape
    for r in range(R):
        vals = {-1: -np.inf}
        for s in range(tp):
            pos = allf[s, r, K:].copy().view(np.int32)
            for c in range(K):
                if pos[c] >= 0:
                    vals[int(pos[c])] = float(allf[s, r, c])
        assert tie_aware_equal(ours[r], ref[r], vals.__getitem__), r
    # the torch restatement in the oracle reproduces the fixture bit for bit
    np.testing.assert_array_equal(O.shard_merge_torch_epilogue(allf, K), ref)


def test_e4m3_encoder_matches_torch_cast():
    rng = np.random.default_rng(0)
    x = np.concatenate([np.linspace(-500, 500, 20001),
                        rng.standard_normal(50000) * np.exp2(rng.integers(-14, 9, 50000)),
                        [0.0, -0.0, 448.0, -448.0, 464.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11]]).astype(np.float32)
    t = torch.from_numpy(np.clip(x, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(O.e4m3_encode_satfinite(x), t)
    codes = np.arange(256, dtype=np.uint8)
    ok = ~np.isnan(O.e4m3_decode(codes))
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(O.e4m3_decode(codes)[ok], ref[ok])


def test_dsmla_roundtrip_error_bound():
    rng = np.random.default_rng(3)
    lat = rng.standard_normal((64, 576)).astype(np.float32)
    rows = O.dsmla_encode_rows(lat)
    back = O.dsmla_decode_rows(rows)
    # e4m3 has 3 mantissa bits: relative rounding <= 2^-4 of the tile's values
    err = np.abs(back[:, :512] - lat[:, :512])
    assert np.all(err <= np.abs(lat[:, :512]) * 2.0 ** -4 + 2.0 ** -9 * np.abs(lat[:, :512]).max())
    np.testing.assert_array_equal(back[:, 512:], lat[:, 512:].astype(np.float16).astype(np.float64))


def test_topk_rows_oracle_tie_rule():
    s = np.array([[1, 3, 3, 2, 3, 0]], np.float32)
    np.testing.assert_array_equal(O.topk_rows(s, [6], 2), [[1, 2]])
    np.testing.assert_array_equal(O.topk_rows(s, [6], 4), [[1, 2, 3, 4]])
    np.testing.assert_array_equal(O.topk_rows(s, [3], 4), [[0, 1, 2, -1]])


def test_global_topk_subset_of_shard_union():
    """The reference's exactness argument for key sharding (full.patch:4778-4786)."""
    rng = np.random.default_rng(5)
    R, S, K, tp = 6, 3000, 128, 4
    score = rng.standard_normal((R, S)).astype(np.float32)
    lens = np.array([3000, 2999, 1500, 129, 700, 2500])
    full = O.topk_rows(score, lens, K)
    payload = []
    for rank in range(tp):
        off, span = O.shard_span(S, tp, rank, page=64)
        v, g = O.sharded_local_candidates(score, lens, K, off, span, rank)
        payload.append(np.concatenate([v, g.view(np.float32)], axis=1))
    merged = O.shard_merge(np.stack(payload), K)
    np.testing.assert_array_equal(np.sort(full, axis=1), merged)


def test_rope_oracle_matches_vllm_rotary_embedding():
    """The writers' rotary embedding (oracle.rope_f32) equals vLLM's own
    PyTorch implementation (RotaryEmbedding.forward_static, the rotary the
    reference's model code calls) bit for bit in f32, in both pair orders."""
    import torch

    try:
        from vllm.model_executor.layers.rotary_embedding.base import RotaryEmbedding
    except Exception as e:  # pragma: no cover - vLLM is part of this image
        pytest.skip(f"vLLM rotary embedding not importable: {e}")
    rng = np.random.default_rng(4)
    inv = 1.0 / 10000.0 ** (np.arange(0, 64, 2, dtype=np.float64) / 64)
    f = np.outer(np.arange(1024, dtype=np.float64), inv)
    cs = np.concatenate([np.cos(f), np.sin(f)], axis=1).astype(np.float32)
    x = rng.standard_normal((17, 64)).astype(np.float32)
    pos = rng.integers(0, 1024, size=17)
    for neox in (True, False):
        _, k = RotaryEmbedding.forward_static(torch.from_numpy(pos), torch.zeros(17, 64),
                                              torch.from_numpy(x.copy()), 64, 64, torch.from_numpy(cs), neox)
        np.testing.assert_array_equal(O.rope_f32(x, pos, cs, neox), k.numpy())
