"""GPU tests of the cache writers against the CPU oracle on the same inputs:
the fp8_ds_mla latent writer with the fused k_pe rotary embedding (bit-exact
cache rows: the quantisation is exact single-precision arithmetic and the
rotation's products and sums are rounded in f32 on both sides) and the
indexer's q / k / weights producer fused into the K store (LayerNorm sums in a
different order than the oracle's float64: every output within one rounding
step of its format)."""
import numpy as np
import pytest
import torch

from oracle import dsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def cos_sin_table(max_pos, base=10000.0):
    inv = 1.0 / base ** (np.arange(0, 64, 2, dtype=np.float64) / 64)
    f = np.outer(np.arange(max_pos, dtype=np.float64), inv)
    return np.concatenate([np.cos(f), np.sin(f)], axis=1).astype(np.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rope", ["neox", "gptj", "none"])
def test_concat_and_cache_ds_mla_bit_exact(dsa, dtype, rope):
    rng = np.random.default_rng(3 + (dtype == torch.float16) + 10 * ["neox", "gptj", "none"].index(rope))
    T, page, nb = 45, 64, 5
    n_rows = nb * page
    kv_c = torch.from_numpy(rng.standard_normal((T, 512)).astype(np.float32) * 3).to(dtype)
    kv_c[5] = 0.0                                   # an all-zero token: scale FLT_MIN, codes 0
    kv_c[6, :128] *= 1000.0                         # one tile far larger than the others
    k_pe = torch.from_numpy(rng.standard_normal((T, 64)).astype(np.float32)).to(dtype)
    slot = rng.permutation(n_rows)[:T].astype(np.int32)
    slot[3], slot[9] = -1, n_rows + 7               # skipped: padding and out of range
    pos = rng.integers(0, 4096, size=T).astype(np.int64)
    cs = cos_sin_table(4096)
    cache = torch.zeros(nb, page, 656, dtype=torch.uint8, device=DEV)
    kw = {}
    if rope != "none":
        kw = dict(positions=torch.from_numpy(pos).to(DEV), cos_sin_cache=torch.from_numpy(cs).to(DEV),
                  is_neox=rope == "neox")
    dsa.ops.concat_and_cache_mla(kv_c.to(DEV), k_pe.to(DEV), cache, torch.from_numpy(slot).to(DEV), "fp8_ds_mla",
                                 None, **kw)
    torch.cuda.synchronize()
    exp = np.zeros((n_rows, 656), np.uint8)
    ok = (slot >= 0) & (slot < n_rows)
    rows = O.dsmla_write_rows(kv_c.float().numpy(), k_pe.float().numpy(),
                              pos if rope != "none" else None, cs, rope == "neox")
    exp[slot[ok]] = rows[ok]
    np.testing.assert_array_equal(cache.cpu().numpy().reshape(n_rows, 656), exp)


def test_latent_writer_feeds_the_decode_kernel(dsa):
    """Rows written by the writer, read back by the sparse decode: the
    attention over them equals the oracle's over the dequantised rows."""
    rng = np.random.default_rng(8)
    page, nb, H, K = 64, 8, 16, 256
    n_rows = nb * page
    lat = rng.standard_normal((n_rows, 576)).astype(np.float32)
    cache = torch.zeros(nb, page, 656, dtype=torch.uint8, device=DEV)
    pos = np.arange(n_rows, dtype=np.int64)
    cs = cos_sin_table(n_rows)
    dsa.ops.concat_and_cache_mla(torch.from_numpy(lat[:, :512]).to(DEV).half(),
                                 torch.from_numpy(lat[:, 512:]).to(DEV).half(), cache,
                                 torch.arange(n_rows, dtype=torch.int32, device=DEV), "fp8_ds_mla",
                                 positions=torch.from_numpy(pos).to(DEV), cos_sin_cache=torch.from_numpy(cs).to(DEV))
    q = torch.from_numpy(rng.standard_normal((2, H, 576)).astype(np.float32)).to(DEV).to(torch.bfloat16)
    idx = torch.from_numpy(np.stack([np.sort(rng.choice(n_rows, K, replace=False)) for _ in range(2)])
                           .astype(np.int32)).to(DEV)
    bt = torch.arange(nb, dtype=torch.int32, device=DEV).view(1, nb).repeat(2, 1)
    seq = torch.full((2,), n_rows, dtype=torch.int32, device=DEV)
    o = torch.empty(2, H, 512, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(2, H, device=DEV)
    scale = 1.0 / np.sqrt(192.0)
    dsa.sm70_sparse_mla_decode(o, lse, q, cache, idx, bt, seq, scale)
    torch.cuda.synchronize()
    rows = O.dsmla_write_rows(torch.from_numpy(lat[:, :512]).half().float().numpy(),
                              torch.from_numpy(lat[:, 512:]).half().float().numpy(), pos, cs, False)
    np.testing.assert_array_equal(cache.cpu().numpy().reshape(n_rows, 656), rows)
    o_ref, lse_ref = O.sparse_mla_decode(q.float().cpu().numpy(), O.dsmla_decode_rows(rows), idx.cpu().numpy(),
                                         bt.cpu().numpy(), seq.cpu().numpy(), page, scale)
    rel = np.linalg.norm(o.float().cpu().numpy() - o_ref, axis=-1) / np.linalg.norm(o_ref, axis=-1)
    assert rel.max() < 6e-3  # bf16 output rounding (~1.7e-3) plus the 2e-3 kernel bound
    assert np.abs(lse.cpu().numpy() - lse_ref).max() < 2e-3


def _ulp_close(got, ref, dtype):
    """|got - ref| <= one unit in the last place of `dtype` at |ref|, plus
    an absolute floor of 1e-6 x max |ref| for the f32 arithmetic's own error
    where |ref| is near zero (a rotation's difference of products, a
    LayerNorm output near its mean)."""
    eps = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7, torch.float32: 2.0 ** -23}[dtype]
    bound = eps * np.abs(ref) + 1e-6 * np.abs(ref).max()
    assert np.all(np.abs(got - ref) <= bound * 1.0001), float(np.max(np.abs(got - ref) / bound))


@pytest.mark.parametrize("cache_fmt", ["fp8", "f16", "bf16"])
@pytest.mark.parametrize("neox", [True, False])
def test_indexer_qk_store(dsa, cache_fmt, neox):
    rng = np.random.default_rng(21 + 2 * ["fp8", "f16", "bf16"].index(cache_fmt) + neox)
    T, H, page, nb = 29, 32, 64, 2
    n_rows = nb * page
    dt = torch.bfloat16
    q = torch.from_numpy(rng.standard_normal((T, H, 128)).astype(np.float32)).to(dt)
    kw = torch.from_numpy(np.concatenate([rng.standard_normal((T, 128)) * 2 + 0.3,
                                          rng.standard_normal((T, H))], axis=1).astype(np.float32)).to(dt)
    ln_w = (1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    ln_b = (0.05 * rng.standard_normal(128)).astype(np.float32)
    slot = rng.permutation(n_rows)[:T].astype(np.int32)
    slot[4] = -1
    pos = rng.integers(0, 2048, size=T).astype(np.int64)
    cs = cos_sin_table(2048)
    w_scale = (128 ** -0.5) * H ** -0.5
    if cache_fmt == "fp8":
        cache = torch.zeros(nb, page, 132, dtype=torch.uint8, device=DEV)
    else:
        cache = torch.zeros(nb, page, 128, dtype=torch.float16 if cache_fmt == "f16" else torch.bfloat16, device=DEV)
    q_out = torch.empty(T, H, 128, dtype=torch.float16, device=DEV)
    w_out = torch.empty(T, H, dtype=torch.float32, device=DEV)
    dsa.ops.indexer_qk_store(q_out, w_out, cache, q.to(DEV), kw.to(DEV), torch.from_numpy(slot).to(DEV),
                             torch.from_numpy(ln_w).to(DEV), torch.from_numpy(ln_b).to(DEV), 1e-6,
                             torch.from_numpy(pos).to(DEV), torch.from_numpy(cs).to(DEV), neox, w_scale)
    torch.cuda.synchronize()
    q_ref, k_ref, w_ref = O.indexer_qk_produce(q.float().numpy(), kw.float().numpy(), ln_w, ln_b, 1e-6, pos, cs,
                                               neox, w_scale)
    _ulp_close(q_out.float().cpu().numpy().astype(np.float64), q_ref, torch.float16)
    _ulp_close(w_out.cpu().numpy().astype(np.float64), w_ref, torch.float32)
    ok = slot >= 0
    flat = cache.cpu().view(torch.uint8).numpy().reshape(n_rows, -1)
    untouched = np.setdiff1d(np.arange(n_rows), slot[ok])
    assert not flat[untouched].any()
    if cache_fmt == "fp8":
        rows = flat[slot[ok]]
        scale = rows[:, 128:132].copy().view(np.float32)[:, 0].astype(np.float64)
        s_ref = np.maximum(np.abs(k_ref[ok]).max(axis=1) / 448.0, np.finfo(np.float32).tiny)
        np.testing.assert_allclose(scale, s_ref, rtol=1e-6)
        y_ref = k_ref[ok] / scale[:, None]
        y = O.e4m3_decode(rows[:, :128])
        a = np.abs(y_ref)
        quantum = np.exp2(np.floor(np.log2(np.maximum(a, 2.0 ** -6))) - 3)
        assert np.all(np.abs(y - y_ref) <= quantum * 1.0001)  # at most one e4m3 step from the exact value
        assert np.mean(np.abs(y - y_ref) <= quantum / 2 * 1.0001) > 0.99  # nearly all rounded to nearest
    else:
        got = torch.from_numpy(flat[slot[ok]].copy()).view(cache.dtype).float().numpy().astype(np.float64)
        _ulp_close(got, k_ref[ok], cache.dtype)
