"""GPU test of dsa_sparse_mla_decode_noalloc, the decode entry point that
allocates nothing.

Some callers cannot allocate device memory when they decode: an engine whose
pool allocator owns the whole GPU, a plugin host that passes only input and
output buffers. This entry point keeps the split partial states in one static
32 MiB array inside the library instead of a caller workspace. The test calls
it through the C ABI and checks it against dsa_sparse_mla_decode (given a
workspace the test allocates) on two calls in a row with different inputs.
The second call finds the first call's partial states still in the shared
array, which it must not need to be cleared. The tolerance is the one of the
other attention tests: 2e-3 relative error per (row, head) on o, 2e-3 absolute
on lse. A call that needs more scratch than the array holds must be rejected
before it launches anything.

The file name makes pytest collect it last.
"""
import ctypes
import importlib
import re

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
L = importlib.import_module("glm5-on-v100_b200._lib")
DEV = "cuda"
ATTN_RTOL = 2e-3
LSE_ATOL = 2e-3
SCRATCH_BYTES = 32 << 20
H, PAGE, SCALE = 64, 64, 1.0 / np.sqrt(192.0)


def make_inputs(seed, fmt, B, seq_len, topk):
    """Random decode inputs on the GPU: a paged cache (fp8_ds_mla rows or bf16),
    a shuffled block table and sorted distinct positions per row."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    bps = (seq_len + PAGE - 1) // PAGE
    nb = B * bps + 2
    if fmt == "fp8":
        kv = torch.randint(0, 256, (nb, PAGE, 656), dtype=torch.uint8, device=DEV, generator=g)
        codes = kv[..., :512]
        codes[(codes & 0x7F) == 0x7F] = 0x7E  # no NaN codes
        sc = (torch.rand(nb, PAGE, 4, device=DEV, generator=g) + 0.5) / 448.0
        kv[..., 512:528] = sc.contiguous().view(torch.uint8).view(nb, PAGE, 16)
        rope = torch.randn(nb, PAGE, 64, device=DEV, generator=g).to(torch.float16)
        kv[..., 528:656] = rope.view(torch.uint8).view(nb, PAGE, 128)
        kv_format = L.DSA_FP8_DS_MLA
    else:
        kv = torch.randn(nb, PAGE, 576, device=DEV, generator=g).to(torch.bfloat16)
        kv_format = L.DSA_BF16
    bt = torch.randperm(nb, device=DEV, generator=g)[: B * bps].view(B, bps).to(torch.int32).contiguous()
    idx = torch.stack([torch.randperm(seq_len, device=DEV, generator=g)[:topk].sort().values
                       for _ in range(B)]).to(torch.int32).contiguous()
    q = torch.randn(B, H, 576, device=DEV, generator=g).to(torch.bfloat16)
    seq_lens = torch.full((B,), seq_len, dtype=torch.int32, device=DEV)
    return dict(q=q, kv=kv, kv_format=kv_format, bt=bt, idx=idx, seq_lens=seq_lens, B=B, topk=topk)


def decode_args(x, o, lse):
    """Arguments shared by both entry points, up to and including scale."""
    return (o.data_ptr(), L.DSA_BF16, lse.data_ptr(), x["q"].data_ptr(), L.DSA_BF16, x["kv"].data_ptr(),
            x["kv_format"], x["kv"].shape[0] * PAGE, PAGE, x["idx"].data_ptr(), x["idx"].stride(0),
            x["bt"].data_ptr(), x["bt"].stride(0), x["bt"].shape[1], x["seq_lens"].data_ptr(), x["B"], H,
            x["topk"], SCALE)


def outputs(B):
    return (torch.full((B, H, 512), float("nan"), dtype=torch.bfloat16, device=DEV),
            torch.full((B, H), float("nan"), dtype=torch.float32, device=DEV))


def run_with_workspace(x):
    o, lse = outputs(x["B"])
    ws_bytes = L.lib().dsa_sparse_mla_decode_workspace_bytes(x["B"], H, x["topk"])
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=DEV)
    L.call("dsa_sparse_mla_decode", *decode_args(x, o, lse), ws.data_ptr(), ws_bytes,
           torch.cuda.current_stream().cuda_stream)
    return o, lse


def run_no_alloc(x):
    o, lse = outputs(x["B"])
    L.call("dsa_sparse_mla_decode_noalloc", *decode_args(x, o, lse), torch.cuda.current_stream().cuda_stream)
    return o, lse


def assert_close(o, lse, o_ref, lse_ref):
    o, o_ref = o.float().cpu().numpy(), o_ref.float().cpu().numpy()
    lse, lse_ref = lse.cpu().numpy(), lse_ref.cpu().numpy()
    assert np.isfinite(o).all() and np.isfinite(lse).all()
    err = np.linalg.norm(o - o_ref, axis=-1)
    ref = np.linalg.norm(o_ref, axis=-1)
    assert (err <= ATTN_RTOL * ref).all(), f"max rel {(err / ref).max():.3e}"
    assert np.abs(lse - lse_ref).max() <= LSE_ATOL


@pytest.mark.parametrize("fmt", ["fp8", "bf16"])
def test_no_alloc_matches_workspace_entry_twice(fmt):
    # small batches, so the decode splits each row into several slices and the
    # partial states really go through the static scratch
    cases = [make_inputs(11, fmt, B=4, seq_len=8192, topk=2048),
             make_inputs(12, fmt, B=6, seq_len=5000, topk=1536)]
    for x in cases:
        assert L.lib().dsa_sparse_mla_decode_workspace_bytes(x["B"], H, x["topk"]) > 0
    for x in cases:  # two calls in a row, each checked against the workspace entry point
        o, lse = run_no_alloc(x)
        torch.cuda.synchronize()
        o_ref, lse_ref = run_with_workspace(x)
        torch.cuda.synchronize()
        assert_close(o, lse, o_ref, lse_ref)


def plan(B, topk, kv_format):
    s, c, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    ws = ctypes.c_size_t()
    assert L.lib().dsa_sparse_mla_decode_plan(B, H, topk, kv_format, ctypes.byref(s), ctypes.byref(c),
                                              ctypes.byref(ws), ctypes.byref(n)) == L.DSA_OK
    return s.value, c.value, ws.value


def test_no_alloc_cases_use_partial_states():
    # the fp8 cases above split into slice counts the kernel merges through
    # partial states (not inside a cluster), so they exercise the scratch
    for B, topk in [(4, 2048), (6, 1536)]:
        s, c, ws = plan(B, topk, L.DSA_FP8_DS_MLA)
        assert s > 1 and c == 1 and 0 < ws <= SCRATCH_BYTES, (B, topk, s, c, ws)


def test_no_alloc_rejects_calls_beyond_the_scratch():
    # many rows with long top-k lists on the bf16 cache (whose kernel always
    # merges slices through partial states): one that needs > 32 MiB
    cand = [(B, topk) for B, topk in [(200, 16384), (400, 16384), (1000, 8192)]
            if plan(B, topk, L.DSA_BF16)[2] > SCRATCH_BYTES]
    assert cand, "no candidate shape needs more than the static scratch"
    B, topk = cand[0]
    q = torch.zeros(B, H, 576, dtype=torch.bfloat16, device=DEV)
    kv = torch.zeros(1, PAGE, 576, dtype=torch.bfloat16, device=DEV)
    idx = torch.zeros(B, topk, dtype=torch.int32, device=DEV)
    bt = torch.zeros(B, 1, dtype=torch.int32, device=DEV)
    x = dict(q=q, kv=kv, kv_format=L.DSA_BF16, bt=bt, idx=idx,
             seq_lens=torch.ones(B, dtype=torch.int32, device=DEV), B=B, topk=topk)
    o, lse = outputs(B)
    stream = torch.cuda.current_stream().cuda_stream
    lib = L.lib()
    # the workspace entry point without a workspace states what this call needs
    st = lib.dsa_sparse_mla_decode(*decode_args(x, o, lse), None, ctypes.c_size_t(0), stream)
    assert st == L.DSA_ERR_WORKSPACE
    need = int(re.search(r"workspace needs (\d+) bytes", lib.dsa_last_error().decode()).group(1))
    assert need > SCRATCH_BYTES
    st = lib.dsa_sparse_mla_decode_noalloc(*decode_args(x, o, lse), stream)
    assert st == L.DSA_ERR_WORKSPACE
    assert "static" in lib.dsa_last_error().decode()
    torch.cuda.synchronize()
    assert torch.isnan(lse).all()  # nothing was launched
