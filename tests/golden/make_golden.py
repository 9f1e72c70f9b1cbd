"""Generate golden fixtures by running the REFERENCE's own Python code.

Run in the build container (it imports the read-only reference checkout, which
does not exist on GPU boxes):

    python tests/golden/make_golden.py /path/to/reference

Writes tests/golden/*.npz. Each fixture stores the generator parameters, a
digest of the regenerated inputs and the reference outputs:

  * mqa_decode_*.npz — TritonMLAImpl._forward_mqa_torch (reference/triton_mla.py
    :494-554), called unbound on a page-size-1 view whose block table lists the
    physical rows of each row's valid top-k positions (seq_lens = their count),
    which makes the reference's dense torch decode compute sparse attention.
  * varlen_prefill.npz — _varlen_attention (vllm/v1/attention/backends/mla/
    prefill/sm70_triton.py:54-187), dense causal prefill; the sparse kernel with
    every causal position selected must equal it (the reference's own gate,
    the reference's docs/INTEGRATION.md:124-128).
  * shard_merge.npz — the torch.topk shard-merge epilogue
    (reference/sparse_attn_indexer.py:1007-1030), executed from the reference
    source text on a seeded all-gather payload with ties and -inf entries.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import textwrap
from types import SimpleNamespace

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _page1_view(kv, idx, bt, seq_lens, page):
    """Block table of physical rows of the valid positions, page size 1."""
    B = idx.shape[0]
    rows = []
    for b in range(B):
        pos = idx[b][(idx[b] >= 0) & (idx[b] < seq_lens[b])].astype(np.int64)
        rows.append(bt[b][pos // page].astype(np.int64) * page + pos % page)
    n = max(1, max(len(r) for r in rows))
    bt1 = np.zeros((B, n), dtype=np.int64)
    sl1 = np.zeros(B, dtype=np.int64)
    for b, r in enumerate(rows):
        bt1[b, : len(r)] = r
        sl1[b] = len(r)
    return bt1, sl1


def mqa_decode_fixture(tmla, name, seed, B, H, page, seq_lens, topk, bps, scale):
    import torch

    c = cases.decode_case(seed, B, H, page, seq_lens, topk, bps)
    bt1, sl1 = _page1_view(c["kv"], c["idx"], c["block_table"], c["seq_lens"], page)
    impl = SimpleNamespace(scale=scale, kv_lora_rank=512)
    md = SimpleNamespace(decode=SimpleNamespace(block_table=torch.from_numpy(bt1),
                                                seq_lens=torch.from_numpy(sl1)))
    cache1 = torch.from_numpy(c["kv"]).reshape(-1, 1, 576)
    o, lse = tmla.TritonMLAImpl._forward_mqa_torch(impl, torch.from_numpy(c["q"]), cache1, md)
    np.savez_compressed(
        os.path.join(HERE, f"mqa_decode_{name}.npz"),
        seed=seed, B=B, H=H, page=page, seq_lens=np.asarray(seq_lens, np.int32),
        topk=topk, bps=bps, scale=scale,
        digest=cases.digest(c["q"], c["kv"], c["idx"], c["block_table"], c["seq_lens"]),
        o=o.numpy().astype(np.float32), lse=lse.numpy().astype(np.float32))
    print(f"mqa_decode_{name}: o {tuple(o.shape)} lse {tuple(lse.shape)}")


def varlen_fixture(st):
    import torch

    st._kv_block_size = lambda: 32  # fork-only env flag is absent here
    rng = np.random.default_rng(7)
    S, T, H = 96, 8, 4
    scale = 1.0 / np.sqrt(192.0)
    q = cases.f16_exact(rng.standard_normal((T, H, 576)))
    kv = cases.f16_exact(rng.standard_normal((S, 576)))
    k = torch.from_numpy(kv)[:, None, :].expand(S, H, 576).contiguous()
    v = torch.from_numpy(kv[:, :512])[:, None, :].expand(S, H, 512).contiguous()
    cu_q = torch.tensor([0, T], dtype=torch.int32)
    cu_k = torch.tensor([0, S], dtype=torch.int32)
    out, lse = st._varlen_attention(torch.from_numpy(q), k, v, cu_q, cu_k, scale, True, True)
    np.savez_compressed(os.path.join(HERE, "varlen_prefill.npz"),
                        seed=7, S=S, T=T, H=H, scale=scale,
                        digest=cases.digest(q, kv),
                        o=out.numpy().astype(np.float32), lse=lse.numpy().astype(np.float32))
    print("varlen_prefill:", tuple(out.shape))


def _epilogue_source(sai_path):
    """The torch.topk shard-merge epilogue block (sparse_attn_indexer.py:1007-1030)."""
    lines = open(sai_path).read().splitlines()
    start = next(i for i, l in enumerate(lines) if l.strip() == "av = (")
    end = next(i for i in range(start, len(lines))
               if lines[i].strip() == ").to(torch.int32)")
    return textwrap.dedent("\n".join(lines[start:end + 1]))


def shard_merge_fixture(sai_path):
    import torch

    src = _epilogue_source(sai_path)
    rng = np.random.default_rng(11)
    tp, R, K = 4, 6, 64
    vals = rng.standard_normal((tp, R, K)).astype(np.float32)
    vals = np.round(vals * 4) / 4  # many exact ties
    vals[0, 1, :5] = -np.inf
    vals[2, 3, :] = -np.inf
    vals[1, 4, 10:] = -np.inf
    # distinct positions per row, so a position identifies its candidate
    pos = np.stack([rng.permutation(100000)[: tp * K].reshape(tp, K) for _ in range(R)], axis=1).astype(np.int32)
    pos[vals == -np.inf] = -1
    allf = np.concatenate([vals, pos.view(np.float32)], axis=2)
    ns = dict(torch=torch, allf=torch.from_numpy(allf.copy()), R=R, K=K, shard_tp=tp)
    exec(src, ns)
    mi = ns["mi"].numpy()
    np.savez_compressed(os.path.join(HERE, "shard_merge.npz"), allf=allf, K=K,
                        mi_sorted=np.sort(mi, axis=1).astype(np.int32),
                        epilogue_source=np.array(src))
    print("shard_merge:", mi.shape)


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    ref = sys.argv[1]
    tmla = _load("ref_triton_mla", os.path.join(ref, "reference/triton_mla.py"))
    st = _load("ref_sm70_triton",
               os.path.join(ref, "vllm/v1/attention/backends/mla/prefill/sm70_triton.py"))
    # the CPU-runnable decode case: B=1, 16 heads, 2,048 cached tokens, top-k 512, scale 1/sqrt(192)
    mqa_decode_fixture(tmla, "config1", seed=1, B=1, H=16, page=64,
                       seq_lens=[2048], topk=512, bps=32, scale=1.0 / np.sqrt(192.0))
    # ragged batch: short rows (seq_len < topk, -1 padding), long rows, odd head count
    mqa_decode_fixture(tmla, "ragged", seed=2, B=4, H=12, page=16,
                       seq_lens=[5, 300, 64, 257], topk=128, bps=20,
                       scale=0.0625)
    varlen_fixture(st)
    shard_merge_fixture(os.path.join(ref, "reference/sparse_attn_indexer.py"))


if __name__ == "__main__":
    main()
