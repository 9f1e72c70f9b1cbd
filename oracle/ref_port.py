"""CPU port of the reference's own torch decode path — TEST / BASELINE ONLY.

Restates ``TritonMLAImpl._forward_mqa_torch`` (reference/triton_mla.py:494-554)
in torch on the host cores: gather the paged latent rows into a fixed-width
buffer, bmm scores in fp32, mask positions >= seq_len, safe-max softmax, bmm
with the value part. The sparse form uses the page-size-1 view the golden
fixtures pin (block table = physical rows of the valid top-k positions), and
the fp8_ds_mla rows are dequantised on the host first (csrc/attention/
sm70_mla_decode.cu:74-100), as the reference's CPU path would have to.

Only bench.py's CPU-baseline legs and tests use this module.
"""
from __future__ import annotations

import torch


def dequant_dsmla(rows_u8: torch.Tensor) -> torch.Tensor:
    """[n, 656] uint8 -> [n, 576] float32."""
    n = rows_u8.shape[0]
    nope = rows_u8[:, :512].contiguous().view(torch.float8_e4m3fn).float().view(n, 4, 128)
    scale = rows_u8[:, 512:528].contiguous().view(torch.float32).view(n, 4, 1)
    rope = rows_u8[:, 528:656].contiguous().view(torch.float16).float()
    return torch.cat([(nope * scale).view(n, 512), rope], dim=1)


def forward_mqa_torch(q, cache_rows, block_table, seq_lens, page, scale, kv_lora_rank=512):
    """tmla.py:494-554 on a flat row cache [n_rows, 576] float32."""
    B, H, Lk = q.shape
    max_blocks = block_table.shape[1]
    max_kv = max_blocks * page
    blk = block_table.to(torch.long)
    rows = (blk * page).unsqueeze(-1) + torch.arange(page).view(1, 1, page)
    rows = rows.reshape(B, max_kv).clamp_(0, cache_rows.shape[0] - 1)
    kv = cache_rows.index_select(0, rows.reshape(-1)).reshape(B, max_kv, Lk)
    scores = torch.bmm(q.float(), kv.transpose(1, 2).float()) * scale
    pos = torch.arange(max_kv).view(1, max_kv)
    valid = pos < seq_lens.view(B, 1)
    scores = scores.masked_fill(~valid.unsqueeze(1), float("-inf"))
    m = scores.max(dim=-1, keepdim=True).values
    m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    p = torch.exp(scores - m_safe)
    denom = p.sum(dim=-1, keepdim=True)
    o = torch.bmm(p.to(kv.dtype), kv[..., :kv_lora_rank]) / denom
    lse = m_safe.squeeze(-1) + torch.log(denom.squeeze(-1))
    return o, lse


def sparse_decode_cpu(q, kv_u8_flat, idx, block_table, seq_lens, page, scale):
    """Sparse decode through the reference torch path: page-size-1 block table
    over the selected rows of an fp8_ds_mla cache [n_rows, 656] (uint8)."""
    B = q.shape[0]
    valid = (idx >= 0) & (idx < seq_lens.view(B, 1))
    pos = idx.clamp(min=0).to(torch.long)
    phys = torch.gather(block_table.to(torch.long), 1, pos // page) * page + pos % page
    counts = valid.sum(dim=1)
    # valid rows first (stable), then padding: the page-size-1 table of the fixtures
    order = torch.argsort((~valid).to(torch.int8), dim=1, stable=True)
    phys = torch.gather(phys, 1, order)
    sel = phys.reshape(-1)
    rows = dequant_dsmla(kv_u8_flat.index_select(0, sel))
    local_bt = torch.arange(sel.numel()).view(B, -1)
    return forward_mqa_torch(q, rows, local_bt, counts, 1, scale)


def indexer_prefill_cpu(q, k_rows, w, lens, K):
    """Indexer prefill on the host: score[i, p] = sum_h w[i,h] * relu(q[i,h,:] . k_p)
    for p < lens[i] (csrc/attention/sm70_mla_decode.cu:132-149, :332-344),
    then the per-row top-K positions (torch.topk, the selection the reference's
    torch shard-merge epilogue uses, reference/sparse_attn_indexer.py:1020).

    q [n, Hi, 128], k_rows [max_len, 128] (the request's keys in position
    order), w [n, Hi], lens [n]. The reference has no CPU implementation of
    this step (its logits are SM70 CUDA kernels), so this is a restatement.
    """
    out = torch.full((q.shape[0], K), -1, dtype=torch.int32)
    kf = k_rows.float()
    for i in range(q.shape[0]):
        n = int(lens[i])
        s = torch.relu(q[i].float() @ kf[:n].T)          # [Hi, n]
        score = (w[i].float().view(-1, 1) * s).sum(0)      # [n]
        k = min(K, n)
        out[i, :k] = torch.topk(score, k).indices.sort().values.to(torch.int32)
    return out
