"""Sparse MLA attention glue — the callers of the sparse attention op.

Mirrors ``TritonMLAImpl._forward_mqa_sparse`` (reference/triton_mla.py:212-302)
and ``_forward_mha_sparse`` (:350-492) without the vLLM backend object: the
metadata the reference reads from ``attn_metadata`` is passed explicitly.
"""
from __future__ import annotations

import torch

from . import ops


def expand_spec_rows(seq_lens: torch.Tensor, block_table: torch.Tensor, n_tokens: int):
    """Spec-as-decode row expansion (triton_mla.py:261-279).

    With uniform verify steps of next_n = n_tokens / n_req query tokens per
    request, token j of request b sits at position seq_lens[b] - next_n + j,
    so its causal length is seq_lens[b] - (next_n - 1) + j and it uses request
    b's block-table row. Static shapes: CUDA-graph safe.
    """
    if seq_lens.dim() == 2:
        seq_lens = seq_lens[:, -1]
    seq_lens = seq_lens.contiguous().to(torch.int32)
    block_table = block_table.to(torch.int32)
    n_req = seq_lens.shape[0]
    if n_tokens == n_req:
        return seq_lens, block_table
    if n_tokens % n_req != 0:
        raise RuntimeError(f"non-uniform decode batch: {n_tokens} tokens, {n_req} requests")
    next_n = n_tokens // n_req
    offs = torch.arange(next_n, device=seq_lens.device, dtype=torch.int32)
    seq = (seq_lens.unsqueeze(1) - (next_n - 1) + offs).reshape(-1).contiguous()
    bt = block_table.repeat_interleave(next_n, dim=0).contiguous()
    return seq, bt


def forward_mqa_sparse(q: torch.Tensor, kv_cache: torch.Tensor, topk_indices_buffer: torch.Tensor,
                       topk_tokens: int, block_table: torch.Tensor, seq_lens: torch.Tensor, scale: float,
                       kv_lora_rank: int = 512):
    """Sparse (top-k) MLA decode over the paged latent cache.

    q [B, H, 576]; kv_cache fp16/bf16 [nb, page, 576] or uint8 fp8_ds_mla
    [nb, page, 656] (passed raw: the kernel dequantises in its gather);
    the top-k rows of the decode tokens are the first B rows of
    topk_indices_buffer. Returns (o [B, H, 512] in q's dtype, lse [B, H] f32).
    """
    B, H, _ = q.shape
    idx = topk_indices_buffer[:B, :topk_tokens]
    if idx.dtype != torch.int32:
        idx = idx.to(torch.int32)
    seq, bt = expand_spec_rows(seq_lens, block_table, B)
    out_dtype = q.dtype if q.dtype in (torch.float16, torch.bfloat16) else torch.float16
    qk = q if q.dtype == out_dtype and q.is_contiguous() else q.to(out_dtype).contiguous()
    o = torch.empty(B, H, kv_lora_rank, dtype=out_dtype, device=q.device)
    lse = torch.empty(B, H, dtype=torch.float32, device=q.device)
    if kv_cache.dtype not in (torch.uint8, torch.float16, torch.bfloat16):
        kv_cache = kv_cache.to(torch.float16)
    ops.sm70_sparse_mla_decode(o, lse, qk, kv_cache, idx, bt, seq, float(scale))
    return o, lse


def per_token_metadata(chunks, nd0: int, q_len: int, query_start_loc: torch.Tensor, block_table: torch.Tensor):
    """Per-token causal lengths and block-table rows for sparse prefill
    (triton_mla.py:414-466): validates that the indexer's chunk entries
    (tok_lo, n_q, ke) tile [nd0, nd0 + q_len) and maps each token to its
    request through query_start_loc."""
    ok = bool(chunks)
    if ok:
        expect = nd0
        for tl, n, _ in chunks:
            if tl != expect:
                ok = False
                break
            expect = tl + n
        ok = ok and (expect - nd0) == q_len
    if not ok:
        raise RuntimeError("sparse prefill: indexer per-token metadata missing/mismatched (chunks="
                           f"{[(e[0], e[1]) for e in chunks] if chunks else None}, need [{nd0}, {nd0 + q_len}))")
    seq = (chunks[0][2] if len(chunks) == 1 else torch.cat([e[2] for e in chunks])).to(torch.int32)
    req_id = (torch.searchsorted(query_start_loc,
                                 torch.arange(q_len, device=query_start_loc.device, dtype=query_start_loc.dtype),
                                 right=True) - 1).clamp_(min=0)
    bt = block_table.to(torch.int32).index_select(0, req_id.to(torch.long)).contiguous()
    return seq.contiguous(), bt


def forward_mha_sparse(q: torch.Tensor, kv_cache: torch.Tensor, topk_indices_buffer: torch.Tensor,
                       topk_tokens: int, nd0: int, chunks, query_start_loc: torch.Tensor,
                       block_table: torch.Tensor, W_UK_T: torch.Tensor, W_UV: torch.Tensor, scale: float,
                       qk_nope_head_dim: int = 192, qk_rope_head_dim: int = 64) -> torch.Tensor:
    """Sparse prefill attention (triton_mla.py:350-492).

    q [q_len, H, qk_nope + qk_rope]; W_UK_T [H, qk_nope, 512]; W_UV [H, 512, V].
    Projects q_nope to the latent space, attends each token's top-k causal
    keys through the sparse op, and up-projects with W_UV. Returns
    [q_len, H * V] in q's dtype.
    """
    q_len, H, _ = q.shape
    q_nope, q_pe = q.split([qk_nope_head_dim, qk_rope_head_dim], dim=-1)
    ql_nope = torch.bmm(q_nope.transpose(0, 1), W_UK_T).transpose(0, 1)
    q_latent = torch.cat([ql_nope, q_pe], dim=-1)
    seq, bt = per_token_metadata(chunks, nd0, q_len, query_start_loc, block_table)
    idx = topk_indices_buffer[nd0:nd0 + q_len, :topk_tokens]
    if idx.dtype != torch.int32:
        idx = idx.to(torch.int32)
    dt = q.dtype if q.dtype in (torch.float16, torch.bfloat16) else torch.float16
    o = torch.empty(q_len, H, W_UK_T.shape[-1], dtype=dt, device=q.device)
    lse = torch.empty(q_len, H, dtype=torch.float32, device=q.device)
    ops.sm70_sparse_mla_decode(o, lse, q_latent.to(dt).contiguous(), kv_cache, idx, bt, seq, float(scale))
    o_nbv = torch.bmm(o.to(q.dtype).transpose(0, 1), W_UV.to(q.dtype))
    return o_nbv.transpose(0, 1).reshape(q_len, H * W_UV.shape[-1])
