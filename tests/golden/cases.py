"""Seeded input generators shared by the golden-fixture script and the tests.

Inputs are regenerated from (seed, shape) with numpy's PCG64 generator; each
fixture also stores a digest of the generated inputs so a generator change is
caught instead of silently comparing against different data.
"""
from __future__ import annotations

import hashlib

import numpy as np


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def f16_exact(x: np.ndarray) -> np.ndarray:
    """Round to the nearest float16 and return as float32 (exactly representable)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def permuted_block_table(rng, B: int, blocks_per_seq: int, n_blocks: int):
    """Each sequence gets distinct physical blocks drawn from a random permutation."""
    assert B * blocks_per_seq <= n_blocks
    perm = rng.permutation(n_blocks)[: B * blocks_per_seq]
    return perm.reshape(B, blocks_per_seq).astype(np.int32)


def sorted_topk_positions(rng, seq_len: int, topk: int) -> np.ndarray:
    """topk distinct positions < seq_len, ascending (all positions when seq_len <= topk, -1 padded)."""
    out = np.full(topk, -1, dtype=np.int32)
    if seq_len <= topk:
        out[:seq_len] = np.arange(seq_len, dtype=np.int32)
    else:
        out[:] = np.sort(rng.choice(seq_len, size=topk, replace=False)).astype(np.int32)
    return out


def decode_case(seed: int, B: int, H: int, page: int, seq_lens, topk: int,
                blocks_per_seq: int, spare_blocks: int = 3):
    """Sparse MLA decode inputs with float16-exact values.

    Returns dict(q [B,H,576] f32, kv [n_rows,576] f32, idx [B,topk] i32,
    block_table [B,bps] i32, seq_lens [B] i32, page).
    """
    rng = np.random.default_rng(seed)
    n_blocks = B * blocks_per_seq + spare_blocks
    bt = permuted_block_table(rng, B, blocks_per_seq, n_blocks)
    q = f16_exact(rng.standard_normal((B, H, 576)))
    kv = f16_exact(rng.standard_normal((n_blocks * page, 576)))
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    idx = np.stack([sorted_topk_positions(rng, int(s), topk) for s in seq_lens])
    return dict(q=q, kv=kv, idx=idx, block_table=bt, seq_lens=seq_lens, page=page)
