"""Paged KV-cache indexing (TEST INFRASTRUCTURE ONLY).

The reference's decode keeps each chip's KV contiguous per position (``model.py:1421-1438``); paged block-64
KV appears in its prefill (``prefill/pp_prefill.py:204-210``: ``[blocks, NKV, 64, HD]``) and in the handoff
that converts pages back to positions (``pp_prefill.py:1243-1244``). This build keeps the decode KV paged
(BASELINE: paged KV, block 64): position p of a user lives in page ``page_table[p // 64]``, row ``p % 64``.
These helpers are the bit-exact contract for that indexing.
"""
import torch

BLOCK = 64


def slot_of(page_table, pos):
    """(page, row) of position pos"""
    return int(page_table[pos // BLOCK]), pos % BLOCK


def scatter(pool, page_table, rows, heads=None):
    """write contiguous rows [nkv, P, HD] (positions 0..P-1) into pool [pages, nkv, 64, HD]"""
    nkv, P, _ = rows.shape
    for p in range(P):
        pg, r = slot_of(page_table, p)
        pool[pg, :, r] = rows[:, p]
    return pool


def gather(pool, page_table, P):
    """contiguous [nkv, P, HD] view of positions 0..P-1"""
    nkv = pool.shape[1]
    out = torch.empty(nkv, P, pool.shape[-1], dtype=pool.dtype)
    for p in range(P):
        pg, r = slot_of(page_table, p)
        out[:, p] = pool[pg, :, r]
    return out
