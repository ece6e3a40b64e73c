"""ColdStore-exact page layout on the device.

A ColdStore record stores K and V payloads head-major, [kv_heads][tokens][D]
bf16 per page (src/cold_store.rs:725-742); GpuRegionStore::append_batch
transposes token-major rows into that layout (src/gpu_region_store.rs:470-483)
and maps each token to (page, offset).  Here the pages live in one device pool
[n_pages][KVH][page_tokens][D] addressed through an int32 page table, so the
decode kernel reads them in place.  Building a pool from token-major K/V is a
device-side scatter (torch indexing), used by tests and the benchmark to lay
out synthetic data; the serving path appends with mslim_cuda_rope_append_paged.
"""
from __future__ import annotations

import numpy as np


def scatter_to_pages(torch, k_tm, v_tm, page_row: np.ndarray, k_pool, v_pool, page_tokens: int) -> None:
    """Writes token-major k_tm/v_tm [T][KVH][D] of one sequence into the pool
    pages listed in page_row (logical page i -> physical page page_row[i])."""
    T = k_tm.shape[0]
    npages = (T + page_tokens - 1) // page_tokens
    for lp in range(npages):
        phys = int(page_row[lp])
        n = min(page_tokens, T - lp * page_tokens)
        k_pool[phys, :, :n, :] = k_tm[lp * page_tokens:lp * page_tokens + n].transpose(0, 1)
        v_pool[phys, :, :n, :] = v_tm[lp * page_tokens:lp * page_tokens + n].transpose(0, 1)


def gather_from_pages(torch, pool, page_row: np.ndarray, tokens: int, page_tokens: int):
    """Token-major [tokens][KVH][D] view of one sequence's pages (a copy)."""
    npages = (tokens + page_tokens - 1) // page_tokens
    idx = torch.as_tensor(page_row[:npages].astype(np.int64), device=pool.device)
    pages = pool.index_select(0, idx)                    # [np][KVH][pt][D]
    tm = pages.permute(0, 2, 1, 3).reshape(npages * page_tokens, pool.shape[1], pool.shape[3])
    return tm[:tokens].contiguous()
