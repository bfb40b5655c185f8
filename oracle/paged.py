"""CPU model of paged latent caches (TEST INFRASTRUCTURE ONLY).

The reference plans a paged variant of its decode op but has not built it (HANDOFF.md:54-55, 126-127;
palu_tt/attention.py:86 and :586 assert a non-paged cache). Its plan names the stock paged flash-decode
op of tt-metal (``paged_scaled_dot_product_attention_decode`` with ``page_table_tensor``, and
``paged_update_cache`` with ``page_table``; tt-metal is imported by the reference but not vendored) as the
template, so the layout restated here is that op's published convention:

* a cache is [n_blocks, heads, block_size, width]: fixed-size blocks of positions;
* a page table [B, blocks per row] maps row b's logical block j (positions j*block_size ..
  (j+1)*block_size - 1) to a physical block.

A paged decode is then the unpaged decode (``reference_decode``, fused.py:82-107) over each row's
gathered positions, which is how the tests check the CUDA path. There are no reference golden vectors for
paging (nothing of the reference implements it): what is pinned is the decode math, through the unpaged
golden vectors; the gather / scatter below are checked against each other and against the unpaged
append on the CPU.
"""
from __future__ import annotations

import torch


def paged_gather(cache: torch.Tensor, page_table: torch.Tensor, n_pos: int) -> torch.Tensor:
    """Paged cache [n_blocks, G, bs, r] -> contiguous [B, G, n_pos, r]: position t of row b is row t % bs of
    block page_table[b, t // bs]. Positions whose table entry lies outside [0, n_blocks) read as zeros (the
    library's behaviour for an unmapped block)."""
    n_blocks, G, bs, r = cache.shape
    B = page_table.shape[0]
    out = torch.zeros(B, G, n_pos, r, dtype=cache.dtype)
    for b in range(B):
        for j in range((n_pos + bs - 1) // bs):
            e = int(page_table[b, j])
            lo, hi = j * bs, min(n_pos, (j + 1) * bs)
            if 0 <= e < n_blocks:
                out[b, :, lo:hi] = cache[e, :, :hi - lo]
    return out


def paged_scatter(contig: torch.Tensor, page_table: torch.Tensor, n_blocks: int, block_size: int) -> torch.Tensor:
    """Contiguous [B, G, S, r] -> paged [n_blocks, G, block_size, r] laid out by ``page_table`` (blocks no
    row maps stay zero). The inverse of ``paged_gather`` over the mapped positions."""
    B, G, S, r = contig.shape
    cache = torch.zeros(n_blocks, G, block_size, r, dtype=contig.dtype)
    for b in range(B):
        for j in range((S + block_size - 1) // block_size):
            e = int(page_table[b, j])
            lo, hi = j * block_size, min(S, (j + 1) * block_size)
            if 0 <= e < n_blocks:
                cache[e, :, :hi - lo] = contig[b, :, lo:hi]
    return cache


def paged_append(cache: torch.Tensor, new: torch.Tensor, cur_pos: torch.Tensor, page_table: torch.Tensor,
                 max_seq: int) -> None:
    """paged_update_cache with a page table (attention.py:622-623, paged): row b's latents new[b]
    [G, r] go to row cur_pos[b] % bs of block page_table[b, cur_pos[b] // bs]; rows with cur_pos outside
    [0, max_seq) and entries outside [0, n_blocks) write nothing."""
    n_blocks, _, bs, _ = cache.shape
    for b in range(new.shape[0]):
        p = int(cur_pos[b])
        if not 0 <= p < max_seq:
            continue
        e = int(page_table[b, p // bs])
        if 0 <= e < n_blocks:
            cache[e, :, p % bs] = new[b]


def shuffled_page_table(batch: int, blocks_per_row: int, n_blocks: int, generator: torch.Generator) -> torch.Tensor:
    """A page table that gives every row its own blocks, drawn as a random permutation of the physical
    blocks (so consecutive logical blocks are scattered): [batch, blocks_per_row] int32."""
    if batch * blocks_per_row > n_blocks:
        raise ValueError(f"{batch} rows x {blocks_per_row} blocks exceed the {n_blocks} physical blocks")
    perm = torch.randperm(n_blocks, generator=generator)[:batch * blocks_per_row]
    return perm.view(batch, blocks_per_row).to(torch.int32)
