"""Paged-cache gathers and selected-token materialisation on CUDA.

Same functions and semantics as the reference
(src/vllm_ascend_kvcompress/methods/triattention/cache.py:9-111): caches are
``[blocks, block_size, heads, dim]`` with contiguous inner dims and any block
stride (K and V may interleave in one padded buffer).  Row copies run in the
``kvc_gather_slots`` / ``kvc_scatter_slots`` kernels; materialisation gathers
every kept row into a workspace before writing, so overlapping source and
destination blocks are safe.  The batched method path uses ``kvc_compact``
instead, which copies source rows straight into private destinations.
"""

from __future__ import annotations

import torch

from . import kernels as K


def token_slots(block_ids: torch.Tensor, token_indices: torch.Tensor, block_size: int) -> torch.Tensor:
    """Logical token index -> flat physical slot ``block_ids[i // bs] * bs + i % bs``."""
    blocks = torch.div(token_indices, block_size, rounding_mode="floor")
    return block_ids.index_select(0, blocks) * block_size + torch.remainder(token_indices, block_size)


def gather_paged_tokens(cache: torch.Tensor, block_ids: torch.Tensor, token_indices: torch.Tensor,
                        block_size: int) -> torch.Tensor:
    if cache.ndim != 4 or cache.shape[1] != block_size:
        raise ValueError("cache must use [blocks, block, heads, dim] layout")
    slots = token_slots(block_ids.to(torch.int64), token_indices.to(torch.int64), block_size).contiguous()
    return K.gather_slots(cache, slots)


def gather_paged_range(cache: torch.Tensor, block_ids: torch.Tensor, *, start: int, count: int,
                       block_size: int) -> torch.Tensor:
    idx = torch.arange(start, start + count, device=block_ids.device, dtype=torch.long)
    return gather_paged_tokens(cache, block_ids, idx, block_size)


def materialize_token_slots(k_cache: torch.Tensor, v_cache: torch.Tensor, source_slots: torch.Tensor,
                            destination_slots: torch.Tensor, k_workspace: torch.Tensor,
                            v_workspace: torch.Tensor) -> None:
    """Move rows ``source_slots -> destination_slots`` through persistent workspaces."""
    src = source_slots.to(torch.int64).contiguous()
    dst = destination_slots.to(torch.int64).contiguous()
    K.gather_slots(k_cache, src, out=k_workspace)
    K.gather_slots(v_cache, src, out=v_workspace)
    K.scatter_slots(k_cache, dst, k_workspace)
    K.scatter_slots(v_cache, dst, v_workspace)


def materialize_selected_tokens(k_cache: torch.Tensor, v_cache: torch.Tensor, source_block_ids: torch.Tensor,
                                destination_block_ids: torch.Tensor, keep_indices: torch.Tensor,
                                block_size: int) -> None:
    """Write the kept tokens densely into the destination blocks (gather first)."""
    src = token_slots(source_block_ids.to(torch.int64), keep_indices.to(torch.int64), block_size).contiguous()
    dense = torch.arange(keep_indices.shape[0], device=keep_indices.device, dtype=torch.long)
    dst = token_slots(destination_block_ids.to(torch.int64), dense, block_size).contiguous()
    gk = K.gather_slots(k_cache, src)
    gv = K.gather_slots(v_cache, src)
    K.scatter_slots(k_cache, dst, gk)
    K.scatter_slots(v_cache, dst, gv)
