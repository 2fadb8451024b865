"""Output-column (N) split of large-M products across GPUs with one exchange.

The reference is single-process (no collective anywhere).  The partitioning
here follows where the work shards:

* decode requests are independent -> data-parallel replicas, no collective
  (bench.py under torchrun);
* a large-M prefill GEMM or the LM head splits by output column: rank r owns
  weight rows [r*N/G, (r+1)*N/G) (with their per-row scales), computes its
  slice of C with the unchanged kernel -- so every column is bit-identical to
  the single-GPU result -- and one NCCL all-gather over NVLink assembles C
  (M*N/G*4 bytes sent per rank);
* for greedy decoding the LM-head exchange shrinks to one (value, index)
  pair per request and rank (8 bytes), merged with the reference's
  tie-break: larger value wins, equal values -> smaller index
  (tokenizer/src/utils.cpp:34-44).

Everything here is host orchestration over torch.distributed; the products
run through the C ABI.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_rows(n: int, world: int, rank: int):
    """[start, stop) of the rows rank `rank` owns (balanced, contiguous)."""
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def gather_columns(local: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """All-gather the column slices [M, n_r] of every rank into C [M, n_total]."""
    world = dist.get_world_size(group)
    M = local.shape[0]
    sizes = [shard_rows(n_total, world, r) for r in range(world)]
    width = max(b - a for a, b in sizes)
    buf = torch.zeros((M, width), dtype=local.dtype, device=local.device)
    buf[:, :local.shape[1]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf.contiguous(), group=group)
    return torch.cat([p[:, :b - a] for p, (a, b) in zip(parts, sizes)], dim=1)


def merge_argmax(values: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """values/indices [world, rows]: per-rank maxima of their column slices
    (indices already global, -1 for "no candidate").  Returns the global
    greedy index per row: max value, ties -> smallest index; a row with no
    candidate gives 0 (the reference's start value)."""
    valid = indices >= 0
    v = torch.where(valid, values, torch.full_like(values, float("-inf")))
    best = v.max(dim=0).values
    is_best = valid & (v == best.unsqueeze(0))
    big = torch.iinfo(indices.dtype).max
    idx = torch.where(is_best, indices, torch.full_like(indices, big)).min(dim=0).values
    return torch.where(idx == big, torch.zeros_like(idx), idx)


def local_argmax(logits_slice: torch.Tensor, start: int):
    """(value, global index) of each row's first maximum over its slice; rows
    whose slice has no value > -FLT_MAX report index -1 (reference start
    value -FLT_MAX with a strict comparison, NaN never wins)."""
    finfo = torch.finfo(torch.float32)
    x = torch.where(torch.isnan(logits_slice), torch.full_like(logits_slice, float("-inf")), logits_slice)
    v, i = x.max(dim=1)                    # torch returns the first maximal index
    i = i.to(torch.int64) + start
    i = torch.where(v > -finfo.max, i, torch.full_like(i, -1))
    return v, i


def split_linear_gather(x, w_local, s_local, n_total: int, linear_fn, group=None):
    """C = x . dequant(W)^T for W split by rows across the group: each rank
    applies `linear_fn(x, w_local, s_local)` (the C-ABI product) to its shard
    and the slices are all-gathered into [M, n_total]."""
    return gather_columns(linear_fn(x, w_local, s_local), n_total, group)


def split_greedy(logits_local: torch.Tensor, start: int, group=None) -> torch.Tensor:
    """Greedy token per row from column-split logits with an 8-byte-per-row
    exchange: all-gather of per-rank (value, index) pairs, then merge."""
    world = dist.get_world_size(group)
    v, i = local_argmax(logits_local.float(), start)
    vs = [torch.empty_like(v) for _ in range(world)]
    is_ = [torch.empty_like(i) for _ in range(world)]
    dist.all_gather(vs, v.contiguous(), group=group)
    dist.all_gather(is_, i.contiguous(), group=group)
    return merge_argmax(torch.stack(vs), torch.stack(is_))
