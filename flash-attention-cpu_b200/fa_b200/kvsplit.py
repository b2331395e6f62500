"""Key-range split of one long attention slice across GPUs (one process per GPU).

For a single (batch, head) slice too long for one GPU to finish quickly
(config 5: 1 x 131072 x 128, causal), every rank holds all query rows and a
share of the keys:

1. The key range is cut into 2*G equal chunks; rank g takes chunks g and
   2G-1-g ("zig-zag"), which gives every rank the same causal work (early
   chunks are seen by many rows, late chunks by few).
2. Each rank computes a partial (O_c, lse_c) for each of its chunks with
   ``fa_forward_partial_device`` (range-normalised output and the row LSE over
   those keys; -inf / zeros for rows that see none of them) and merges its two
   partials with ``fa_lse_combine_device``.
3. One all-to-all (NCCL) sends row block s of every rank's partial to rank s,
   which merges the G partials of its rows with ``fa_lse_combine_device``:
   lse = log(sum_r exp(lse_r)),  O = sum_r exp(lse_r - lse) * O_r.

Rank s ends up owning output rows [s*R/G, (s+1)*R/G).  The only collective is
that single exchange of (O, lse) partials, (G-1)/G of ~R*(d+1)*4 bytes per rank.

The compute steps are passed in as functions so the host logic (chunking, the
exchange layout, the merge) is testable on CPU ranks with a CPU stand-in; the
defaults are this library's GPU kernels and there is no CPU path in them.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Chunk:
    start: int  # first key (global position)
    stop: int   # one past the last key


def zigzag_chunks(seq_len_k: int, world: int, rank: int) -> list[Chunk]:
    """The two key chunks of `rank` out of 2*world equal (last one ragged) chunks."""
    n = 2 * world
    size = -(-seq_len_k // n)
    out = []
    for c in (rank, n - 1 - rank):
        a, b = min(c * size, seq_len_k), min((c + 1) * size, seq_len_k)
        out.append(Chunk(a, b))
    return out


def row_blocks(rows: int, world: int) -> list[tuple[int, int]]:
    """Equal row blocks owned by each rank after the exchange (rows % world == 0)."""
    if rows % world:
        raise ValueError("the number of query rows must be a multiple of the world size")
    b = rows // world
    return [(i * b, (i + 1) * b) for i in range(world)]


def _gpu_partial(q, k, v, out, lse, causal, q_offset, k_offset):
    import fa_b200
    fa_b200.forward_partial_device(q, k, v, out, lse, causal, q_offset, k_offset)


def _gpu_combine(o_parts, lse_parts, out, lse_out):
    import fa_b200
    fa_b200.lse_combine_device(o_parts, lse_parts, out, lse_out)


def kv_split_forward(q, k_full, v_full, causal, group=None, partial_fn=None, combine_fn=None,
                     k_chunks=None, v_chunks=None):
    """Attention of one slice with the keys split across the ranks of `group`.

    q: [1, R, d] (every rank holds all rows); k_full / v_full: [1, S, d] on this
    rank, or pass only this rank's two chunks as ``k_chunks`` / ``v_chunks``
    (lists of [1, len, d] tensors in zigzag_chunks order; k_full / v_full then
    only give the shape).  Returns (out_rows, lse_rows, (row_start, row_stop)):
    this rank's block of the result.
    """
    import torch
    import torch.distributed as dist

    partial_fn = partial_fn or _gpu_partial
    combine_fn = combine_fn or _gpu_combine
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    _, rows, d = q.shape
    seq_k = k_full.shape[1]
    dev = q.device
    chunks = zigzag_chunks(seq_k, world, rank)
    o_parts = torch.zeros(2, rows, d, device=dev, dtype=torch.float32)
    l_parts = torch.full((2, rows), float("-inf"), device=dev, dtype=torch.float32)
    for i, c in enumerate(chunks):
        if c.stop <= c.start:
            continue
        kc = k_chunks[i] if k_chunks is not None else k_full[:, c.start:c.stop].contiguous()
        vc = v_chunks[i] if v_chunks is not None else v_full[:, c.start:c.stop].contiguous()
        partial_fn(q, kc, vc, o_parts[i].view(1, rows, d), l_parts[i].view(1, rows), causal,
                   0, c.start)
    o_local = torch.empty(rows, d, device=dev, dtype=torch.float32)
    l_local = torch.empty(rows, device=dev, dtype=torch.float32)
    combine_fn(o_parts, l_parts, o_local, l_local)
    # exchange: row block s of every rank -> rank s
    blocks = row_blocks(rows, world)
    rb = rows // world
    o_recv = torch.empty(world * rb, d, device=dev, dtype=torch.float32)
    l_recv = torch.empty(world * rb, device=dev, dtype=torch.float32)
    dist.all_to_all_single(o_recv, o_local, group=group)
    dist.all_to_all_single(l_recv, l_local, group=group)
    out = torch.empty(rb, d, device=dev, dtype=torch.float32)
    lse = torch.empty(rb, device=dev, dtype=torch.float32)
    combine_fn(o_recv.view(world, rb, d), l_recv.view(world, rb), out, lse)
    return out, lse, blocks[rank]
