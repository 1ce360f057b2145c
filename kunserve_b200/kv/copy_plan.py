"""Copy plans: every KV movement of the framework as equal-size byte chunks.

A layer slice of one page is contiguous in the pool (``Ls`` consecutive
layer slots), so balloon-time reshard, live restore, extend→base packing and
cross-instance block transfer all reduce to "copy chunk ``src_off[i]`` of pool
A to ``dst_off[i]`` of pool B", with one chunk size per plan.  The copy kernel
(``csrc/kernels/copy.cu``) and the torch fallback both execute such plans.
"""
from typing import List, Sequence, Tuple

from .layout import KVLayout


def slice_offset(layout: KVLayout, page_id: int, fusion_size: int) -> int:
    """Byte offset of the first layer slot of ``page_id`` under fusion size ``N``."""
    return layout.kv_offset(page_id, 0, fusion_size)


def whole_page_slice_offset(layout: KVLayout, page: int, slice_idx: int, fusion_size: int) -> int:
    """Offset of layer slice ``slice_idx`` of an unfused (whole) page."""
    return layout.kv_offset(slice_idx * layout.num_pages + page, 0, fusion_size)


def chunk_bytes(layout: KVLayout, fusion_size: int) -> int:
    return layout.slice_layers(fusion_size) * layout.layer_stride


def reshard_plan(layout: KVLayout, fusion_size: int, my_rank: int,
                 pages_of_instances: Sequence[Sequence[int]]) -> Tuple[dict, dict]:
    """Balloon-time KV exchange (``kv_exchange`` contract, reference
    ``kunserve/flash_backend.py:858-895``).

    ``pages_of_instances[my_rank]`` are my stale requests' whole pages;
    ``pages_of_instances[j]`` (j != me) are the fusion ids I allocated for
    peer ``j``'s stale pages, in the same order as ``j``'s own list.

    Returns ``(sends, recvs)``: ``sends[k]`` = source offsets of slice ``k``
    of each of my pages (to peer ``k``); ``recvs[j]`` = destination offsets
    for the chunks peer ``j`` sends me.
    """
    sends, recvs = {}, {}
    mine = pages_of_instances[my_rank]
    for k in range(fusion_size):
        if k == my_rank:
            continue
        sends[k] = [whole_page_slice_offset(layout, b, k, fusion_size) for b in mine]
        recvs[k] = [slice_offset(layout, f, fusion_size) for f in pages_of_instances[k]]
    return sends, recvs


def restore_plan(layout: KVLayout, fusion_size: int, src_rank: int,
                 fusion_pages: Sequence[int], dp_pages: Sequence[int]) -> Tuple[List[int], List[int]]:
    """Live restore: slice ``src_rank`` of a pipeline request (its fusion ids
    on instance ``src_rank``) → layer slots ``[src_rank*Ls, ...)`` of the
    request's new whole pages on its home instance."""
    assert len(fusion_pages) == len(dp_pages)
    src = [slice_offset(layout, f, fusion_size) for f in fusion_pages]
    dst = [whole_page_slice_offset(layout, b, src_rank, fusion_size) for b in dp_pages]
    return src, dst


def local_move_plan(layout: KVLayout, fusion_size: int,
                    moves: Sequence[Tuple[int, int]]) -> Tuple[List[int], List[int]]:
    """Extend→base packing inside one pool (``(src_id, dst_id)`` fusion ids)."""
    return ([slice_offset(layout, s, fusion_size) for s, _ in moves],
            [slice_offset(layout, d, fusion_size) for _, d in moves])
