"""Page-id algebra of the paged KV pool.

One instance owns ``P`` physical pages.  A page holds, for every one of the
``L`` decoder layers the instance stores, the K and V of ``block_size``
tokens: ``[L][K|V][block_size][kv_heads][head_dim]``.

When ``N`` instances fuse into one pipeline (balloon), each instance runs
only ``Ls = L / N`` layers, so one physical page can hold ``N`` *slices* of
``Ls`` layers.  Page ids then mean (``kunserve/block_manager.py:250-252,
276-278, 753-760`` use the same numbering):

* ``f < N*P``  — slice ``s = f // P`` of physical page ``b = f % P``; local
  layer ``l`` of the slice lives at layer slot ``s*Ls + l`` of page ``b``;
* ``f >= N*P`` — extend page ``e = f - N*P``: a small page of ``Ls`` layer
  slots in the memory freed by dropped weights, mapped right after the
  ``P`` base pages in the pool's virtual address range.

With ``N = 1`` (data-parallel) this reduces to "page ``f``, layer ``l``", and
slice ``j`` of a page written in the unfused layout already holds layers
``[j*Ls, (j+1)*Ls)`` — which is why a stale request's own slice needs no copy
when its instance joins a pipeline.

``kv_offset`` below is the byte offset the CUDA kernels compute in-line;
the Python copy is the oracle the tests compare against.
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class KVLayout:
    num_pages: int          # P, physical base pages
    num_layers: int         # L, layer slots per physical page
    block_size: int
    num_kv_heads: int
    head_dim: int
    elem_bytes: int = 2

    @property
    def layer_stride(self) -> int:
        """Bytes of one (page, layer) slot: K then V."""
        return 2 * self.block_size * self.num_kv_heads * self.head_dim * self.elem_bytes

    @property
    def page_stride(self) -> int:
        return self.num_layers * self.layer_stride

    @property
    def base_bytes(self) -> int:
        return self.num_pages * self.page_stride

    def slice_layers(self, fusion_size: int) -> int:
        assert self.num_layers % fusion_size == 0, (self.num_layers, fusion_size)
        return self.num_layers // fusion_size

    def extend_page_bytes(self, fusion_size: int) -> int:
        return self.slice_layers(fusion_size) * self.layer_stride

    def kv_offset(self, page_id: int, local_layer: int, fusion_size: int = 1,
                  is_value: bool = False) -> int:
        """Byte offset of the K (or V) block of ``(page_id, local_layer)``."""
        n, p = fusion_size, self.num_pages
        ls = self.slice_layers(n)
        assert 0 <= local_layer < ls
        if page_id < n * p:
            off = (page_id % p) * self.page_stride + ((page_id // p) * ls + local_layer) * self.layer_stride
        else:
            e = page_id - n * p
            off = self.base_bytes + e * ls * self.layer_stride + local_layer * self.layer_stride
        if is_value:
            off += self.layer_stride // 2
        return off


def fusion_id(slice_idx: int, phys_page: int, num_pages: int) -> int:
    return slice_idx * num_pages + phys_page


def split_fusion_id(f: int, num_pages: int):
    """(slice, physical page) of a fusion id below ``N*P``."""
    return f // num_pages, f % num_pages
