"""Paged KV block manager with data-parallel, fused-pipeline and extend pages.

Parity: ``kunserve/block_manager.py:76-1087`` (``BlockManager``).  Same
capabilities — base pages, fused-pipeline (fusion) page ids, extend pages from
dropped parameters, stale-request pages that become fusion pages, CPU swap,
packing extend pages back into the base region before a restore — on a
different bookkeeping model:

* every physical page ``b`` carries a bitmask of its ``N`` occupied slices
  (``N`` = fusion size, 1 when unfused).  A page is either *whole* (owned by
  one request in the unfused layout, all slices used), *sliced* (some slices
  owned by pipeline requests), or *free*;
* a request's table is homogeneous: whole page ids (``b < P``) or fusion /
  extend ids (see ``layout.py``);
* free pages and pages with free slices live in sorted sets, so allocation is
  O(k log P) instead of list slicing, and allocation picks slices from
  partly-used pages first so that whole pages stay available for
  data-parallel requests while a group is restoring.

All allocations are all-or-nothing: ``NoFreeBlocksError`` leaves the manager
unchanged.  ``check_invariants`` recounts everything from the tables and is
called by the tests after every transition.
"""
import asyncio
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

from sortedcontainers import SortedSet

from ..request import BatchedRequests, Request
from ..utils.logger import init_logger
from ..utils.misc import cdiv

logger = init_logger(__name__)

WHOLE = "whole"
SLICE = "slice"


class NoFreeBlocksError(RuntimeError):
    pass


class BlockLocation:
    GPU = "gpu"
    CPU = "cpu"


class BlockManager:
    def __init__(self, num_gpu_blocks: int, num_cpu_blocks: int = 0, block_size: int = 16,
                 rank: int = 0, reserved_blocks_ratio: float = 0.0):
        self.P = int(num_gpu_blocks)
        self.block_size = int(block_size)
        self.rank = rank
        self.max_num_cpu_blocks = int(num_cpu_blocks)
        self.reserved_blocks_ratio = reserved_blocks_ratio

        self.fusion_size = 1
        self.is_fusion_state = False
        self._mask: List[int] = [0] * self.P
        self._whole_pages = set()
        self._free_pages = SortedSet(range(self.P))
        self._partial = SortedSet()            # sliced pages that still have a free slice

        self._ext_ids = SortedSet()            # free extend ids
        self._ext_capacity = 0                 # extend pages currently part of the pool
        self._ext_next = 0                     # next unused extend index
        self._ext_reclaiming = False

        self._free_cpu = SortedSet(range(self.max_num_cpu_blocks))
        self.block_table: Dict[int, List[int]] = {}
        self.request_location: Dict[int, str] = {}
        self._kind: Dict[int, str] = {}

    # ------------------------------------------------------------------ sizes
    @property
    def full_mask(self) -> int:
        return (1 << self.fusion_size) - 1

    @property
    def num_base_gpu_blocks(self) -> int:
        """``N*P``: the first extend id (reference name)."""
        return self.fusion_size * self.P

    @property
    def num_extend_gpu_blocks(self) -> int:
        return self._ext_capacity

    @property
    def max_num_pages(self) -> int:
        """Extent of the page-id space the engine must address."""
        return self.fusion_size * self.P + self._ext_next

    def get_num_blocks_needed(self, request: Request) -> int:
        return cdiv(request.get_num_tokens(), self.block_size)

    def _missing(self, request: Request, extra: int = 0) -> int:
        have = len(self.block_table.get(request.request_id, ()))
        return max(0, self.get_num_blocks_needed(request) + extra - have)

    def num_free_whole(self) -> int:
        return len(self._free_pages)

    def num_free_slices(self) -> int:
        n = self.fusion_size
        part = sum(n - bin(self._mask[b]).count("1") for b in self._partial)
        return part + n * len(self._free_pages)

    def num_free_extend(self) -> int:
        return 0 if self._ext_reclaiming else len(self._ext_ids)

    def get_num_avail_gpu_blocks(self) -> int:
        """Free pages in the unit a new request of the current state uses."""
        if self.is_fusion_state:
            return self.num_free_slices() + self.num_free_extend()
        return self.num_free_whole()

    # page-equivalents (1 whole page == N slices == N extend pages)
    def capacity_pages(self) -> float:
        return self.P + self._ext_capacity / self.fusion_size

    def used_pages(self) -> float:
        n = self.fusion_size
        used_slices = sum(bin(self._mask[b]).count("1") for b in range(self.P)
                          if b not in self._whole_pages)
        used_ext = self._ext_capacity - len(self._ext_ids)
        return len(self._whole_pages) + (used_slices + used_ext) / n

    def free_pages(self) -> float:
        return self.capacity_pages() - self.used_pages()

    # ----------------------------------------------------------- primitives
    def _take_whole(self, k: int) -> List[int]:
        if len(self._free_pages) < k:
            raise NoFreeBlocksError(f"need {k} whole pages, {len(self._free_pages)} free")
        out = [self._free_pages.pop(0) for _ in range(k)]
        for b in out:
            self._mask[b] = self.full_mask
            self._whole_pages.add(b)
        return out

    def _take_slices(self, k: int, allow_extend: bool = True) -> List[int]:
        n, p = self.fusion_size, self.P
        avail = self.num_free_slices() + (self.num_free_extend() if allow_extend else 0)
        if avail < k:
            raise NoFreeBlocksError(f"need {k} slices, {avail} free")
        out: List[int] = []
        while len(out) < k and (self._partial or self._free_pages):
            if self._partial:
                b = self._partial[0]
            else:
                b = self._free_pages.pop(0)
            m = self._mask[b]
            for s in range(n):
                if len(out) == k:
                    break
                if not (m >> s) & 1:
                    m |= 1 << s
                    out.append(s * p + b)
            self._mask[b] = m
            if m == self.full_mask:
                self._partial.discard(b)
            else:
                self._partial.add(b)
        while len(out) < k:
            out.append(self._ext_ids.pop(0))
        return out

    def _release_whole(self, b: int) -> None:
        assert b in self._whole_pages, f"page {b} is not a whole page"
        self._whole_pages.discard(b)
        self._mask[b] = 0
        self._free_pages.add(b)

    def _release_id(self, f: int) -> None:
        n, p = self.fusion_size, self.P
        if f >= n * p:
            if self._ext_reclaiming:
                self._ext_capacity -= 1       # extend page leaves the pool
            else:
                self._ext_ids.add(f)
            return
        s, b = divmod(f, p)
        assert (self._mask[b] >> s) & 1 and b not in self._whole_pages, f"slice {f} not allocated"
        self._mask[b] &= ~(1 << s)
        if self._mask[b] == 0:
            self._partial.discard(b)
            self._free_pages.add(b)
        else:
            self._partial.add(b)

    # ------------------------------------------------------------ allocation
    def is_allocated(self, request_id: int) -> bool:
        return request_id in self.block_table

    def get_location(self, request_id: int) -> Optional[str]:
        return self.request_location.get(request_id)

    def _kind_for(self, request: Request, only_new_blocks: bool) -> str:
        if only_new_blocks or request.fusion_exec:
            return SLICE
        return WHOLE

    def can_allocate(self, request: Request, only_new_blocks: bool = False) -> bool:
        k = self._missing(request)
        kind = self._kind.get(request.request_id) or self._kind_for(request, only_new_blocks)
        if kind == WHOLE:
            return self.num_free_whole() >= k
        return self.num_free_slices() + self.num_free_extend() >= k

    def allocate_blocks(self, request: Request, only_new_blocks: bool = False,
                        live_reshard: bool = False) -> List[int]:
        """Grow ``request``'s table to cover ``get_num_tokens()`` (+1 page with
        ``live_reshard``).  Returns the newly added ids."""
        rid = request.request_id
        if self.request_location.get(rid, BlockLocation.GPU) != BlockLocation.GPU:
            raise AssertionError(f"request {rid} is on CPU; swap it in first")
        k = self._missing(request, 1 if live_reshard else 0)
        kind = self._kind.get(rid) or self._kind_for(request, only_new_blocks)
        if k == 0:
            return []
        new = self._take_whole(k) if kind == WHOLE else self._take_slices(k)
        self.block_table.setdefault(rid, []).extend(new)
        self.request_location[rid] = BlockLocation.GPU
        self._kind[rid] = kind
        return new

    def allocate_blocks_batched(self, batch: BatchedRequests) -> None:
        for r in batch.requests:
            self.allocate_blocks(r)

    def check_blocks(self, request: Request) -> int:
        return self._missing(request)

    def check_blocks_batched(self, batch: BatchedRequests) -> int:
        return sum(self._missing(r) for r in batch.requests)

    def free_blocks(self, request: Request, only_new_blocks: bool = False) -> None:
        self.free_request(request.request_id)

    def free_request(self, rid: int) -> None:
        if rid not in self.block_table:
            raise AssertionError(f"request {rid} not allocated")
        ids = self.block_table.pop(rid)
        loc = self.request_location.pop(rid)
        kind = self._kind.pop(rid)
        if loc == BlockLocation.CPU:
            self._free_cpu.update(ids)
            return
        for f in ids:
            if kind == WHOLE:
                self._release_whole(f)
            else:
                self._release_id(f)

    def free_blocks_batched(self, requests: Iterable[Request]) -> None:
        for r in requests:
            self.free_blocks(r)

    def get_free_gpu_blocks(self, k: int) -> List[int]:
        """Take ``k`` whole pages that are not yet attached to a request (live
        restore builds a new table out of them); ``[]`` if not enough."""
        try:
            return self._take_whole(k)
        except NoFreeBlocksError:
            return []

    def attach_blocks(self, request_id: int, ids: List[int], kind: str = WHOLE) -> None:
        """Give pages returned by ``get_free_gpu_blocks`` to a request."""
        assert request_id not in self.block_table
        self.block_table[request_id] = list(ids)
        self.request_location[request_id] = BlockLocation.GPU
        self._kind[request_id] = kind

    def release_unattached(self, ids: Sequence[int]) -> None:
        for b in ids:
            self._release_whole(b)

    # ------------------------------------------------------------ tables
    def get_single_block_table(self, request_id: int) -> List[int]:
        if request_id not in self.block_table:
            raise AssertionError(f"request {request_id} not allocated")
        return self.block_table[request_id]

    def get_partial_block_table(self, request_ids: Sequence[int]) -> List[List[int]]:
        return [self.block_table.get(rid, []) for rid in request_ids]

    def get_block_table(self, requests: Sequence[Request]) -> List[List[int]]:
        out = []
        for r in requests:
            ids = self.block_table.get(r.request_id, [])
            if r.is_context_stage():
                ids = ids[:cdiv(r.prefill_end_index, self.block_size)]
            out.append(ids)
        return out

    def get_allocated_num_blocks(self, request_id: int) -> int:
        return len(self.block_table.get(request_id, ()))

    # --------------------------------------------------------- fusion state
    def convert_to_pipeline_format(self, num_pipeline_stages: int) -> None:
        """Enter the fused state with ``N`` instances (INITIAL→BALLOON and
        RESTORE→BALLOON; ``convert_to_pipeline_format_w_reserve`` is the same
        operation in this model).  Whole pages of running requests stay whole
        until they are resharded or recomputed."""
        n = int(num_pipeline_stages)
        if n < 1 or n > 30:
            raise ValueError(f"bad fusion size {n}")
        if self.fusion_size not in (1, n):
            raise AssertionError(f"already fused with N={self.fusion_size}")
        if self.fusion_size == 1 and n > 1:
            if self._ext_next:
                raise AssertionError("extend pages left from a previous balloon")
            self.fusion_size = n
            full = self.full_mask
            for b in self._whole_pages:
                self._mask[b] = full
        self.is_fusion_state = True

    convert_to_pipeline_format_w_reserve = convert_to_pipeline_format

    def add_ex_fusion_blocks(self, ex_blocks: int) -> List[int]:
        """Pages made from dropped parameter memory (ids from ``N*P`` on)."""
        base = self.fusion_size * self.P
        new = list(range(base + self._ext_next, base + self._ext_next + int(ex_blocks)))
        self._ext_next += int(ex_blocks)
        self._ext_capacity += int(ex_blocks)
        self._ext_ids.update(new)
        self._ext_reclaiming = False
        return new

    def convert_all_reserved_blocks_into_fusion(self) -> None:
        """Kept for API parity: free pages are directly usable as slices here."""

    def free_blocks_into_fusion_except(self, request_id: int, fusion_size: int, fusion_rank: int) -> None:
        """A stale request now keeps only slice ``fusion_rank`` of each of its
        whole pages (where its own layers already are); other slices free."""
        assert fusion_size == self.fusion_size
        assert self._kind.get(request_id) == WHOLE, f"request {request_id} has no whole pages"
        p = self.P
        new_ids = []
        for b in self.block_table[request_id]:
            self._whole_pages.discard(b)
            self._mask[b] = 1 << fusion_rank
            if fusion_size > 1:
                self._partial.add(b)
            new_ids.append(fusion_rank * p + b)
        self.block_table[request_id] = new_ids
        self._kind[request_id] = SLICE

    def free_blocks_into_fusion_except_batched(self, requests: Iterable[Request], fusion_size: int,
                                               fusion_rank: int) -> None:
        for r in requests:
            self.free_blocks_into_fusion_except(r.request_id, fusion_size, fusion_rank)

    def num_used_extend(self) -> int:
        return self._ext_capacity - len(self._ext_ids)

    def start_extend_reclaim(self) -> None:
        """Stop handing out extend pages; free ones leave the pool right away."""
        self._ext_reclaiming = True
        self._ext_capacity -= len(self._ext_ids)
        self._ext_ids.clear()

    def extend_reclaimed(self) -> bool:
        return self._ext_reclaiming and self._ext_capacity == 0

    async def wait_for_ex_blocks_to_return(self, poll_s: float = 0.0) -> None:
        self.start_extend_reclaim()
        while self._ext_capacity > 0:
            await asyncio.sleep(poll_s)
        self._ext_next = 0

    def pack_blocks_into_base_region(self, requests: Iterable[Request]) -> List[Tuple[int, int]]:
        """Move extend pages of ``requests`` into free base slices.  Returns the
        ``(src_id, dst_id)`` copies the engine must perform before the next
        step touches these requests."""
        moves: List[Tuple[int, int]] = []
        base = self.fusion_size * self.P
        for r in requests:
            ids = self.block_table.get(r.request_id)
            if not ids or self._kind.get(r.request_id) != SLICE:
                continue
            ext_pos = [i for i, f in enumerate(ids) if f >= base]
            if not ext_pos:
                continue
            if self.num_free_slices() < len(ext_pos):
                break
            dst = self._take_slices(len(ext_pos), allow_extend=False)
            for i, d in zip(ext_pos, dst):
                moves.append((ids[i], d))
                self._release_id(ids[i])
                ids[i] = d
        return moves

    def restore_kvblocks(self) -> None:
        """Leave the fused state (parameters are back).  Pipeline requests keep
        their slices; new unfused requests take whole free pages."""
        if self._ext_capacity:
            raise AssertionError("extend pages must be reclaimed before restore")
        self._ext_next = 0
        self._ext_reclaiming = False
        self.is_fusion_state = False

    def num_slice_requests(self) -> int:
        return sum(1 for k in self._kind.values() if k == SLICE)

    def restore_from_fusion(self) -> None:
        """Back to ``N = 1`` once no request holds slices."""
        if self.num_slice_requests():
            raise AssertionError("pipeline requests still hold slices")
        assert not self._partial
        self.fusion_size = 1
        self.is_fusion_state = False
        for b in self._whole_pages:
            self._mask[b] = 1

    # ----------------------------------------------------------------- swap
    def get_num_avail_cpu_blocks(self) -> int:
        return len(self._free_cpu)

    def swap_out_requests(self, requests: Sequence[Request]) -> Optional[List[Tuple[int, int]]]:
        """Move whole-page requests to CPU pages; returns ``(gpu, cpu)`` copies
        or ``None`` if the CPU pool is too small (nothing changes then)."""
        need = sum(len(self.block_table[r.request_id]) for r in requests)
        if need > len(self._free_cpu) or any(self._kind[r.request_id] != WHOLE for r in requests):
            return None
        pairs = []
        for r in requests:
            rid = r.request_id
            gpu_ids = self.block_table[rid]
            cpu_ids = [self._free_cpu.pop(0) for _ in gpu_ids]
            pairs.extend(zip(gpu_ids, cpu_ids))
            for b in gpu_ids:
                self._release_whole(b)
            self.block_table[rid] = cpu_ids
            self.request_location[rid] = BlockLocation.CPU
        return pairs

    def swap_in_requests(self, requests: Sequence[Request]) -> Optional[List[Tuple[int, int]]]:
        need = sum(len(self.block_table[r.request_id]) for r in requests)
        if need > self.num_free_whole():
            return None
        pairs = []
        for r in requests:
            rid = r.request_id
            cpu_ids = self.block_table[rid]
            gpu_ids = self._take_whole(len(cpu_ids))
            pairs.extend(zip(cpu_ids, gpu_ids))
            self._free_cpu.update(cpu_ids)
            self.block_table[rid] = gpu_ids
            self.request_location[rid] = BlockLocation.GPU
        return pairs

    def swap_out_one_request(self, request: Request):
        return self.swap_out_requests([request])

    def swap_in_one_request(self, request: Request):
        return self.swap_in_requests([request])

    # ----------------------------------------------------------- invariants
    def check_invariants(self) -> None:
        n, p = self.fusion_size, self.P
        mask = [0] * p
        whole = set()
        ext_used = set()
        cpu_used = set()
        for rid, ids in self.block_table.items():
            kind, loc = self._kind[rid], self.request_location[rid]
            if loc == BlockLocation.CPU:
                for c in ids:
                    assert c not in cpu_used
                    cpu_used.add(c)
                continue
            for f in ids:
                if kind == WHOLE:
                    assert 0 <= f < p and f not in whole and mask[f] == 0, (rid, f)
                    whole.add(f)
                    mask[f] = self.full_mask
                elif f >= n * p:
                    assert f not in ext_used and f not in self._ext_ids, (rid, f)
                    ext_used.add(f)
                else:
                    s, b = divmod(f, p)
                    assert b not in whole and not (mask[b] >> s) & 1, (rid, f)
                    mask[b] |= 1 << s
        assert whole == self._whole_pages, "whole-page set drifted"
        for b in range(p):
            assert mask[b] == self._mask[b], f"mask of page {b} drifted"
            if mask[b] == 0:
                assert b in self._free_pages and b not in self._partial
            else:
                assert b not in self._free_pages
                assert (b in self._partial) == (b not in whole and mask[b] != self.full_mask), b
        assert len(ext_used) + len(self._ext_ids) == self._ext_capacity, "extend count drifted"
        assert not (cpu_used & set(self._free_cpu))
        assert len(cpu_used) + len(self._free_cpu) == self.max_num_cpu_blocks

    def __repr__(self) -> str:
        return (f"BlockManager(P={self.P}, N={self.fusion_size}, fused={self.is_fusion_state}, "
                f"free_whole={self.num_free_whole()}, free_slices={self.num_free_slices()}, "
                f"ext={self.num_free_extend()}/{self._ext_capacity})")
