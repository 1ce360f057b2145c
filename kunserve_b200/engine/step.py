"""The argument bundle of one engine step (one forward over a ragged batch).

It carries what the reference's ``LlamaOp.pforward`` receives
(``kunserve/worker.py:270-314``): the batch's input tokens, RoPE start
positions, prefill flags, page tables and the layer slice ``[layer_start,
layer_end)`` to run, plus the page-addressing mode (``fusion_size``) and
per-request sampling parameters.  Tensors are built once per step on the
host and copied to the device in a single pinned transfer by the native
runner.
"""
from dataclasses import dataclass, field
from typing import List, Optional

import torch


@dataclass
class StepInput:
    request_ids: List[int]
    input_tokens: List[List[int]]
    start_positions: List[int]
    page_tables: List[List[int]]
    is_prefill: List[int]
    layer_start: int
    layer_end: int
    fusion_size: int = 1
    temperature: Optional[List[float]] = None
    top_k: Optional[List[int]] = None
    top_p: Optional[List[float]] = None
    seeds: Optional[List[int]] = None
    step_id: int = 0
    # live restore inside the step (the reference pforward's pages_of_pp /
    # pages_of_dp / receiver_rank): (home member, group size, this member,
    # per-member fusion page ids, the home's new whole pages), concatenated
    # over the requests that move home.  After its layers, each member copies
    # its layer slice of those pages into the home member's pool.
    restore: Optional[tuple] = None

    @property
    def num_requests(self) -> int:
        return len(self.request_ids)

    @property
    def num_tokens(self) -> int:
        return sum(len(t) for t in self.input_tokens)

    def query_lens(self) -> List[int]:
        return [len(t) for t in self.input_tokens]

    def context_lens(self) -> List[int]:
        return [s + len(t) for s, t in zip(self.start_positions, self.input_tokens)]

    def is_greedy(self) -> bool:
        return self.temperature is None or all(t <= 1e-5 for t in self.temperature)

    def flat_tokens(self) -> torch.Tensor:
        return torch.tensor([t for ts in self.input_tokens for t in ts], dtype=torch.int32)

    def padded_page_table(self, width: Optional[int] = None) -> torch.Tensor:
        w = width or max([len(p) for p in self.page_tables] + [1])
        out = torch.zeros((len(self.page_tables), w), dtype=torch.int32)
        for i, p in enumerate(self.page_tables):
            if p:
                out[i, :len(p)] = torch.tensor(p, dtype=torch.int32)
        return out
