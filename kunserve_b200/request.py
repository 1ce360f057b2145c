"""Request model: sampling parameters, per-token outputs, requests and batches.

Parity: ``kunserve/request.py`` — ``SamplingParams`` (:17-165),
``TokenOutput``/``RequestOutput`` (:168-207), ``Request`` (:210-501),
``BatchedRequests`` (:504-670), ``create_request`` (:673-707) and
``MigratingRequest`` (:710-735).

Differences by design:

* Sampling parameters reach the device (the reference always decodes
  greedily): the sampling kernel applies temperature, top-k and top-p
  (radix select on the logits, then Gumbel-max over the kept tokens).
* ``start_position()`` is the RoPE position of the first input token of the
  next step (prefill chunk start, or ``len(prompt) + len(generated) - 1`` for
  a decode step).  The reference passes ``input_len + output_len`` for decode
  and leaves the ``-1`` to its native side.
"""
import itertools
import math
import time
from dataclasses import dataclass
from typing import Iterable, List, Optional, Sequence, Tuple, Union


class SamplingParams:
    """OpenAI-completions style sampling parameters.

    ``temperature == 0`` means greedy decoding.  ``top_k == -1`` and
    ``top_p == 1`` disable those filters.
    """

    _EPS = 1e-5

    def __init__(self, n: int = 1, best_of: Optional[int] = None,
                 presence_penalty: float = 0.0, frequency_penalty: float = 0.0,
                 temperature: float = 1.0, top_p: float = 1.0, top_k: int = -1,
                 use_beam_search: bool = False, stop: Union[None, str, List[str]] = None,
                 ignore_eos: bool = False, max_tokens: int = 16,
                 logprobs: Optional[int] = None, stop_token_ids: Optional[List[int]] = None,
                 seed: Optional[int] = None) -> None:
        self.n = n
        self.best_of = n if best_of is None else best_of
        self.presence_penalty = presence_penalty
        self.frequency_penalty = frequency_penalty
        self.temperature = temperature
        self.top_p = top_p
        self.top_k = top_k
        self.use_beam_search = use_beam_search
        self.stop = [] if stop is None else ([stop] if isinstance(stop, str) else list(stop))
        self.stop_token_ids = list(stop_token_ids or [])
        self.ignore_eos = ignore_eos
        self.max_tokens = max_tokens
        self.logprobs = logprobs
        self.seed = seed
        self._verify()

    @property
    def is_greedy(self) -> bool:
        return self.temperature < self._EPS

    def _verify(self) -> None:
        if self.n < 1:
            raise ValueError(f"n must be at least 1, got {self.n}.")
        if self.best_of < self.n:
            raise ValueError(f"best_of ({self.best_of}) must be >= n ({self.n}).")
        for name in ("presence_penalty", "frequency_penalty"):
            v = getattr(self, name)
            if not -2.0 <= v <= 2.0:
                raise ValueError(f"{name} must be in [-2, 2], got {v}.")
        if self.temperature < 0.0:
            raise ValueError(f"temperature must be non-negative, got {self.temperature}.")
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError(f"top_p must be in (0, 1], got {self.top_p}.")
        if self.top_k < -1 or self.top_k == 0:
            raise ValueError(f"top_k must be -1 (disable), or at least 1, got {self.top_k}.")
        if self.max_tokens < 1:
            raise ValueError(f"max_tokens must be at least 1, got {self.max_tokens}.")
        if self.logprobs is not None and self.logprobs < 0:
            raise ValueError(f"logprobs must be non-negative, got {self.logprobs}.")
        if self.use_beam_search:
            if self.best_of == 1:
                raise ValueError("best_of must be > 1 with beam search.")
            if not self.is_greedy or self.top_p < 1.0 - self._EPS or self.top_k != -1:
                raise ValueError("beam search needs temperature 0, top_p 1 and top_k -1.")
        elif self.is_greedy:
            if self.best_of > 1:
                raise ValueError("best_of must be 1 with greedy sampling.")
            if self.top_p < 1.0 - self._EPS or self.top_k != -1:
                raise ValueError("greedy sampling needs top_p 1 and top_k -1.")

    def __repr__(self) -> str:
        return (f"SamplingParams(temperature={self.temperature}, top_p={self.top_p}, "
                f"top_k={self.top_k}, max_tokens={self.max_tokens}, ignore_eos={self.ignore_eos})")


@dataclass
class TokenOutput:
    new_token: str
    new_token_id: int
    new_token_time: float


@dataclass
class ServerInfo:
    """Which front-end server a request's outputs go back to."""

    server_id: int = 0
    queue: object = None


class RequestOutput:
    """What the engine returns for a request (sent once it finishes)."""

    def __init__(self, request_id: int, prompt_token_ids: Optional[List[int]],
                 outputs: List[TokenOutput], start_time: Optional[float],
                 server_info: Optional[ServerInfo], finished: bool, text: Optional[str] = None,
                 arrival_time: Optional[float] = None):
        self.request_id = request_id
        self.prompt_token_ids = prompt_token_ids
        self.outputs = outputs
        self.start_time = start_time
        self.server_info = server_info
        self.finished = finished
        self.text = text
        self.arrival_time = arrival_time

    def __repr__(self) -> str:
        return (f"RequestOutput(id={self.request_id}, tokens={len(self.outputs)}, "
                f"finished={self.finished})")


class Request:
    """One generation request and all of its scheduling state."""

    def __init__(self, arrival_time: float, request_id: int, prompt: Optional[str],
                 prompt_token_ids: List[int], sampling_params: Optional[SamplingParams] = None,
                 server_info: Optional[ServerInfo] = None, priority: int = 0,
                 fusion_exec: bool = False):
        self.arrival_time = arrival_time
        self.request_id = request_id
        self.prompt = prompt
        self.prompt_token_ids = list(prompt_token_ids)
        self.sampling_params = sampling_params if sampling_params is not None else SamplingParams()
        self.server_info = server_info
        self.priority = priority

        self.outputs: List[TokenOutput] = []
        self.generated_tokens: List[str] = []
        self.generated_token_ids: List[int] = []
        self.is_finished = False
        self.is_running = False
        self.output_capacity = 0
        self.sched_timestamp = 0.0
        self.start_time: Optional[float] = None
        self.process_time = 0.0
        self.execution_time = 0.0
        self.last_step_time = 0.0

        # chunked prefill window [prefill_begin_index, prefill_end_index)
        self.prefill_begin_index = 0
        self.prefill_end_index = len(self.prompt_token_ids)
        self.chunk_size = 0
        self.is_last_chunk = False
        self.is_assigned = False

        # KV placement across a balloon group
        self.fusion_exec = fusion_exec        # runs through the fused pipeline
        self.once_fusion_exec = False
        self.kv_fusion_rank = 0               # home instance for replica requests
        self.kvcache_ready = True

        # preemption / migration / reshard bookkeeping
        self.preempted_times = 0
        self.preempting = False
        self.resched_times = 0
        self.is_migrating_out = False
        self.migration_dst_engine = 0
        self.is_resharding = False
        self.use_mock_block = False

    # -- lengths -------------------------------------------------------------
    def get_input_len(self) -> int:
        return len(self.prompt_token_ids)

    def get_output_len(self) -> int:
        return len(self.generated_token_ids)

    def is_context_stage(self) -> bool:
        return not self.generated_token_ids

    def get_num_tokens(self) -> int:
        """Tokens whose KV the request will hold after its next step."""
        return self.get_input_len() + self.get_output_len()

    def get_kvcache_slots(self) -> int:
        return self.get_input_len() + self.get_output_len()

    def get_input_tokens_ids(self) -> List[int]:
        if self.is_context_stage():
            return self.prompt_token_ids[self.prefill_begin_index:self.prefill_end_index]
        return [self.generated_token_ids[-1]]

    def get_num_input_tokens(self) -> int:
        if self.is_context_stage():
            return self.prefill_end_index - self.prefill_begin_index
        return 1

    def start_position(self) -> int:
        if self.is_context_stage():
            return self.prefill_begin_index
        return self.get_input_len() + self.get_output_len() - 1

    def get_first_new_token_index(self) -> int:
        """Reference-compatible value (``request.py:442-459``)."""
        if self.is_context_stage():
            return self.prefill_begin_index
        return self.get_input_len() + self.get_output_len()

    def context_len_after_step(self) -> int:
        return self.start_position() + self.get_num_input_tokens()

    def get_unfinished_prefill_tokens(self) -> int:
        if not self.is_context_stage():
            return 0
        return self.get_input_len() - self.prefill_end_index

    # -- chunked prefill -----------------------------------------------------
    def have_follow_up_chunk(self) -> bool:
        return self.is_context_stage() and (self.prefill_end_index < self.get_input_len()
                                            or self.prefill_begin_index >= self.prefill_end_index)

    def set_chunk(self, chunk_size: int) -> int:
        """Set the current chunk to start at ``prefill_begin_index``; returns the
        unused part of ``chunk_size``."""
        if chunk_size <= 0:
            raise ValueError(f"chunk size must be positive, got {chunk_size}")
        self.chunk_size = chunk_size
        self.prefill_end_index = min(self.get_input_len(), self.prefill_begin_index + chunk_size)
        self.is_last_chunk = self.prefill_end_index >= self.get_input_len()
        return chunk_size - (self.prefill_end_index - self.prefill_begin_index)

    def set_next_chunk(self, chunk_size: int) -> int:
        self.prefill_begin_index = self.prefill_end_index
        return self.set_chunk(chunk_size)

    def allocate_next_chunk(self, additional_tokens: int = 0) -> int:
        self.chunk_size += additional_tokens
        self.prefill_begin_index = self.prefill_end_index
        self.prefill_end_index = min(self.prefill_begin_index + self.chunk_size, self.get_input_len())
        return self.chunk_size - (self.prefill_end_index - self.prefill_begin_index)

    def get_optimal_chunk_size(self, budget: int, floor: int = 1024) -> int:
        """Largest chunk n whose attention cost n*(n + 2*begin + 1)/2 fits ``budget``
        (positive root of n^2 + (2b+1)n - 2*budget = 0), at least ``floor``."""
        b = 2 * self.prefill_begin_index + 1
        disc = b * b + 8 * budget
        n = math.floor((-b + math.sqrt(disc)) / 2)
        return max(n, floor)

    def prepare_for_sequence_parallel_chunk(self) -> None:
        self.prefill_begin_index = self.prefill_end_index
        self.prefill_end_index = self.get_input_len()

    # -- generation ----------------------------------------------------------
    def _check_finish_condition(self) -> None:
        sp = self.sampling_params
        if self.get_output_len() >= sp.max_tokens:
            self.is_finished = True
        elif not sp.ignore_eos and self.generated_token_ids:
            last_id = self.generated_token_ids[-1]
            last_txt = self.generated_tokens[-1]
            if last_id in sp.stop_token_ids or (last_txt and last_txt in sp.stop):
                self.is_finished = True

    def add_generated_token(self, token: str, token_id: int, when: Optional[float] = None) -> None:
        if self.get_output_len() >= self.sampling_params.max_tokens:
            raise ValueError(f"request {self.request_id} already generated max_tokens")
        self.generated_tokens.append(token)
        self.generated_token_ids.append(int(token_id))
        self.outputs.append(TokenOutput(token, int(token_id), time.time() if when is None else when))
        self._check_finish_condition()

    def used_up_blocks(self) -> bool:
        return self.get_output_len() >= self.output_capacity

    def need_to_responsed(self) -> bool:
        return self.is_finished

    def prepare_for_recompute(self) -> None:
        """Fold generated tokens into the prompt so the request can be re-prefilled."""
        self.prompt_token_ids.extend(self.generated_token_ids)
        self.sampling_params.max_tokens -= len(self.generated_token_ids)
        self.sampling_params.max_tokens = max(self.sampling_params.max_tokens, 1)
        self.generated_tokens = []
        self.generated_token_ids = []
        self.prefill_begin_index = 0
        self.prefill_end_index = self.get_input_len()
        self.fusion_exec = True
        self.kv_fusion_rank = 0

    # -- timing --------------------------------------------------------------
    def add_process_time(self, t: float) -> None:
        self.process_time += t

    def add_execution_time(self, t: float) -> None:
        self.execution_time += t

    def get_response(self) -> str:
        return "".join(self.generated_tokens)

    def __repr__(self) -> str:
        return (f"Request(id={self.request_id}, in={self.get_input_len()}, "
                f"out={self.get_output_len()}, prefill=[{self.prefill_begin_index},"
                f"{self.prefill_end_index}), fusion={self.fusion_exec}, "
                f"kv_rank={self.kv_fusion_rank}, finished={self.is_finished})")


class BatchedRequests:
    """An ordered batch of requests for one engine step."""

    def __init__(self, requests: Optional[Iterable[Request]] = None):
        self.requests: List[Request] = list(requests) if requests is not None else []
        self.start_time: Optional[float] = None
        self.step_method = "step"

    def __len__(self) -> int:
        return len(self.requests)

    def __iter__(self):
        return iter(self.requests)

    def __repr__(self) -> str:
        return f"BatchedRequests({[r.request_id for r in self.requests]})"

    def add_request(self, request: Request) -> None:
        if any(r.request_id == request.request_id for r in self.requests):
            raise AssertionError(f"request {request.request_id} already in batch")
        self.requests.append(request)

    def add_requests(self, requests: Iterable[Request]) -> None:
        for r in requests:
            self.add_request(r)

    def pop_finished_requests(self) -> List[Request]:
        done = [r for r in self.requests if r.is_finished]
        self.requests = [r for r in self.requests if not r.is_finished]
        return done

    def pop_unassigned_requests(self) -> List[Request]:
        out = [r for r in self.requests if not r.is_assigned]
        self.requests = [r for r in self.requests if r.is_assigned]
        return out

    def set_sched_time(self) -> None:
        now = time.time()
        for r in self.requests:
            r.sched_timestamp = now

    def start_one_iteration(self, start_time: float) -> None:
        if not self.requests:
            return
        if self.start_time is not None:
            raise AssertionError("the batch already started an iteration")
        self.start_time = start_time
        for r in self.requests:
            if r.start_time is None:
                r.start_time = start_time

    def finish_one_iteration(self, generated_tokens: Sequence[str], generated_token_ids: Sequence[int],
                             end_time: float) -> None:
        if not self.requests:
            return
        assert self.start_time is not None, "the batch has not been started"
        for r, tok, tid in zip(self.requests, generated_tokens, generated_token_ids):
            r.last_step_time = end_time
            r.add_process_time(end_time - self.start_time)
            if r.have_follow_up_chunk():
                # the chunk only filled KV: the next window starts where this
                # one ended and stays empty until the scheduler sizes it
                r.prefill_begin_index = r.prefill_end_index
            else:
                r.add_generated_token(tok, tid, end_time)
        self.start_time = None

    def get_request_ids(self) -> List[int]:
        return [r.request_id for r in self.requests]

    def get_kvcache_slots(self) -> int:
        return sum(r.get_kvcache_slots() for r in self.requests)

    def get_unfinished_prefill_tokens(self) -> int:
        return sum(r.get_unfinished_prefill_tokens() for r in self.requests)

    def get_context_requests(self) -> List[Request]:
        return [r for r in self.requests if r.is_context_stage()]

    def get_decode_requests(self) -> List[Request]:
        return [r for r in self.requests if not r.is_context_stage()]

    def split_requests(self) -> Tuple[List[Request], List[Request]]:
        return self.get_context_requests(), self.get_decode_requests()

    def get_fusion_requests(self) -> Tuple[List[Request], List[Request]]:
        return ([r for r in self.requests if r.fusion_exec],
                [r for r in self.requests if not r.fusion_exec])

    # engine arguments
    def get_input_tokens_batched(self) -> List[List[int]]:
        return [r.get_input_tokens_ids() for r in self.requests]

    def get_num_input_tokens_batched(self) -> List[int]:
        return [r.get_num_input_tokens() for r in self.requests]

    def get_num_input_tokens(self) -> int:
        return sum(r.get_num_input_tokens() for r in self.requests)

    def get_first_token_indexes(self) -> List[int]:
        return [r.get_first_new_token_index() for r in self.requests]

    def get_start_positions(self) -> List[int]:
        return [r.start_position() for r in self.requests]

    def get_is_context_stage(self, use_tensor_cores: bool = False) -> List[int]:
        if use_tensor_cores:
            return [1] * len(self.requests)
        return [int(r.is_context_stage()) for r in self.requests]


_request_counter = itertools.count()


def create_request(prompt: Optional[str], prompt_token_ids: Optional[List[int]],
                   sampling_params: SamplingParams, server_info: Optional[ServerInfo] = None,
                   request_counter=None, tokenizer=None, max_model_len: int = 16384,
                   arrival_time: Optional[float] = None, request_id: Optional[int] = None) -> Request:
    """Tokenize (if needed), truncate to ``max_model_len`` and build a Request."""
    if request_id is None:
        request_id = next(request_counter if request_counter is not None else _request_counter)
    if prompt_token_ids is None:
        if prompt is None or tokenizer is None:
            raise ValueError("need prompt_token_ids, or a prompt and a tokenizer")
        prompt_token_ids = tokenizer.encode(prompt)
    if prompt is None and tokenizer is not None:
        prompt = tokenizer.decode(prompt_token_ids)
    room = max_model_len - sampling_params.max_tokens
    if len(prompt_token_ids) > room:
        prompt_token_ids = list(prompt_token_ids)[:max(room, 1)]
    return Request(time.time() if arrival_time is None else arrival_time, request_id, prompt,
                   list(prompt_token_ids), sampling_params, server_info=server_info)


class MigratingRequest:
    """A request whose KV blocks still sit on another engine (KV handoff)."""

    def __init__(self, req: Request, block_indexes: List[int], source_rank: int = 0):
        self.req = req
        self.block_indexes = block_indexes
        self.source_rank = source_rank
