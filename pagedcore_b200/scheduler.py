"""Credit-based admission and the decode loop of one GPU worker.

PagedCore specifies this worker but has not built it (docs/DESIGN.md,
"Admission without preemption" and "Scheduler iteration"); this is that
specification over the KV path:

* A request is admitted only with a free active slot and KV credits for
  ``ceil((prompt + max_new - 1) / 16)`` blocks (prefill caches the prompt,
  every decode step caches the token before it, the last emitted token is
  never cached), and only if ``prompt + max_new <= 2048``.  Credits are
  reserved at admission (``KVAllocator.create``); blocks are assigned as
  tokens are cached.
* The pending queue is strict FIFO: only its head is tried, and a head that
  does not fit blocks everything behind it.
* One iteration: release the requests that finished in the previous one,
  admit at most one request and prefill it (its first token comes from the
  prompt logits), then one decode step for every active request, one token
  each.  A request finishes at its token limit or on EOS (unless told to
  ignore it); its resources return at the start of the next iteration.

The model is passed in as two callables, so the same loop drives the full
decoder, or synthetic K/V for KV-path stress runs.
"""

from __future__ import annotations

from collections import deque
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field

from pagedcore_b200.engine_types import FinishReason, KVReservation, RequestId

BLOCK_TOKENS = 16
CONTEXT_LIMIT = 2048
EOS_TOKEN = 2


def required_blocks(prompt_tokens: int, max_new_tokens: int) -> int:
    """KV credits a request needs to finish without preemption."""
    return -(-(prompt_tokens + max_new_tokens - 1) // BLOCK_TOKENS)


@dataclass
class Request:
    request_id: RequestId
    prompt_tokens: int
    max_new_tokens: int
    ignore_eos: bool = False
    output: list[int] = field(default_factory=list)
    finish_reason: FinishReason | None = None

    @property
    def last_token(self) -> int:
        return self.output[-1]


# prefill(request) -> first token id; decode(requests) -> one token id per request
PrefillFn = Callable[[Request], int]
DecodeFn = Callable[[Sequence[Request]], Sequence[int]]


class Worker:
    """Admission queue, active set and the iteration loop for one allocator.

    ``allocator`` needs ``create(KVReservation)``, ``release_all(request_id)``
    and ``capacity()``, as ``KVAllocator`` has them.
    """

    def __init__(self, allocator, prefill: PrefillFn, decode: DecodeFn, *, max_active: int) -> None:
        if type(max_active) is not int or max_active < 1:
            raise ValueError("max_active must be a positive integer")
        self.allocator = allocator
        self.prefill = prefill
        self.decode = decode
        self.max_active = max_active
        self.pending: deque[Request] = deque()
        self.active: dict[RequestId, Request] = {}
        self.finished: list[Request] = []  # finished in the last iteration, released in the next
        self.completed: list[Request] = []
        self.iterations = 0

    # -- admission ---------------------------------------------------------------
    def submit(self, request: Request) -> None:
        """Queue a request (checked against the context limit and the pool)."""
        if request.prompt_tokens < 1 or request.max_new_tokens < 1:
            raise ValueError("a request needs at least one prompt token and one new token")
        if request.prompt_tokens + request.max_new_tokens > CONTEXT_LIMIT:
            raise ValueError("prompt tokens plus requested output must not exceed 2048")
        if required_blocks(request.prompt_tokens, request.max_new_tokens) > self.allocator.capacity().total_blocks:
            raise ValueError("request exceeds the total KV pool capacity")
        self.pending.append(request)

    def _admit_head(self) -> Request | None:
        if not self.pending or len(self.active) >= self.max_active:
            return None
        head = self.pending[0]
        blocks = required_blocks(head.prompt_tokens, head.max_new_tokens)
        counts = self.allocator.capacity()
        if blocks > counts.total_blocks - counts.reserved_blocks:
            return None  # strict FIFO: the head waits, and so does everything behind it
        self.allocator.create(KVReservation(head.request_id, blocks))
        self.pending.popleft()
        self.active[head.request_id] = head
        return head

    # -- the loop ----------------------------------------------------------------
    def _emit(self, request: Request, token: int) -> None:
        request.output.append(int(token))
        if token == EOS_TOKEN and not request.ignore_eos:
            request.finish_reason = FinishReason.EOS
        elif len(request.output) >= request.max_new_tokens:
            request.finish_reason = FinishReason.LENGTH
        if request.finish_reason is not None:
            del self.active[request.request_id]
            self.finished.append(request)

    def iterate(self) -> int:
        """One worker iteration; returns the number of tokens emitted."""
        for request in self.finished:
            self.allocator.release_all(request.request_id)
            self.completed.append(request)
        self.finished = []
        emitted = 0
        admitted = self._admit_head()
        if admitted is not None:
            try:
                token = self.prefill(admitted)
            except BaseException:
                # The caller owns cleanup of a failed prefill: give its credits back.
                del self.active[admitted.request_id]
                self.allocator.release_all(admitted.request_id)
                raise
            self._emit(admitted, token)
            emitted += 1
        batch = list(self.active.values())
        if batch:
            tokens = self.decode(batch)
            if len(tokens) != len(batch):
                raise RuntimeError("decode must return one token per active request")
            for request, token in zip(batch, tokens, strict=True):
                self._emit(request, token)
            emitted += len(batch)
        self.iterations += 1
        return emitted

    def idle(self) -> bool:
        return not (self.pending or self.active or self.finished)
