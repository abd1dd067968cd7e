"""Credit-based FIFO admission and the worker loop (pagedcore_b200.scheduler), on CPU.

The worker runs over the C++ block ledger alone (no pool, no GPU): prefill
caches the prompt, each decode step caches one token per active request,
exactly the bookkeeping the KV path does, so credits, block assignment and
release are checked against the real ledger.
"""

from __future__ import annotations

import random

import pytest

from pagedcore_b200.engine_types import CapacityCounts, FinishReason, RequestId
from pagedcore_b200.ledger import BlockLedger
from pagedcore_b200.scheduler import Request, Worker, required_blocks


class LedgerAllocator:
    """The bookkeeping surface of KVAllocator on the ledger alone."""

    def __init__(self, blocks: int) -> None:
        self.ledger = BlockLedger(blocks)
        self.handles: dict[RequestId, int] = {}
        self.next = 0

    def create(self, reservation) -> None:
        self.ledger.reserve(self.next, reservation.maximum_block_credits)
        self.handles[reservation.request_id] = self.next
        self.next += 1

    def release_all(self, request_id: RequestId) -> None:
        self.ledger.release(self.handles.pop(request_id))

    def capacity(self) -> CapacityCounts:
        return CapacityCounts(*self.ledger.capacity())

    def cached_length(self, request_id: RequestId) -> int:
        return self.ledger.length(self.handles[request_id])


def make_worker(blocks: int, max_active: int, tokens=None):
    allocator = LedgerAllocator(blocks)
    log = []

    def prefill(request: Request) -> int:
        allocator.ledger.append(allocator.handles[request.request_id], request.prompt_tokens)
        log.append(("prefill", request.request_id))
        return 100 if tokens is None else tokens(request)

    def decode(batch) -> list[int]:
        handles = [allocator.handles[r.request_id] for r in batch]
        allocator.ledger.decode_begin(handles)
        for layer in range(22):
            for handle in handles:
                allocator.ledger.decode_check(handle, layer)
                allocator.ledger.decode_mark(handle, layer)
        allocator.ledger.decode_commit()
        log.append(("decode", tuple(r.request_id for r in batch)))
        return [100 if tokens is None else tokens(r) for r in batch]

    return Worker(allocator, prefill, decode, max_active=max_active), allocator, log


def request(name: str, prompt: int, new: int, **kw) -> Request:
    return Request(RequestId(name), prompt, new, **kw)


def run(worker: Worker, limit: int = 10_000) -> None:
    while not worker.idle() and worker.iterations < limit:
        worker.iterate()
    assert worker.idle()


def test_required_blocks_counts_every_cached_token() -> None:
    # prompt + max_new - 1 tokens are cached: the last emitted token never is.
    assert required_blocks(16, 1) == 1
    assert required_blocks(16, 2) == 2
    assert required_blocks(1, 16) == 1
    assert required_blocks(2047, 1) == 128
    assert required_blocks(1, 2047) == 128


def test_a_request_caches_prompt_plus_outputs_minus_one_and_frees_everything() -> None:
    worker, allocator, log = make_worker(32, 4)
    worker.submit(request("a", 20, 13))
    lengths = []
    while not worker.idle():
        worker.iterate()
        if RequestId("a") in allocator.handles:
            lengths.append(allocator.cached_length(RequestId("a")))
    done = worker.completed[0]
    assert done.finish_reason == FinishReason.LENGTH and len(done.output) == 13
    assert max(lengths) == 20 + 13 - 1
    assert allocator.capacity() == CapacityCounts(32, 32, 0, 0, 0, 0)
    assert log[0] == ("prefill", "a") and sum(1 for kind, _ in log if kind == "decode") == 12


def test_the_queue_head_blocks_later_requests_that_would_fit() -> None:
    worker, allocator, log = make_worker(64, 8)
    worker.submit(request("big", 600, 40))     # 40 blocks
    worker.submit(request("next", 400, 80))    # 30 blocks: does not fit beside "big"
    worker.submit(request("small", 16, 16))    # 2 blocks: would fit, but waits behind "next"
    worker.iterate()
    assert list(worker.active) == ["big"]
    for _ in range(30):
        worker.iterate()
        assert "small" not in worker.active and [r.request_id for r in worker.pending] == ["next", "small"]
    run(worker)
    prefills = [name for kind, name in log if kind == "prefill"]
    assert prefills == ["big", "next", "small"]
    assert allocator.capacity().reserved_blocks == 0


def test_active_slots_limit_admission() -> None:
    worker, _, _ = make_worker(256, 2)
    for i in range(4):
        worker.submit(request(f"r{i}", 10, 50))
    for _ in range(5):
        worker.iterate()
        assert len(worker.active) <= 2
    run(worker)
    assert len(worker.completed) == 4


def test_one_admission_per_iteration_and_release_on_the_next() -> None:
    worker, allocator, log = make_worker(64, 8)
    for i in range(3):
        worker.submit(request(f"r{i}", 8, 2))
    worker.iterate()  # admits r0 (prefill + decode: finishes with 2 tokens)
    assert [name for kind, name in log if kind == "prefill"] == ["r0"]
    assert worker.finished and allocator.capacity().reserved_blocks == 1  # not released yet
    worker.iterate()  # releases r0, admits r1
    assert allocator.capacity().reserved_blocks == 1 and "r1" in [r.request_id for r in worker.finished]
    run(worker)
    assert [r.request_id for r in worker.completed] == ["r0", "r1", "r2"]


def test_eos_finishes_early_unless_ignored() -> None:
    worker, allocator, _ = make_worker(64, 8, tokens=lambda r: 2 if len(r.output) == 3 else 7)
    worker.submit(request("stops", 5, 50))
    worker.submit(request("ignores", 5, 10, ignore_eos=True))
    run(worker)
    by_name = {r.request_id: r for r in worker.completed}
    assert by_name["stops"].finish_reason == FinishReason.EOS and len(by_name["stops"].output) == 4
    assert by_name["ignores"].finish_reason == FinishReason.LENGTH and len(by_name["ignores"].output) == 10
    assert allocator.capacity() == CapacityCounts(64, 64, 0, 0, 0, 0)


def test_submit_rejects_what_can_never_run() -> None:
    worker, _, _ = make_worker(16, 4)
    with pytest.raises(ValueError, match="2048"):
        worker.submit(request("long", 2000, 100))
    with pytest.raises(ValueError, match="total KV pool capacity"):
        worker.submit(request("wide", 300, 10))
    with pytest.raises(ValueError, match="at least one"):
        worker.submit(request("empty", 0, 5))


def test_a_failed_prefill_returns_its_credits() -> None:
    allocator = LedgerAllocator(16)

    def prefill(_: Request) -> int:
        raise RuntimeError("prefill failed")

    worker = Worker(allocator, prefill, lambda batch: [0] * len(batch), max_active=2)
    worker.submit(request("r", 10, 5))
    with pytest.raises(RuntimeError, match="prefill failed"):
        worker.iterate()
    assert allocator.capacity() == CapacityCounts(16, 16, 0, 0, 0, 0)
    assert not worker.active


def test_a_long_random_run_keeps_the_ledger_consistent() -> None:
    rng = random.Random(11)
    worker, allocator, _ = make_worker(400, 24, tokens=lambda r: 2 if rng.random() < 0.02 else 9)
    expected = 0
    for i in range(120):
        prompt = rng.randint(1, 600)
        new = rng.randint(1, min(300, 2048 - prompt))
        worker.submit(request(f"q{i}", prompt, new))
        expected += new
    while not worker.idle():
        worker.iterate()
        counts = allocator.capacity()
        assert counts.owned_blocks <= counts.reserved_blocks <= counts.total_blocks
        if worker.iterations % 50 == 0:
            allocator.ledger.audit()
    assert len(worker.completed) == 120
    assert sum(len(r.output) for r in worker.completed) <= expected
    assert allocator.capacity() == CapacityCounts(400, 400, 0, 0, 0, 0)
