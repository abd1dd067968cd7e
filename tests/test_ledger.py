"""The C++ block ledger against the oracle and the reference's known answers.

Ports the bookkeeping half of the reference's allocator tests
(tests/unit/test_kv_cache.py, tests/unit/test_kv_cache_properties.py) to
``BlockLedger`` (no GPU needed): block order, credits, capacity tuples,
staged decode, error classes and messages, corruption detection.  The data
half of those tests runs on the GPU in test_kv_allocator_gpu.py.
"""

from __future__ import annotations

import hashlib
import math
import re

import numpy as np
import pytest
from hypothesis import settings
from hypothesis import strategies as st
from hypothesis.stateful import RuleBasedStateMachine, invariant, precondition, rule, run_state_machine_as_test

from oracle.allocator import OracleAllocator
from pagedcore_b200 import workloads
from pagedcore_b200.ledger import BlockLedger


@pytest.fixture(params=["full", "incremental"])
def validation(request: pytest.FixtureRequest) -> str:
    return request.param


def test_first_pops_are_zero_one_two(validation: str) -> None:
    ledger = BlockLedger(8, validation)
    assert ledger.free_list() == list(reversed(range(8)))
    ledger.reserve(1, 3)
    assert ledger.append(1, 33).tolist()[::16] == [0, 16, 32]
    assert ledger.table(1) == (0, 1, 2)


@pytest.mark.parametrize("tokens,blocks,last", [(1, 1, 1), (15, 1, 15), (16, 1, 16), (17, 2, 1), (32, 2, 16), (33, 3, 1)])
def test_token_to_block_mapping(tokens: int, blocks: int, last: int, validation: str) -> None:
    # tests/unit/test_kv_cache.py:150-181
    ledger = BlockLedger(4, validation)
    ledger.reserve(7, blocks)
    assert ledger.table(7) == () and ledger.length(7) == 0
    slots = ledger.append(7, tokens)
    table = ledger.table(7)
    assert len(table) == blocks and len(set(table)) == blocks
    assert ledger.length(7) == tokens
    assert slots.tolist() == [table[p // 16] * 16 + p % 16 for p in range(tokens)]
    assert tokens - 16 * (blocks - 1) == last


def test_fragmented_appends_golden_table(validation: str) -> None:
    # tests/unit/test_kv_cache.py:184-211: tables (0, 2, 3) and (1,)
    ledger = BlockLedger(4, validation)
    ledger.reserve(1, 3)
    ledger.reserve(2, 1)
    ledger.append(1, 15)
    first = ledger.table(1)
    ledger.append(2, 16)
    ledger.append(1, 1)
    assert ledger.table(1) == first
    ledger.append(1, 1)
    ledger.append(1, 16)
    assert ledger.table(1) == (0, 2, 3)
    assert ledger.table(2) == (1,)
    assert ledger.length(1) == 33


def test_capacity_sequence_across_requests(validation: str) -> None:
    # tests/unit/test_kv_cache.py:454-481
    ledger = BlockLedger(8, validation)
    assert ledger.capacity() == (8, 8, 0, 0, 0, 0)
    ledger.reserve(1, 3)
    assert ledger.capacity() == (8, 8, 0, 3, 1, 0)
    ledger.reserve(2, 2)
    assert ledger.capacity() == (8, 8, 0, 5, 2, 0)
    ledger.append(1, 15)
    assert ledger.capacity() == (8, 7, 1, 5, 2, 15)
    ledger.append(2, 16)
    assert ledger.capacity() == (8, 6, 2, 5, 2, 31)
    ledger.append(1, 1)
    assert ledger.capacity() == (8, 6, 2, 5, 2, 32)
    ledger.append(1, 1)
    assert ledger.capacity() == (8, 5, 3, 5, 2, 33)
    ledger.append(1, 16)
    assert ledger.capacity() == (8, 4, 4, 5, 2, 49)
    ledger.release(1)
    assert ledger.capacity() == (8, 7, 1, 2, 1, 16)
    ledger.release(2)
    assert ledger.capacity() == (8, 8, 0, 0, 0, 0)


def test_prefill_into_reused_fragmented_pages(validation: str) -> None:
    # tests/unit/test_decoder.py:439-476: table (2, 0, 3, 4)[:blocks]
    for tokens in (1, 15, 16, 17, 49):
        ledger = BlockLedger(6, validation)
        for request in (1, 2, 3):
            ledger.reserve(request, 1)
            ledger.append(request, 16)
        ledger.release(1)
        ledger.release(3)
        blocks = (tokens + 15) // 16
        ledger.reserve(9, blocks)
        ledger.append(9, tokens)
        assert ledger.table(9) == (2, 0, 3, 4)[:blocks]
        assert ledger.capacity() == (6, 5 - blocks, blocks + 1, blocks + 1, 2, tokens + 16)


def test_attention_blocker_table(validation: str) -> None:
    # tests/unit/test_attention.py:189-197: table (0, 2)
    ledger = BlockLedger(3, validation)
    ledger.reserve(1, 2)
    ledger.append(1, 16)
    ledger.reserve(2, 1)
    ledger.append(2, 16)
    ledger.append(1, 1)
    assert ledger.table(1) == (0, 2)


def test_release_order_puts_first_block_on_top(validation: str) -> None:
    ledger = BlockLedger(5, validation)
    ledger.reserve(1, 3)
    ledger.append(1, 40)
    assert ledger.table(1) == (0, 1, 2)
    ledger.release(1)
    assert ledger.free_list() == [4, 3, 2, 1, 0]
    with pytest.raises(KeyError):
        ledger.release(1)


def test_reservation_errors(validation: str) -> None:
    ledger = BlockLedger(3, validation)
    ledger.reserve(1, 3)
    with pytest.raises(ValueError, match="already has a KV cache"):
        ledger.reserve(1, 1)
    with pytest.raises(RuntimeError, match="insufficient unreserved blocks"):
        ledger.reserve(2, 1)
    assert ledger.capacity() == (3, 3, 0, 3, 1, 0)
    with pytest.raises(ValueError, match="total KV pool capacity"):
        BlockLedger(2).reserve(1, 3)
    with pytest.raises(ValueError, match="KV context capacity"):
        BlockLedger(129).reserve(1, 129)
    with pytest.raises(ValueError, match="positive"):
        ledger.reserve(5, 0)


def test_append_limits_preserve_state(validation: str) -> None:
    # tests/unit/test_kv_cache.py:236-260, 360-372
    ledger = BlockLedger(2, validation)
    ledger.reserve(1, 1)
    ledger.reserve(2, 1)
    ledger.append(1, 15)
    ledger.append(2, 16)
    before = ledger.capacity()
    with pytest.raises(RuntimeError, match="exceeds request reservation"):
        ledger.append_plan(1, 2)
    assert ledger.capacity() == before and ledger.length(1) == 15
    ledger.append(1, 1)
    big = BlockLedger(128, validation)
    big.reserve(1, 128)
    big.append(1, 2048)
    with pytest.raises(ValueError, match="2048"):
        big.append_plan(1, 1)
    assert big.length(1) == 2048
    with pytest.raises(KeyError):
        big.append_plan(99, 1)


def test_plan_does_not_mutate_and_commit_publishes(validation: str) -> None:
    ledger = BlockLedger(4, validation)
    ledger.reserve(1, 4)
    slots, start = ledger.append_plan(1, 20)
    assert start == 0 and ledger.length(1) == 0 and ledger.capacity() == (4, 4, 0, 4, 1, 0)
    ledger.append_commit(1, 20)
    assert ledger.table(1) == (0, 1)
    assert slots.tolist() == list(range(16)) + list(range(16, 20))


def churned_ledger(validation: str) -> BlockLedger:
    """A ledger with a fragmented free list and three reserved, partly filled requests."""
    ledger = BlockLedger(64, validation)
    for request in range(10, 20):
        ledger.reserve(request, 3)
        ledger.append(request, 5 + request)
    for request in (11, 14, 15, 18):
        ledger.release(request)
    for request, credits, filled in ((1, 8, 0), (2, 4, 20), (3, 6, 7)):
        ledger.reserve(request, credits)
        if filled:
            ledger.append(request, filled)
    return ledger


def test_batched_append_takes_the_slots_of_sequential_appends(validation: str) -> None:
    batched, sequential = churned_ledger(validation), churned_ledger(validation)
    requests, tokens = [3, 1, 2], [40, 100, 13]
    slots, starts = batched.append_plan_many(requests, tokens)
    assert batched.capacity() == sequential.capacity()  # planning changes nothing
    expected = [sequential.append(r, t) for r, t in zip(requests, tokens, strict=True)]
    assert slots.tolist() == np.concatenate(expected).tolist()
    assert starts.tolist() == [7, 0, 20]
    batched.append_commit_many(requests, tokens)
    assert batched.capacity() == sequential.capacity()
    assert batched.free_list() == sequential.free_list()
    for request in requests:
        assert batched.table(request) == sequential.table(request)
        assert batched.length(request) == sequential.length(request)


@pytest.mark.parametrize(
    "requests, tokens, error, match",
    [
        ([3, 2], [40, 60], RuntimeError, "exceeds request reservation"),  # the second overruns its credits
        ([3, 2], [10, 2040], ValueError, "2048|invalid KV append"),  # 20 cached + 2040 > 2048
        ([3, 99], [10, 1], KeyError, "99"),
        ([3, 3], [1, 1], ValueError, "only once"),
        ([3, 1], [10, 0], ValueError, "tokens|invalid KV append"),
    ],
)
def test_a_failing_batched_append_changes_nothing(requests, tokens, error, match, validation: str) -> None:
    ledger = churned_ledger(validation)
    before = (ledger.capacity(), ledger.free_list(), [ledger.table(r) for r in (1, 2, 3)])
    with pytest.raises(error, match=match):
        ledger.append_plan_many(requests, tokens)
    with pytest.raises(error, match=match):
        ledger.append_commit_many(requests, tokens)
    assert (ledger.capacity(), ledger.free_list(), [ledger.table(r) for r in (1, 2, 3)]) == before


def test_batched_append_fills_the_pool_with_disjoint_slots(validation: str) -> None:
    ledger = BlockLedger(6, validation)
    for request in (1, 2):
        ledger.reserve(request, 3)
    ledger.append(1, 1)
    slots, starts = ledger.append_plan_many([1, 2], [40, 48])
    assert len(set(slots.tolist())) == 88 and starts.tolist() == [1, 0]
    ledger.append_commit_many([1, 2], [40, 48])
    assert ledger.length(1) == 41 and ledger.length(2) == 48
    assert ledger.free_list() == [] and sorted(ledger.table(1) + ledger.table(2)) == list(range(6))


def test_staged_decode_semantics(validation: str) -> None:
    # tests/unit/test_kv_cache.py:375-418
    ledger = BlockLedger(4, validation)
    for request in (1, 2):
        ledger.reserve(request, 2)
        ledger.append(request, 16)
    counts = ledger.capacity()
    tables = [ledger.table(1), ledger.table(2)]
    slots, positions = ledger.decode_begin([1, 2])
    # Both rows start a new block: free[-1] then free[-2].
    assert slots.tolist() == [2 * 16, 3 * 16] and positions.tolist() == [16, 16]
    with pytest.raises(RuntimeError, match="unwritten"):
        ledger.view(1, 0)
    for operation in (lambda: ledger.reserve(9, 1), lambda: ledger.append_plan(1, 1), lambda: ledger.release(1),
                      lambda: ledger.decode_begin([1])):
        with pytest.raises(RuntimeError, match="staged decode"):
            operation()
    for layer in range(22):
        for request in (1, 2):
            ledger.decode_check(request, layer)
            ledger.decode_mark(request, layer)
            blocks, length = ledger.view(request, layer)
            assert len(blocks) == 2 and length == 17
            assert ledger.length(request) == 16 and ledger.capacity() == counts
    assert [ledger.table(1), ledger.table(2)] == tables
    ledger.decode_commit()
    assert ledger.capacity() == (4, 0, 4, 4, 2, 34)
    assert ledger.table(1) == (0, 2) and ledger.table(2) == (1, 3)


@pytest.mark.parametrize("fault", ["incomplete", "order", "layer"])
def test_staged_decode_rejections_leave_state(fault: str, validation: str) -> None:
    ledger = BlockLedger(2, validation)
    ledger.reserve(1, 2)
    ledger.append(1, 16)
    counts = ledger.capacity()
    ledger.decode_begin([1])
    if fault == "incomplete":
        ledger.decode_mark(1, 0)
        with pytest.raises(RuntimeError, match="every cache layer"):
            ledger.decode_commit()
    elif fault == "order":
        with pytest.raises(ValueError, match="once in order"):
            ledger.decode_check(1, 1)
        ledger.decode_abort()
    else:
        with pytest.raises(ValueError, match="layer_index"):
            ledger.decode_check(1, 22)
        ledger.decode_abort()
    assert not ledger.staging
    assert ledger.capacity() == counts and ledger.length(1) == 16
    ledger.release(1)
    assert ledger.capacity() == (2, 2, 0, 0, 0, 0)


def test_decode_rejects_bad_batches(validation: str) -> None:
    ledger = BlockLedger(130, validation)
    ledger.reserve(1, 128)
    ledger.append(1, 2048)
    ledger.reserve(2, 1)
    with pytest.raises(ValueError, match="nonempty, distinct"):
        ledger.decode_begin([])
    with pytest.raises(ValueError, match="nonempty, distinct"):
        ledger.decode_begin([1, 1])
    with pytest.raises(ValueError, match="2047"):
        ledger.decode_begin([1])
    with pytest.raises(ValueError, match="2047"):
        ledger.decode_begin([2])  # empty cache
    with pytest.raises(KeyError):
        ledger.decode_begin([77])
    ledger.append(2, 16)
    with pytest.raises(RuntimeError, match="exceeds request reservation"):
        ledger.decode_begin([2])
    assert not ledger.staging


def test_batch_metadata_matches_views(validation: str) -> None:
    ledger = BlockLedger(40, validation)
    lengths = [1, 16, 17, 100, 300]
    for request, length in enumerate(lengths):
        ledger.reserve(request, workloads.blocks_for(length + 1))
        ledger.append(request, length)
    got_lengths, prefix, flat = ledger.batch([4, 0, 2], 3)
    assert got_lengths.tolist() == [300, 1, 17]
    assert prefix.tolist() == [0, 19, 20, 22]
    assert flat.tolist() == list(ledger.table(4)) + list(ledger.table(0)) + list(ledger.table(2))
    ledger.reserve(99, 1)
    with pytest.raises(ValueError, match="nonempty cache"):
        ledger.batch([99], 0)
    ledger.decode_begin([0, 1])
    with pytest.raises(RuntimeError, match="unwritten"):
        ledger.batch([0, 1], 0)
    ledger.decode_mark(-1, 0)
    got_lengths, prefix, flat = ledger.batch([0, 1], 0)
    assert got_lengths.tolist() == [2, 17]
    assert prefix.tolist() == [0, 1, 3]
    ledger.decode_abort()


@pytest.mark.parametrize("corruption", ["duplicate", "foreign", "free", "negative", "outside", "short", "length"])
def test_corrupt_tables_are_detected(corruption: str) -> None:
    # tests/unit/test_kv_cache.py:572-624 (the Python-type corruptions have no C analogue)
    ledger = BlockLedger(4, "full")
    ledger.reserve(1, 3)
    ledger.reserve(2, 1)
    ledger.append(1, 17)
    ledger.append(2, 1)
    first, last = ledger.table(1)
    tables = {
        "duplicate": (first, first),
        "foreign": (ledger.table(2)[0], last),
        "free": (ledger.free_list()[-1], last),
        "negative": (-1, last),
        "outside": (4, last),
        "short": (first,),
        "length": (first, last),
    }
    ledger.debug_set_table(1, tables[corruption], 16 if corruption == "length" else 17)
    free = ledger.free_list()
    for operation in (lambda: ledger.table(1), lambda: ledger.append_plan(1, 1), lambda: ledger.release(1)):
        with pytest.raises(RuntimeError, match="KV"):
            operation()
    assert ledger.free_list() == free
    ledger.debug_set_table(1, (first, last), 17)
    assert ledger.capacity() == (4, 1, 3, 4, 2, 18)


def test_swapped_tables_report_foreign_ownership() -> None:
    # tests/unit/test_kv_cache.py:627-651
    ledger = BlockLedger(4, "full")
    ledger.reserve(1, 2)
    ledger.reserve(2, 2)
    ledger.append(1, 1)
    ledger.append(2, 1)
    a, b = ledger.table(1), ledger.table(2)
    ledger.debug_set_table(1, b, 1)
    ledger.debug_set_table(2, a, 1)
    with pytest.raises(RuntimeError, match="owned"):
        ledger.release(1)


@pytest.mark.parametrize("corruption", ["duplicate", "missing", "owned", "invalid"])
def test_corrupt_free_lists_are_detected(corruption: str) -> None:
    # tests/unit/test_kv_cache.py:654-677
    ledger = BlockLedger(3, "full")
    ledger.reserve(1, 1)
    ledger.append(1, 1)
    free = ledger.free_list()
    if corruption == "duplicate":
        free.append(free[-1])
    elif corruption == "missing":
        free.pop()
    elif corruption == "owned":
        free[-1] = ledger.table(1)[0]
    else:
        free[-1] = -1
    ledger.debug_set_free(free)
    with pytest.raises(RuntimeError, match="KV"):
        ledger.release(1)


def test_incremental_mode_checks_touched_requests() -> None:
    ledger = BlockLedger(4, "incremental")
    ledger.reserve(1, 2)
    ledger.append(1, 17)
    ledger.debug_set_table(1, (0, 9), 17)
    with pytest.raises(RuntimeError, match="invalid physical KV block"):
        ledger.table(1)
    with pytest.raises(RuntimeError, match="invalid physical KV block"):
        ledger.audit()


def test_reorder_free_requires_permutation() -> None:
    ledger = BlockLedger(4)
    ledger.reorder_free([2, 0, 3, 1])
    ledger.reserve(1, 2)
    ledger.append(1, 17)
    assert ledger.table(1) == (1, 3)
    with pytest.raises(ValueError, match="permutation"):
        ledger.reorder_free([2, 2])


def replay_churn(ledger: BlockLedger, case: workloads.AppendCase) -> None:
    for op in case.churn:
        if op.kind == "create":
            ledger.reserve(op.request, op.credits)
            ledger.append(op.request, op.tokens)
        else:
            ledger.release(op.request)


def test_config2_bookkeeping_matches_reference(append_golden: dict) -> None:
    """10k-op churn, 8 prompts, 256 staged decode rows: identical to the reference."""
    case = workloads.append_case()
    ledger = BlockLedger(case.num_blocks, "incremental")
    replay_churn(ledger, case)
    assert list(ledger.capacity()) == append_golden["after_churn"]["capacity"]
    assert ledger.free_list() == append_golden["after_churn"]["free_list"]
    for prompt in case.prompts:
        ledger.reserve(prompt.request, prompt.credits)
        ledger.append(prompt.request, prompt.key.shape[1])
    assert list(ledger.capacity()) == append_golden["after_prompts"]["capacity"]
    for request, table in append_golden["after_prompts"]["tables"].items():
        assert list(ledger.table(int(request))) == table
    ledger.decode_begin(list(case.decode.requests))
    ledger.decode_mark(-1, 0)
    for layer in range(1, 22):
        ledger.decode_mark(-1, layer)
    ledger.decode_commit()
    ledger.audit()
    assert list(ledger.capacity()) == append_golden["after_decode"]["capacity"]
    for request, table in append_golden["after_decode"]["tables"].items():
        assert list(ledger.table(int(request))) == table
        assert ledger.length(int(request)) == append_golden["after_decode"]["lengths"][request]
    digest = hashlib.sha256(np.asarray(ledger.free_list(), dtype=np.int64)).hexdigest()
    assert digest == append_golden["after_decode"]["free_list_sha256"]


def test_churn_matches_oracle_step_by_step() -> None:
    case = workloads.append_case(seed=11, num_blocks=256, churn_count=1500, prompt_count=2, decode_rows=16,
                                 max_prompt=300, churn_tokens=40)
    ledger = BlockLedger(case.num_blocks, "full")
    oracle = OracleAllocator(case.num_blocks, audit=False)
    for op in case.churn:
        if op.kind == "create":
            ledger.reserve(op.request, op.credits)
            oracle.create(op.request, op.credits)
            assert ledger.append(op.request, op.tokens).tolist() == oracle.append(op.request, op.tokens)
        else:
            ledger.release(op.request)
            oracle.release(op.request)
        assert ledger.capacity() == oracle.capacity_unchecked()
    assert ledger.free_list() == oracle.free
    for prompt in case.prompts:
        ledger.reserve(prompt.request, prompt.credits)
        oracle.create(prompt.request, prompt.credits)
        tokens = prompt.key.shape[1]
        assert ledger.append(prompt.request, tokens).tolist() == oracle.append(prompt.request, tokens)
    slots, positions = ledger.decode_begin(list(case.decode.requests))
    oracle_slots, oracle_positions = oracle.decode_begin(case.decode.requests)
    assert slots.tolist() == oracle_slots and positions.tolist() == oracle_positions


class _LedgerMachine(RuleBasedStateMachine):
    """Random create/append/decode/release against the oracle (test_kv_cache_properties.py:35-183)."""

    def __init__(self, blocks: int) -> None:
        super().__init__()
        self.ledger = BlockLedger(blocks, "full")
        self.oracle = OracleAllocator(blocks)
        self.total = blocks

    @rule(slot=st.integers(0, 3), credits=st.integers(1, 9))
    def create(self, slot: int, credits: int) -> None:
        outcome = _outcome(lambda: self.oracle.create(slot, credits))
        if outcome is None:
            self.ledger.reserve(slot, credits)
        else:
            with pytest.raises(type(outcome), match=_pattern(outcome)):
                self.ledger.reserve(slot, credits)

    @precondition(lambda self: bool(self.oracle.sequences))
    @rule(data=st.data(), tokens=st.sampled_from((1, 2, 15, 16, 17, 31, 32, 33)))
    def append(self, data: st.DataObject, tokens: int) -> None:
        request = data.draw(st.sampled_from(sorted(self.oracle.sequences)))
        expected = []
        outcome = _outcome(lambda: expected.extend(self.oracle.append(request, tokens)))
        if outcome is None:
            assert self.ledger.append(request, tokens).tolist() == expected
        else:
            with pytest.raises(type(outcome), match=_pattern(outcome)):
                self.ledger.append(request, tokens)

    @precondition(lambda self: bool(self.oracle.sequences))
    @rule(data=st.data())
    def decode(self, data: st.DataObject) -> None:
        requests = tuple(data.draw(st.lists(st.sampled_from(sorted(self.oracle.sequences)), min_size=1, max_size=3,
                                            unique=True)))
        result = []
        outcome = _outcome(lambda: result.append(self.oracle.decode_begin(requests)))
        if outcome is not None:
            with pytest.raises(type(outcome), match=_pattern(outcome)):
                self.ledger.decode_begin(list(requests))
            return
        slots, positions = self.ledger.decode_begin(list(requests))
        assert (slots.tolist(), positions.tolist()) == result[0]
        for layer in range(22):
            self.ledger.decode_mark(-1, layer)
        self.ledger.decode_commit()
        self.oracle.decode_commit()

    @rule(slot=st.integers(0, 3))
    def release(self, slot: int) -> None:
        if slot in self.oracle.sequences:
            self.oracle.release(slot)
            self.ledger.release(slot)
        else:
            with pytest.raises(KeyError):
                self.ledger.release(slot)

    @invariant()
    def matches_oracle(self) -> None:
        assert self.ledger.capacity() == self.oracle.capacity()
        assert self.ledger.free_list() == self.oracle.free
        for request in self.oracle.sequences:
            assert self.ledger.table(request) == self.oracle.table(request)
            assert self.ledger.length(request) == self.oracle.length(request)


def _pattern(error: Exception) -> str | None:
    return None if isinstance(error, KeyError) else re.escape(str(error))


def _outcome(action) -> Exception | None:
    try:
        action()
    except (ValueError, RuntimeError, KeyError) as error:
        return error
    return None


@pytest.mark.parametrize("blocks", [1, 2, 4, 8])
def test_randomized_operations_match_oracle(blocks: int) -> None:
    run_state_machine_as_test(
        lambda: _LedgerMachine(blocks),
        settings=settings(max_examples=50, stateful_step_count=40, deadline=None, derandomize=True, database=None),
    )


def test_ceil_helper() -> None:
    assert [workloads.blocks_for(n) for n in (1, 16, 17)] == [math.ceil(n / 16) for n in (1, 16, 17)]


def test_marking_a_run_of_layers_at_once_checks_like_one_by_one() -> None:
    ledger = BlockLedger(8)
    ledger.reserve(1, 2)
    ledger.append(1, 5)
    ledger.reserve(2, 2)
    ledger.append(2, 16)
    with pytest.raises(RuntimeError, match="staged append"):
        ledger.decode_mark_layers(0, 22)
    ledger.decode_begin([1, 2])
    with pytest.raises(ValueError, match="in order"):
        ledger.decode_mark_layers(1, 3)
    with pytest.raises(ValueError, match="22 decoder layers"):
        ledger.decode_mark_layers(20, 3)
    ledger.decode_mark_layers(0, 10)
    ledger.decode_check(-1, 10)
    ledger.decode_mark_layers(10, 12)
    ledger.decode_commit()
    assert ledger.length(1) == 6 and ledger.length(2) == 17
