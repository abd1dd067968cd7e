"""Config 5's churn workload (pagedcore_b200.stress) at a small scale on the GPU.

Requests reserve their whole context, finish at seeded steps and are replaced;
admission is credit-bound.  After many iterations the ledger must still audit
clean, every finished request's blocks must be back, and no kernel may have
flagged an error.
"""

from __future__ import annotations

import pytest

from pagedcore_b200.stress import StressRun
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu


def test_churn_keeps_the_ledger_consistent_and_admits_as_credits_free() -> None:
    run = StressRun(cuda_device(), seed=9, rows=16, context=256, new_prompt=64)
    result = run.run(warmup=20, iterations=150)
    assert result.decode_tokens > 0 and result.prefill_tokens > 0
    assert result.completed > 5 and result.admitted > 5
    counts = run.allocator.capacity()
    assert counts.reserved_blocks <= counts.total_blocks
    # At most as many active rows as the credits allow (each reserves its full context).
    assert len(run.worker.active) <= counts.total_blocks // (256 // 16)
    run.allocator.ledger.audit()
    run.allocator.check_device_errors()
    for request in run.worker.completed:
        assert request.finish_reason is not None
