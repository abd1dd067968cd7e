"""The dense TinyLlama math restated in pagedcore_b200.dense, against the reference on the CPU.

On one device the restatement performs the reference's floating-point
operations in the same order, so the prompt logits of the reduced model
(tests/golden/decoder_small.npz, made by the reference's own prefill) match
with zero tolerance.
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest
import torch

from pagedcore_b200.decoder import prefill
from pagedcore_b200.dense import apply_rope
from pagedcore_b200.weights import random_weights
from tests.conftest import ROOT


@pytest.fixture(scope="module")
def small():
    weights = random_weights(5, layers=2, vocab=31, intermediate=32)
    return replace(weights, layers=weights.layers * 11)


@pytest.mark.parametrize("tokens", [1, 15, 16, 17, 49])
def test_prefill_logits_equal_the_reference_bit_for_bit(small, tokens: int) -> None:
    golden = np.load(ROOT / "tests" / "golden" / "decoder_small.npz")
    ids = (torch.arange(tokens)[None] + tokens) % 31
    logits, cache = prefill(ids, small)
    assert np.array_equal(logits[0].float().numpy(), golden[f"prefill_{tokens}"])
    assert len(cache) == 22 and cache[0][0].shape == (1, 4, tokens, 64)


def test_rope_rejects_positions_of_the_wrong_shape() -> None:
    query = torch.zeros(1, 32, 3, 64, dtype=torch.float16)
    key = torch.zeros(1, 4, 3, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="position_ids"):
        apply_rope(query, key, torch.arange(2)[None])
