"""Host-side pieces of bench.py that need no GPU: the peaks it reports against
and the prefill line's CPU baseline (the dense prefill on the host cores)."""

from __future__ import annotations

import json
from dataclasses import replace

import torch

import bench
from pagedcore_b200.weights import random_weights
from tests.conftest import ROOT


def test_peaks_come_from_the_measured_file_when_present() -> None:
    path = ROOT / "MEASURED_PEAKS.json"
    hbm, hbm_kind = bench._peak_hbm()
    tensor, tensor_kind = bench._peak_tensor()
    if path.exists():
        measured = json.loads(path.read_text())
        assert (hbm, hbm_kind) == (float(measured["hbm_gbs"]), "measured")
        assert (tensor, tensor_kind) == (float(measured["bf16_tflops"]), "measured")
    else:
        assert (hbm_kind, tensor_kind) == ("fallback", "fallback")


def test_prefill_cpu_baseline_times_the_dense_prefill_on_a_sample() -> None:
    weights = random_weights(5, layers=2, vocab=31, intermediate=32)
    weights = replace(weights, layers=weights.layers * 11)
    ids = torch.randint(0, 31, (1, 40), generator=torch.Generator().manual_seed(1))
    line = bench._prefill_cpu_baseline(weights, ids, sample_tokens=16, budget_s=0.05)
    assert line["unit"] == "tokens/s" and line["kind"] == "port"
    assert line["value"] > 0 and line["cores"] == torch.get_num_threads()
    assert "first 16 tokens" in line["sample"]
