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


def test_clock_samples_are_kept_only_inside_the_timed_window(monkeypatch) -> None:
    """The sampler runs from before the warm-up; only samples taken between
    begin() and end() (the recording event) reach the report.  A fake NVML
    reports 1965 MHz inside the window and 100 MHz outside it."""
    import sys
    import threading
    import time
    import types

    clock = [100.0]
    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=0,
        NVMLError=Exception,
        nvmlInit=lambda: None,
        nvmlDeviceGetHandleByPciBusId=lambda bus: "gpu",
        nvmlDeviceGetHandleByIndex=lambda index: "gpu",
        nvmlDeviceGetMaxClockInfo=lambda handle, kind: 1965,
        nvmlDeviceGetClockInfo=lambda handle, kind: clock[0],
        nvmlDeviceGetCurrentClocksEventReasons=lambda handle: 0x4,
    )
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    ready, recording, stop = threading.Event(), threading.Event(), threading.Event()
    sent = []
    sink = types.SimpleNamespace(send=sent.append)
    worker = threading.Thread(target=bench._sample_clocks,
                              args=("00000000:01:00.0", 0, 0.001, ready, recording, stop, sink))
    worker.start()
    assert ready.wait(5)
    time.sleep(0.05)  # the warm-up: not kept
    clock[0] = 1965.0
    recording.set()
    time.sleep(0.05)  # the timed region
    recording.clear()
    time.sleep(0.02)  # a read in flight at the clear finishes first
    clock[0] = 100.0
    time.sleep(0.05)
    stop.set()
    worker.join(5)
    samples, max_mhz, error = sent[0]
    assert error is None and max_mhz == 1965.0
    assert samples and all(mhz == 1965.0 and bits == 0x4 for mhz, bits in samples)


def test_decoder_launch_count_follows_the_projection_routing() -> None:
    """The decoder and prefill legs' `gpu_launches` per step: 256 rows (library GEMMs) 5 per
    layer + the final norm; 32 rows adds the tcgen05 linear layer's 4 per layer
    + the LM head and a Q/K/V split-sum per layer (the launch list of a 32-row
    step, two steps of 448 launches of which 4 are ATen, gives 222); one row
    adds the matrix-vector kernel's 4 per layer + the LM head."""
    assert bench._step_launches(256) == 22 * 5 + 1
    assert bench._step_launches(32) == 222
    assert bench._step_launches(1) == 22 * 5 + 1 + 22 * 4 + 1
