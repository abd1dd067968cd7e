"""Benchmark of the paged KV-cache hot path on B200.

One step = one batched one-token decode step of the KV path over all 22
layers for the rank's 256 sequences (contexts U[1, 2048 - room for the run's appends], tables
fragmented by allocator churn): staged append in the C++ ledger, then per
layer the fused K/Q-RoPE + KV scatter kernel and the split-K GQA decode
attention (+ combine), then the commit.  The dense TinyLlama GEMMs around it
are not part of this path.  Sequences shard across GPUs with no collective
(weak scaling: every rank owns 256 sequences and its own pool).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`value` is decode tokens/s over all ranks with inputs resident in HBM;
`e2e` is the same through the public API with host (pinned) inputs copied in
and attention outputs copied out inside the timed region; `roofline` is the
decode attention (split + combine launches) against the measured HBM copy
bandwidth; `cpu_baseline` is the oracle port of the reference's CPU path on a
bounded sample.  `--impl reference` times that CPU path alone on all host
cores (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged decode-attn HBM GB/s (% of peak) and decode tokens/s at 1/2/4/8 B200"
SEQUENCES = 256  # per GPU (config 4); --sequences overrides it for small profiling cases
LAYERS = 22
CALIBRATION_STEPS = 8  # staged steps in which KVAllocator(balance="measured") learns its piece weights
FALLBACK_HBM_GBS = 6650.0
FALLBACK_TENSOR_TFLOPS = 1590.0
PREFILL_DRAM_BYTES_2047 = 10_529_280  # prefill_tc_kernel, one launch, ncu (read 10.53 MB, write 0)
# DRAM bytes (ncu dram__bytes_read.sum + dram__bytes_write.sum) of one fused
# decode-layer launch over its algorithmic bytes, from one capture of the
# config 4 step; the committed ncu summary of decode_kernel gives the command.
DECODE_TRAFFIC_PER_ALGORITHMIC_BYTE = 1.013


# ---------------------------------------------------------------------------
# CPU path: the oracle port of the reference (bench's CPU-baseline leg).
# ---------------------------------------------------------------------------
def oracle_decode_rows(lengths: list[int], num_blocks: int, steps: int, warmup: int, seed: int) -> float:
    """Seconds for `steps` decode steps of the reference algorithm over `lengths` rows.

    Follows kv_cache.py (staged append with full re-validation on every
    call), dense.apply_rope and attention.paged_attention's page loop, via the
    oracle restatement, on a pool of `num_blocks` blocks.
    """
    from oracle import attention as oracle_attention
    from oracle import kv_write, rope
    from oracle.allocator import OracleAllocator
    from pagedcore_b200 import workloads

    table = rope.cos_sin_table()
    allocator = OracleAllocator(num_blocks, audit=True)
    pool = np.empty((22, 2, num_blocks, 16, 4, 64), dtype=np.float16)
    pattern = workloads.normal_f16(workloads.rng(seed, 9), (22, 16, 4, 64))
    rows = list(range(len(lengths)))
    for row, length in zip(rows, lengths):
        allocator.create(row, workloads.blocks_for(length + steps + warmup))
        slots = np.asarray(allocator.append(row, length))
        for start in range(0, length, 16):
            part = slots[start : start + 16]
            kv_write.write_rows(pool, 0, pattern[:, : len(part)], pattern[:, : len(part)], part)
    q, k, v = workloads.decode_step_inputs(seed, len(rows), 0)
    elapsed = 0.0
    for step in range(warmup + steps):
        begin = time.perf_counter()
        slots, positions = allocator.decode_begin(tuple(rows))
        slots, positions = np.asarray(slots), np.asarray(positions)
        for layer in range(LAYERS):
            q_rot = rope.rotate(q[layer][None], positions, table)[0]
            kv_write.append_rotated(pool, k[layer][None], v[layer][None], slots, positions, table, layer_begin=layer)
            for row in rows:
                blocks, length = allocator.view(row)
                oracle_attention.paged_attention(pool, layer, q_rot[row], blocks, length)
        allocator.decode_commit()
        if step >= warmup:
            elapsed += time.perf_counter() - begin
    return elapsed


def _reference_worker(args: tuple) -> float:
    lengths, num_blocks, steps, warmup, seed = args
    from threadpoolctl import threadpool_limits

    with threadpool_limits(1):
        return oracle_decode_rows(lengths, num_blocks, steps, warmup, seed)


def run_reference_arm(args: argparse.Namespace) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import multiprocessing as mp

    from pagedcore_b200 import workloads

    cores = os.cpu_count() or 1
    case = workloads.decode_case(seed=4, batch=SEQUENCES, steps=args.warmup + args.steps)
    # A bounded sample of the workload: `sample` rows of the rank-0 batch, one
    # row per process, all host cores busy.
    sample = min(SEQUENCES, max(cores, 8))
    lengths = [int(n) for n in case.lengths[:sample]]
    per_worker = [[n] for n in lengths]
    ctx = mp.get_context("spawn")
    start = time.perf_counter()
    with ctx.Pool(processes=min(cores, sample)) as pool:
        times = pool.map(_reference_worker, [(rows, case.num_blocks, args.steps, args.warmup, 4 + i)
                                             for i, rows in enumerate(per_worker)])
    wall = time.perf_counter() - start
    busiest = max(times)
    tokens = sample * args.steps
    value = tokens / busiest
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * busiest / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded)",
        "config": _config(args.gpus),
        "cpu_baseline": {
            "value": value,
            "unit": "tokens/s",
            "cores": min(cores, sample),
            "kind": "port",
            "sample": f"{sample} of {SEQUENCES} rows (one per process), {args.steps} timed decode steps x 22 layers, "
                      f"oracle restatement of the reference CPU path, full ledger re-validation per call; "
                      f"wall {wall:.1f}s incl. setup",
        },
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU path.
# ---------------------------------------------------------------------------
def _config(n_gpus: int) -> dict:
    return {
        "workload": "BASELINE config 4, KV hot path: 256 sequences per GPU, contexts U[1, 2048 - room for the "
                    "run's appends], churned block tables; one step = staged append + 22 fused decode-layer launches (Q/K RoPE, "
                    "new-token KV write, split-K GQA decode attention) + commit; dense GEMMs not included",
        "sequences_per_gpu": SEQUENCES,
        "sharing": "BASELINE config 4 spreads 256 sequences over the N GPUs; this line keeps 256 per GPU so "
                   "per-GPU work is fixed as N grows (weak scaling); --sequences 256/N gives the shared-batch point",
        "layers": LAYERS,
        "heads": "32 query / 4 KV, head_dim 64, block 16",
        "l2": "inputs larger than L2: each attention launch streams ~0.25 GB of K/V (L2 is 126 MB)",
        "parallelism": f"dp{n_gpus} (independent sequences, one KV pool per GPU, no collective)",
        "pieces": "one per CTA slot, cut to balance blocks + row switches, weighted by each slot's measured speed "
                  f"(KVAllocator balance='measured', learnt in {CALIBRATION_STEPS} untimed setup steps, then frozen)",
        "launch": "each step's 22 decode-layer launches (split + combine) replayed as CUDA graphs (DecodeStepGraph), "
                  "captured during setup",
    }


def _peak_hbm() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def _peak_tensor() -> tuple[float, str]:
    """Dense FP16/BF16 tensor peak in TFLOP/s (the burst figure: the kernel is timed alone)."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["bf16_tflops"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_TENSOR_TFLOPS, "fallback"


def _bind_host_cores(device: int) -> str:
    """Run this rank on the host cores NVML reports as closest to its GPU.

    Pinned host buffers allocated afterwards then sit in that NUMA node's
    memory, so the e2e copies do not cross sockets.  Read-only NVML queries.
    """
    try:
        import pynvml

        pynvml.nvmlInit()
        handle = _nvml_handle(pynvml, device)
        words = pynvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        cores = {64 * w + b for w, mask in enumerate(words) for b in range(64) if mask >> b & 1}
        cores &= set(range(os.cpu_count()))
        if not cores:
            return "unbound (NVML reported no cores)"
        os.sched_setaffinity(0, cores)
        return f"{len(cores)} cores local to GPU {device}"
    except Exception as error:  # noqa: BLE001 - binding is an optimisation, never required
        return f"unbound ({error})"


def _nvml_handle(pynvml, device: int):
    """NVML handle of CUDA device `device` (matched by PCI bus id when torch reports it)."""
    import torch

    props = torch.cuda.get_device_properties(device)
    bus = getattr(props, "pci_bus_id", None)
    if bus is not None:
        domain = getattr(props, "pci_domain_id", 0)
        slot = getattr(props, "pci_device_id", 0)
        try:
            return pynvml.nvmlDeviceGetHandleByPciBusId(f"{domain:08x}:{bus:02x}:{slot:02x}.0")
        except pynvml.NVMLError:
            pass
    return pynvml.nvmlDeviceGetHandleByIndex(device)


def _sample_clocks(bus_id: str | None, index: int, period: float, ready, recording, stop, sink) -> None:
    """Child process: NVML SM clock and throttle reasons every `period` s while `recording`, until `stop`."""
    samples, max_mhz, error = [], None, None
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus_id) if bus_id else pynvml.nvmlDeviceGetHandleByIndex(index)
        except pynvml.NVMLError:
            handle = pynvml.nvmlDeviceGetHandleByIndex(index)
        max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))
        # First calls can be slow: make them before the timed region starts.
        pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
        pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
        ready.set()
        while not stop.is_set():
            if recording.wait(period):
                samples.append((float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)),
                                int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle))))
                stop.wait(period)
    except Exception as exc:  # noqa: BLE001 - clocks are reported, never required
        error = f"NVML unavailable: {exc}"
        ready.set()
    sink.send((samples, max_mhz, error))


class ClockSampler:
    """SM clock and throttle-reason samples (NVML, read-only) every 2 ms of the timed region.

    Sampled in a separate (spawned) process, so the sampling never competes
    with the launching thread for the interpreter lock.  The process starts
    (about 0.15 s, the GPU idle) when the context is entered, which a leg does
    before its warm-up, so the timed steps follow the warm-up without a gap;
    only samples between ``begin()`` and ``end()`` (the timed regions) are kept.
    """

    # NVML clock-event reason bits.
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}
    PERIOD = 0.002

    def __init__(self, device: int) -> None:
        self.device = device
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.error = None
        self._child = None

    def __enter__(self) -> "ClockSampler":
        import multiprocessing as mp

        import torch

        props = torch.cuda.get_device_properties(self.device)
        bus = getattr(props, "pci_bus_id", None)
        bus_id = None if bus is None else (f"{getattr(props, 'pci_domain_id', 0):08x}:{bus:02x}:"
                                           f"{getattr(props, 'pci_device_id', 0):02x}.0")
        ctx = mp.get_context("spawn")
        self._ready, self._recording, self._stop = ctx.Event(), ctx.Event(), ctx.Event()
        self._receive, send = ctx.Pipe(duplex=False)
        self._child = ctx.Process(target=_sample_clocks,
                                  args=(bus_id, self.device, self.PERIOD, self._ready, self._recording, self._stop,
                                        send), daemon=True)
        self._child.start()
        if not self._ready.wait(timeout=120):
            self.error = "clock sampler did not start"
        return self

    def begin(self) -> None:
        """A timed region starts: keep samples from now on."""
        if self._child is not None:
            self._recording.set()

    def end(self) -> None:
        """The timed region has ended (after its closing synchronisation)."""
        if self._child is not None:
            self._recording.clear()

    def __exit__(self, *exc) -> None:
        if self._child is None:
            return
        self._recording.clear()
        self._stop.set()
        if self._receive.poll(30):
            self.samples, self.max_mhz, error = self._receive.recv()
            self.error = self.error or error
        else:
            self.error = self.error or "clock sampler returned nothing"
        self._child.join(timeout=10)

    def summary(self) -> dict:
        reasons = set()
        for _, bits in self.samples:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        summary = {
            "sm_mhz": statistics.median(mhz for mhz, _ in self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "samples": len(self.samples),
            "reasons": sorted(reasons),
            "source": "NVML every 2 ms during the timed region, in a separate process",
        }
        if self.error:
            summary["error"] = self.error
        return summary


def kv_leg(args: argparse.Namespace, device, rank: int, world: int, local_rank: int, sequences: int,
           repeats: int) -> dict:
    """Config 4's KV path for `sequences` sequences on this rank (all ranks take part).

    One step = staged append + 22 fused decode-layer launches (Q/K RoPE,
    new-token KV write, split-K GQA attention + combine) + commit, replayed as
    CUDA graphs.  Returns the timed regions (max over ranks), the e2e time
    through the public API with pinned host inputs and outputs, and the
    algorithmic bytes of one layer launch.
    """
    import torch
    import torch.distributed as dist

    from pagedcore_b200 import workloads
    from pagedcore_b200.engine_types import KVReservation, RequestId
    from pagedcore_b200.graph import DecodeStepGraph
    from pagedcore_b200.kv_cache import KVAllocator

    seed = 4 + 1000 * rank
    # Room for every append of the run: calibration, warm-up, plan, the timed
    # regions, e2e warm-up and e2e steps.
    room = CALIBRATION_STEPS + args.warmup + 1 + (repeats + 1) * args.steps + 2 + 4
    case = workloads.decode_case(seed=seed, batch=sequences, steps=room)
    context_high = 2048 - room
    pool = torch.empty((22, 2, case.num_blocks, 16, 4, 64), dtype=torch.float16, device=device)
    allocator = KVAllocator(pool, validation="incremental", balance="measured")

    # Fragment the free list with seeded churn, then prefill the batch.
    generator = torch.Generator(device=device).manual_seed(seed)
    zero = torch.zeros(22, 64, 4, 64, dtype=torch.float16, device=device)
    for op in case.churn:
        rid = RequestId(f"churn{op.request}")
        if op.kind == "create":
            allocator.create(KVReservation(rid, op.credits))
            allocator.append(rid, zero[:, : op.tokens], zero[:, : op.tokens])
        else:
            allocator.release_all(rid)
    requests = tuple(RequestId(f"seq{i}") for i in range(sequences))
    for request, length, credits in zip(requests, case.lengths.tolist(), case.credits.tolist()):
        allocator.create(KVReservation(request, credits))
        key = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        value = torch.randn(22, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        allocator.append(request, key, value, rotate=True)
    torch.cuda.synchronize(device)

    def inputs(index: int) -> tuple[torch.Tensor, ...]:
        g = torch.Generator(device=device).manual_seed(seed * 7919 + index)
        q = torch.randn(22, sequences, 32, 64, dtype=torch.float16, device=device, generator=g)
        k = torch.randn(22, sequences, 4, 64, dtype=torch.float16, device=device, generator=g)
        v = torch.randn(22, sequences, 4, 64, dtype=torch.float16, device=device, generator=g)
        return q, k, v

    device_inputs = [inputs(i) for i in range(2)]
    out = torch.empty(22, sequences, 32, 64, dtype=torch.float16, device=device)
    stream = torch.cuda.current_stream(device)

    # Each step's 22 fused decode-layer launches (+ combines) replay as one CUDA
    # graph per (upload buffer, input buffer set); warm-up captures them all.
    engine = DecodeStepGraph(allocator, requests)

    def step(q, k, v, dst=None) -> None:
        engine.step(q, k, v, out if dst is None else dst)

    def barrier() -> None:
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(device)

    # Setup, untimed: the allocator learns each CTA slot's speed over its first
    # staged steps and then freezes the piece weights.  The clock sampler starts
    # first, so the timed regions follow the warm-up without an idle gap.
    with ClockSampler(local_rank) as clocks:
        for i in range(CALIBRATION_STEPS):
            step(*device_inputs[i % 2])
        for i in range(args.warmup):
            step(*device_inputs[i % 2])
        allocator.check_device_errors()

        # Algorithmic bytes of one fused decode-layer launch, from the staged
        # batch: K/V streamed (1024 B per cached token, the new one included),
        # block-table entries, Q in / attention out (4 KiB each), the new token's
        # K/V in (1 KiB) and written to the pool (1 KiB), lengths and prefix.  The
        # split partials are not counted: they are a by-product of the split, not
        # bytes the operation needs.
        plan_info = {}

        def layer_bytes() -> float:
            with allocator.append_decode(requests):
                batch = allocator.staged_decode_batch()
                for layer in range(LAYERS):
                    allocator.decode_layer(layer, *(x[layer] for x in device_inputs[0]), out=out[layer])
            big, tail = batch.plan.pieces()
            plan_info.update(grid=batch.plan.grid, blocks_per_cta=batch.plan.blocks_per_cta, big_ctas=big,
                             tail_blocks=tail, total_blocks=batch.total_blocks)
            lengths = batch.host_lengths.astype(np.int64)
            blocks = (lengths + 15) // 16
            per_row = 1024 * lengths + 4 * blocks + 2 * 4096 + 2 * 1024 + 8
            return float(per_row.sum())

        # One extra staged step (its tokens are real appends) measures the plan.
        layer_bytes_per_launch = layer_bytes()

        # No events inside the timed region: an event recorded between two layer
        # launches delays the next launch by several microseconds, so the layer
        # time below is the timed region's time over its 22 * K layer launches
        # (split + combine + the gaps between them, plus each step's table upload).
        # The timed region is repeated `repeats` times, each exactly `steps` steps
        # bracketed by a barrier and a device synchronisation; `value` is the
        # median region, the others give the spread.
        regions = []
        for _ in range(repeats):
            barrier()
            clocks.begin()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push("timed")
            start.record(stream)
            for i in range(args.steps):
                step(*device_inputs[i % 2])
            end.record(stream)
            torch.cuda.nvtx.range_pop()
            barrier()
            clocks.end()
            regions.append(start.elapsed_time(end))
    allocator.check_device_errors()

    # End to end through the public API with host buffers: every step copies
    # its Q/K/V in from pinned host memory and its attention outputs back out.
    # The copies run on two copy streams, double-buffered by step, so step
    # i+1's inputs load and step i's outputs drain while layers compute.
    host_inputs = [tuple(t.cpu().pin_memory() for t in device_inputs[i]) for i in range(2)]
    staging = [[torch.empty_like(t) for t in device_inputs[0]] for _ in range(2)]
    outs = [torch.empty_like(out) for _ in range(2)]
    host_out = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    h2d_bytes = sum(t.numel() * t.element_size() for t in host_inputs[0])
    d2h_bytes = host_out[0].numel() * host_out[0].element_size()
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def e2e_steps(count: int) -> None:
        loaded = [torch.cuda.Event() for _ in range(2)]    # staging[b] holds its step's inputs
        consumed = [torch.cuda.Event() for _ in range(2)]  # the step reading staging[b] is done
        computed = [torch.cuda.Event() for _ in range(2)]  # outs[b] holds its step's outputs
        drained = [torch.cuda.Event() for _ in range(2)]   # outs[b] is copied out

        def load(i: int) -> None:
            b = i % 2
            copy_in.wait_event(consumed[b])
            with torch.cuda.stream(copy_in):
                for dst, src in zip(staging[b], host_inputs[i % 2]):
                    dst.copy_(src, non_blocking=True)
            loaded[b].record(copy_in)

        copy_in.wait_stream(stream)  # the first copy starts after the timer does
        load(0)
        for i in range(count):
            b = i % 2
            if i + 1 < count:
                load(i + 1)
            stream.wait_event(loaded[b])
            stream.wait_event(drained[b])
            step(*staging[b], dst=outs[b])
            consumed[b].record(stream)
            computed[b].record(stream)
            copy_out.wait_event(computed[b])
            with torch.cuda.stream(copy_out):
                host_out[b].copy_(outs[b], non_blocking=True)
            drained[b].record(copy_out)
        for b in range(2):
            stream.wait_event(drained[b])

    e2e_steps(2)
    barrier()
    e2e_start, e2e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_start.record(stream)
    e2e_steps(args.steps)
    e2e_end.record(stream)
    barrier()
    e2e_ms = e2e_start.elapsed_time(e2e_end)
    print(f"rank {rank}: {sequences} sequences, timed regions {[round(r, 2) for r in regions]} ms, "
          f"e2e {e2e_ms:.2f} ms", file=sys.stderr, flush=True)
    allocator.check_device_errors()

    times = torch.tensor([*regions, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)  # per region: the slowest rank
    *regions, e2e_ms = times.tolist()
    del engine
    return {"regions": regions, "e2e_ms": e2e_ms, "layer_bytes": layer_bytes_per_launch, "plan": plan_info,
            "h2d_bytes": h2d_bytes, "d2h_bytes": d2h_bytes, "context_high": context_high, "clocks": clocks.summary(),
            "case": case, "seed": seed}



def run_gpu_arm(args: argparse.Namespace) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    affinity = _bind_host_cores(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)

    repeats = args.repeats
    leg = kv_leg(args, device, rank, world, local_rank, SEQUENCES, repeats)
    regions, e2e_ms, layer_bytes_per_launch, plan_info = leg["regions"], leg["e2e_ms"], leg["layer_bytes"], leg["plan"]
    h2d_bytes, d2h_bytes, context_high, case, seed = (leg[k] for k in ("h2d_bytes", "d2h_bytes", "context_high",
                                                                       "case", "seed"))
    elapsed_ms = statistics.median(regions)
    layer_ms = elapsed_ms
    # BASELINE config 4 spreads 256 sequences over the N GPUs: at N > 1 the
    # shared-batch point, 256 / N sequences per GPU, is measured too.
    shared = None
    if world > 1 and not args.no_shared:
        shared = kv_leg(args, device, rank, world, local_rank, max(1, 256 // world), 1)

    # The whole decoder on the same per-GPU batch size, with the token gather
    # across ranks (its own pool, weights and batch; all ranks take part).
    decoder = None if args.no_decoder else decoder_leg(args, device, rank, world, local_rank)

    if rank == 0:
        tokens = world * SEQUENCES * args.steps
        value = tokens / (elapsed_ms / 1000.0)
        peak, peak_kind = _peak_hbm()
        launch_ms = layer_ms / (args.steps * LAYERS)
        achieved = layer_bytes_per_launch / (launch_ms / 1000.0) / 1e9
        traffic = DECODE_TRAFFIC_PER_ALGORITHMIC_BYTE * layer_bytes_per_launch
        launches_per_step = LAYERS * (2 if plan_info["grid"] > 1 else 1)  # split + combine
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": f"synthetic (seeded K/V/Q ~N(0,1), contexts U[1, {context_high}]); the reference publishes "
                    "no inputs",
            "config": _config(world),
            "attn_hbm_gbs": achieved,
            "attn_frac_of_peak": achieved / peak,
            "roofline": {
                "bound": "hbm",
                "kernel": "fused decode layer: decode_kernel<4,true> (Q/K RoPE, new-token KV write, split-K GQA "
                          "attention) + decode_combine_kernel (programmatic dependent launch), per layer",
                "achieved": achieved,
                "peak": peak,
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "unit": "GB/s",
                "frac": achieved / peak,
                "algorithmic_bytes_per_launch": layer_bytes_per_launch,
                "plan": plan_info,
                "avg_launch_ms": launch_ms,
                "avg_launch_source": "CUDA events around the timed region / (steps x 22 layer launches); "
                                     "includes the combine, the gaps between launches and each step's table upload",
                "traffic": traffic,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one decode-layer launch "
                                  "over its algorithmic bytes (1.013, one capture of this step), times this run's "
                                  "algorithmic bytes",
            },
            "repeats": {
                "regions": args.repeats,
                "ms_per_step": [r / args.steps for r in regions],
                "median_ms_per_step": elapsed_ms / args.steps,
                "spread": (max(regions) - min(regions)) / elapsed_ms,
                "note": "each region exactly `steps` steps between barriers; value is the median region",
            },
            "e2e": {
                "value": tokens / (e2e_ms / 1000.0),
                "unit": "tokens/s",
                "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": d2h_bytes,
                "path": "pinned host Q/K/V -> device and attention outputs -> pinned host every step, on two "
                        "copy streams overlapped with the neighbouring steps; DecodeStepGraph.step "
                        "(KVAllocator.append_decode and the 22 decode layers replayed as one CUDA graph)",
            },
            "gpu_launches": args.steps * launches_per_step,
            "clocks": leg["clocks"],
            "host_affinity": affinity,
        }
        if shared is not None:
            shared_ms = statistics.median(shared["regions"])
            shared_rows = max(1, 256 // world)
            shared_launch_ms = shared_ms / (args.steps * LAYERS)
            line["shared_batch"] = {
                "what": f"BASELINE config 4's own split: 256 sequences over {world} GPUs, {shared_rows} per GPU",
                "value": world * shared_rows * args.steps / (shared_ms / 1000.0),
                "unit": "tokens/s",
                "ms_per_step": shared_ms / args.steps,
                "attn_hbm_gbs": shared["layer_bytes"] / (shared_launch_ms / 1000.0) / 1e9,
                "attn_frac_of_peak": shared["layer_bytes"] / (shared_launch_ms / 1000.0) / 1e9 / peak,
            }
        if decoder is not None:
            line["decoder"] = {
                "what": "the same per-GPU batch size (256 sequences) through the whole TinyLlama decoder: greedy "
                        "decode replayed as one CUDA graph per step, token ids all-gathered over NCCL at N > 1",
                **decoder,
            }
            if world == 1 and not args.no_cpu_baseline:
                line["decoder"]["cpu_baseline"] = _decoder_cpu_baseline(seed=4, budget_s=10.0)
        if world == 1 and not args.no_cpu_baseline:
            from threadpoolctl import threadpool_limits

            sample_rows = [int(n) for n in case.lengths[:192]]  # about 10 s of one core
            with threadpool_limits(1):
                seconds = oracle_decode_rows(sample_rows, case.num_blocks, steps=2, warmup=0, seed=seed)
            line["cpu_baseline"] = {
                "value": len(sample_rows) * 2 / seconds,
                "unit": "tokens/s",
                "cores": 1,
                "kind": "port",
                "sample": f"{len(sample_rows)} of the {SEQUENCES} rows x 2 decode steps x 22 layers of the same "
                          f"workload, one thread, oracle restatement of the reference CPU path ({seconds:.1f}s)",
            }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def run_stress_arm(args: argparse.Namespace) -> None:
    """BASELINE config 5 (pagedcore_b200.stress): sustained decode under allocator churn."""
    import torch
    import torch.distributed as dist

    from pagedcore_b200.stress import NEW_PROMPT, ROWS, StressRun, pool_blocks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    _bind_host_cores(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    run = StressRun(device, seed=5 + 1000 * rank)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
    with ClockSampler(local_rank) as clocks:
        run.warm(args.stress_warmup)
        clocks.begin()
        result = run.run(0, args.stress_iterations)
        clocks.end()
    totals = torch.tensor([result.seconds, result.decode_tokens, result.attention_bytes], dtype=torch.float64,
                          device=device)
    if world > 1:
        seconds = totals[:1].clone()
        dist.all_reduce(seconds, op=dist.ReduceOp.MAX)
        dist.all_reduce(totals, op=dist.ReduceOp.SUM)
        totals[0] = seconds[0]
    seconds, tokens, attention_bytes = totals.tolist()
    if rank == 0:
        peak, peak_kind = _peak_hbm()
        line = {
            "metric": "sustained decode tokens/s under allocator churn (BASELINE config 5)",
            "value": tokens / seconds,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.stress_iterations,
            "warmup": args.stress_warmup,
            "ms_per_step": 1000.0 * seconds / args.stress_iterations,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded prompts, finish steps and K/V/Q)",
            "config": {
                "workload": f"config 5 per GPU: {ROWS} sequences reserving full 2048-token contexts, pool of "
                            f"{pool_blocks()} blocks (90 % of their need), each finishing at a seeded step and "
                            f"replaced by a {NEW_PROMPT}-token prompt; strict FIFO credit admission, one prefill "
                            "write per iteration, one fused decode step per iteration for every active sequence",
                "launch": "each decode step's 22 decode-layer launches replayed as one CUDA graph (DecodeStepGraph "
                          f"with {ROWS} rows: padded step tables, so one graph serves every batch)",
                "warmup": f"{args.stress_warmup} untimed iterations before the timed ones",
                "parallelism": f"dp{world} (independent sequences, one KV pool per GPU)",
            },
            "attn_gbs": attention_bytes / seconds / 1e9,
            "attn_frac_of_peak": attention_bytes / seconds / 1e9 / peak,
            "peak_kind": peak_kind,
            "rank0": {"decode_tokens": result.decode_tokens, "prefill_tokens": result.prefill_tokens,
                      "admitted": result.admitted, "completed": result.completed,
                      "active_mean": result.active_mean},
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def run_append_arm(args: argparse.Namespace) -> None:
    """BASELINE config 2(a): prompt K/V appends with fused K-RoPE after allocator churn.

    A 4096-block pool fragmented by the seeded 10k-op churn, then 8 prompts of
    U[1, 2047] tokens, written by one batched append.  `value` times that
    append's kernel (`pkv_append_kv`, K rotated at its positions, K and V
    scattered through the prompts' slots, one launch for all 8) with K/V
    resident in HBM; `e2e` times the public `KVAllocator.append_many(...,
    rotate=True)` with the prompts' K/V copied in from pinned host memory,
    the requests released and re-created around it, and the device error
    flag read back per step.
    """
    import torch
    import torch.distributed as dist

    from pagedcore_b200 import kernels, workloads
    from pagedcore_b200.engine_types import KVReservation, RequestId
    from pagedcore_b200.kv_cache import KVAllocator

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    host_affinity = _bind_host_cores(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    seed = 2 + 1000 * rank
    case = workloads.append_case(seed=seed)
    pool = torch.empty((LAYERS, 2, case.num_blocks, 16, 4, 64), dtype=torch.float16, device=device)
    allocator = KVAllocator(pool, validation="incremental")
    fill = torch.zeros(LAYERS, 128, 4, 64, dtype=torch.float16, device=device)  # churn data is irrelevant
    for op in case.churn:
        request = RequestId(f"churn{op.request}")
        if op.kind == "create":
            allocator.create(KVReservation(request, op.credits))
            allocator.append(request, fill[:, : op.tokens], fill[:, : op.tokens])
        else:
            allocator.release_all(request)
    # The 8 prompts are written by one batched append (KVAllocator.append_many):
    # their tokens concatenated in request order, one kernel launch.
    requests = [RequestId(f"prompt{prompt.request}") for prompt in case.prompts]
    credits = [prompt.credits for prompt in case.prompts]
    counts = [prompt.key.shape[1] for prompt in case.prompts]
    key_host = torch.from_numpy(np.concatenate([p.key for p in case.prompts], axis=1)).pin_memory()
    value_host = torch.from_numpy(np.concatenate([p.value for p in case.prompts], axis=1)).pin_memory()
    key, value = key_host.to(device), value_host.to(device)
    for request, credit in zip(requests, credits, strict=True):
        allocator.create(KVReservation(request, credit))
    allocator.append_many(requests, key, value, counts, rotate=True)
    slots, positions = [], []
    for request, count in zip(requests, counts, strict=True):
        table = np.asarray(allocator.block_table(request), dtype=np.int64)
        position = np.arange(count, dtype=np.int32)
        slots.append((table[position // 16] * 16 + position % 16).astype(np.int32))
        positions.append(position)
    slots_device = torch.from_numpy(np.concatenate(slots)).to(device)
    positions_device = torch.from_numpy(np.concatenate(positions)).to(device)
    total_tokens = sum(counts)
    # Algorithmic bytes: per (layer, token) K and V read and written (4 x 512 B);
    # per token its slot and position and one RoPE row (32 cos + 32 sin FP16).
    step_bytes = total_tokens * (LAYERS * 4 * 512 + 8 + 128)
    stream = torch.cuda.current_stream(device)

    def kernel_step() -> None:
        kernels.append_kv(pool, key, value, slots_device, layer_begin=0, error_flag=allocator._error,
                          positions=positions_device, rope_table=allocator._rope)

    with ClockSampler(local_rank) as clocks:
        for _ in range(args.warmup):
            kernel_step()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.begin()
        torch.cuda.nvtx.range_push("timed")
        start.record(stream)
        for _ in range(args.steps):
            kernel_step()
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(device)
        clocks.end()
    kernel_ms = start.elapsed_time(end) / args.steps
    allocator.check_device_errors()

    # End to end through the public API, K/V from pinned host memory.
    key_staging, value_staging = torch.empty_like(key), torch.empty_like(value)

    def public_step() -> None:
        for request in requests:
            allocator.release_all(request)
        for request, credit in zip(requests, credits, strict=True):
            allocator.create(KVReservation(request, credit))
        key_staging.copy_(key_host, non_blocking=True)
        value_staging.copy_(value_host, non_blocking=True)
        allocator.append_many(requests, key_staging, value_staging, counts, rotate=True)
        allocator.check_device_errors()  # the step's device-to-host read

    for _ in range(args.warmup):
        public_step()
    torch.cuda.synchronize(device)
    start.record(stream)
    for _ in range(args.steps):
        public_step()
    end.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = start.elapsed_time(end) / args.steps

    times = torch.tensor([kernel_ms, e2e_ms], dtype=torch.float64, device=device)
    counts = torch.tensor([total_tokens], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.all_reduce(counts, op=dist.ReduceOp.SUM)
    kernel_ms, e2e_ms = times.tolist()
    all_tokens = counts.item()
    if rank == 0:
        peak, peak_kind = _peak_hbm()
        achieved = step_bytes / (kernel_ms / 1000.0) / 1e9
        line = {
            "metric": "prompt KV append tokens/s with fused K-RoPE (BASELINE config 2a)",
            "value": all_tokens / (kernel_ms / 1000.0),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": kernel_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded K/V ~N(0,1), prompt lengths U[1, 2047]); the reference publishes no inputs",
            "config": {
                "workload": f"config 2a per GPU: pool of {case.num_blocks} blocks after a seeded "
                            f"{len(case.churn)}-op alloc/free churn, {len(requests)} prompts ({total_tokens} tokens "
                            "on rank 0) appended with K rotated at positions 0..T-1; one step = all prompts in one "
                            "batched append (KVAllocator.append_many: one kernel launch)",
                "l2": f"inputs larger than L2: each step reads {2 * LAYERS * total_tokens * 512 / 1e6:.0f} MB of "
                      "K/V (L2 is 126 MB)",
                "parallelism": f"dp{world} (independent prompts, one KV pool per GPU, no collective)",
                "launch": "one append launch per step (value); e2e makes the public calls",
            },
            "roofline": {
                "bound": "hbm",
                "kernel": "append_kv_kernel (K-RoPE + K/V scatter through slot ids)",
                "achieved": achieved,
                "peak": peak,
                "peak_kind": peak_kind,
                "unit": "GB/s",
                "frac": achieved / peak,
                "algorithmic_bytes_per_step": step_bytes,
                "avg_launch_ms": kernel_ms,
                "traffic": None,
                "traffic_note": "ncu per launch: reads 1.004 x the K/V input (read once), writes 103-108 of the "
                                "152 MB written (the rest still dirty in L2 at the launch's end)",
            },
            "e2e": {
                "value": all_tokens / (e2e_ms / 1000.0),
                "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * LAYERS * total_tokens * 512 + 8 * total_tokens,
                "d2h_bytes_per_step": 4,
                "path": "KVAllocator.release_all + create per prompt, then append_many(rotate=True) of the 8 "
                        "prompts, K/V copied from pinned host memory each step, error flag read back per step",
            },
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
            "host_affinity": host_affinity,
        }
        if world == 1 and not args.no_cpu_baseline:
            from oracle import kv_write, rope

            table = rope.cos_sin_table()
            host_pool = np.zeros((LAYERS, 2, case.num_blocks, 16, 4, 64), dtype=np.float16)
            sample = case.prompts[:2]
            begin = time.perf_counter()
            repeats = 0
            while time.perf_counter() - begin < 10.0:
                for prompt, prompt_slots in zip(sample, slots, strict=False):
                    tokens = prompt.key.shape[1]
                    kv_write.append_rotated(host_pool, prompt.key, prompt.value, prompt_slots,
                                            np.arange(tokens, dtype=np.int32), table)
                repeats += 1
            seconds = time.perf_counter() - begin
            sample_tokens = sum(p.key.shape[1] for p in sample)
            line["cpu_baseline"] = {
                "value": repeats * sample_tokens / seconds,
                "unit": "tokens/s",
                "cores": 1,
                "kind": "port",
                "sample": f"the first 2 prompts ({sample_tokens} tokens) appended {repeats} times, one thread, "
                          f"oracle restatement of apply_rope + the pool copy ({seconds:.1f}s)",
            }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def decoder_leg(args: argparse.Namespace, device, rank: int, world: int, local_rank: int) -> dict | None:
    """Config 4 through the whole TinyLlama decoder: sharded greedy decode with the token gather.

    Random-init TinyLlama weights (the reference publishes no checkpoint
    here), 256 sequences per GPU (rank r owns batch positions i % N == r of
    the 256 N-row batch) with contexts U[1, 2048 - room] of seeded K/V.  One
    step = embedding, 22 x (norm, fused Q/K/V GEMM, fused decode layer,
    output projection, norm, gate/up GEMM, SwiGLU product, down projection),
    final norm and LM head, replayed as one CUDA graph (``DecoderStepGraph``),
    then each row's greedy token (argmax on the device) and, at N > 1, the
    all-gather of the whole batch's tokens over NCCL (``ShardedGreedyDecoder``,
    ``StepExchange``): the next step's input ids never leave the device.
    `e2e`: the same loop as a serving process runs it, the step's ids copied
    in from pinned host memory and the gathered tokens read back every step.
    Returns the leg's figures on rank 0 (None elsewhere).
    """
    import torch
    import torch.distributed as dist

    from pagedcore_b200 import workloads
    from pagedcore_b200.decoder import BatchedDecoder
    from pagedcore_b200.engine_types import KVReservation, RequestId
    from pagedcore_b200.kv_cache import KVAllocator
    from pagedcore_b200.sharding import ShardedGreedyDecoder, StepExchange, shard
    from pagedcore_b200.weights import random_weights

    seed = 4 + 1000 * rank
    rows = args.sequences
    room = CALIBRATION_STEPS + args.warmup + 2 * args.steps + 4
    lengths = workloads.decode_lengths(seed, rows, high=2048 - room).tolist()
    need = sum(-(-(n + room) // 16) for n in lengths) + 8
    pool = torch.empty((LAYERS, 2, need, 16, 4, 64), dtype=torch.float16, device=device)
    allocator = KVAllocator(pool, validation="incremental", balance="measured")
    batch = tuple(RequestId(f"s{i}") for i in range(rows * world))  # the whole batch, all ranks
    requests = shard(batch, rank, world)
    generator = torch.Generator(device=device).manual_seed(seed)
    for request, length in zip(requests, lengths, strict=True):
        allocator.create(KVReservation(request, -(-(length + room) // 16)))
        kv = torch.randn(LAYERS, length, 4, 64, dtype=torch.float16, device=device, generator=generator)
        allocator.append(request, kv, kv, rotate=True)
    weights = random_weights(seed, device, generator_device=device)
    decoder = BatchedDecoder(weights)
    # Peers are checked in the store every 16th step (a rank's failure is then
    # noticed within 16 steps, or by the process group's timeout): a store
    # round trip per step would hold every host back to the slowest rank's.
    exchange = StepExchange(wait=timedelta(seconds=120), check_every=16) if world > 1 else None
    sharded = ShardedGreedyDecoder(decoder, allocator, batch, exchange)
    first = torch.randint(0, 32000, (rows, 1), device=device, generator=generator)
    stream = torch.cuda.current_stream(device)

    def barrier() -> None:
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(device)

    with ClockSampler(local_rank) as clocks:
        ids = first
        for _ in range(CALIBRATION_STEPS + args.warmup):
            ids, gathered = sharded.step(ids)
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.begin()
        torch.cuda.nvtx.range_push("timed")  # marks the timed launches for an ncu launch list
        start.record(stream)
        for _ in range(args.steps):
            ids, gathered = sharded.step(ids)
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        barrier()
        clocks.end()
    step_ms = start.elapsed_time(end) / args.steps
    allocator.check_device_errors()

    # As a serving loop runs it: this rank's input ids from pinned host memory,
    # the whole batch's tokens read back (and waited for) every step.
    host_all = torch.empty(rows * world, dtype=torch.int64).pin_memory()
    host_in = torch.empty((rows, 1), dtype=torch.int64).pin_memory()
    host_in.copy_(ids.cpu())
    staged = torch.empty_like(ids)
    read = torch.cuda.Event()

    def serve_step() -> None:
        staged.copy_(host_in, non_blocking=True)
        _, tokens = sharded.step(staged)
        host_all.copy_(tokens, non_blocking=True)
        read.record(stream)
        read.synchronize()
        host_in.copy_(host_all[rank::world].view(rows, 1))

    serve_step()
    serve_step()
    barrier()
    e2e_start, e2e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_start.record(stream)
    for _ in range(args.steps):
        serve_step()
    e2e_end.record(stream)
    barrier()
    e2e_ms = e2e_start.elapsed_time(e2e_end) / args.steps
    allocator.check_device_errors()
    times = torch.tensor([step_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    step_ms, e2e_ms = (float(x) for x in times.tolist())
    if rank != 0:
        return None
    # Bytes a step must move: every weight matrix once (the fused Q/K/V and
    # gate/up copies are what the step reads), the embedding rows, and per
    # layer the attention's K/V stream (the cached tokens, the new one
    # included), its block tables, and the new token's K/V written.
    cached = np.array([allocator.cached_length(r) for r in requests], dtype=np.int64)
    weight_bytes = sum(t.numel() * t.element_size() for t in (*decoder.qkv, *decoder.gate_up)) + sum(
        (layer.o_proj.numel() + layer.down_proj.numel() + 2 * layer.input_norm.numel()) * 2
        for layer in weights.layers) + weights.lm_head.numel() * 2
    kv_bytes = LAYERS * float((1024 * cached + 4 * ((cached + 15) // 16) + 1024).sum())
    step_bytes = weight_bytes + kv_bytes + rows * 2048 * 2
    peak, peak_kind = _peak_hbm()
    achieved = step_bytes / (step_ms / 1000.0) / 1e9
    launches = _step_launches(rows)
    return {
        "value": world * rows / (step_ms / 1000.0),
        "unit": "tokens/s",
        "ms_per_step": step_ms,
        "steps": args.steps,
        "sequences_per_gpu": rows,
        "contexts": f"U[1, {2048 - room}]",
        "e2e": {
            "value": world * rows / (e2e_ms / 1000.0),
            "unit": "tokens/s",
            "h2d_bytes_per_step": rows * 8,
            "d2h_bytes_per_step": rows * world * 8,
            "path": "ShardedGreedyDecoder.step with this rank's ids copied from pinned host memory and the "
                    "gathered tokens of the whole batch read back and waited for every step",
        },
        "token_gather": ("NCCL all_gather_into_tensor of int64 next-token ids every step "
                         f"({rows * world * 8} B gathered), peers checked in the store every 16th step")
        if world > 1 else "none at N = 1 (one rank holds the whole batch)",
        "roofline": {
            "bound": "hbm",
            "kernel": "whole decoder step (GEMMs, fused decode layers, norms, argmax, gather)",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            "bytes_per_step": step_bytes,
            "weight_bytes": weight_bytes,
            "attention_bytes": kv_bytes,
            "traffic": None,
        },
        "gpu_launches": args.steps * launches,
        "clocks": clocks.summary(),
    }


def _step_launches(rows: int) -> int:
    """This library's kernel launches in one pass of ``BatchedDecoder.forward`` over ``rows`` rows.

    Per layer five: the two fused residual-add norms, the SwiGLU product and
    the attention's two (a decode step: the decode layer's split and combine;
    a prefill: the K/V write and the causal attention), then the final norm.
    The projections follow ``kernels.linear``'s routing: one row runs this
    library's matrix-vector kernel (four per layer and the LM head), 2 to
    ``TC_MAX_ROWS`` rows its tcgen05 linear layer (the same five launches, plus
    a split-sum launch where the fused Q/K/V or the LM head is split over K;
    the other splits are added by the fused norm and SwiGLU kernels), more
    rows the library GEMM.  Embedding, argmax and the NCCL gather are library
    kernels.
    """
    from pagedcore_b200 import kernels

    launches = LAYERS * 5 + 1
    if rows <= kernels.GEMV_MAX_ROWS:
        launches += 4 * LAYERS + 1
    elif rows <= kernels.TC_MAX_ROWS:
        launches += 4 * LAYERS + 1
        launches += LAYERS * (kernels.linear_splits(rows, 2560, 2048) > 1)
        launches += kernels.linear_splits(rows, 32000, 2048) > 1
    return launches


def run_decoder_arm(args: argparse.Namespace) -> None:
    """Row f1 / config 4 on the whole model: ``decoder_leg`` as its own line."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    host_affinity = _bind_host_cores(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    leg = decoder_leg(args, device, rank, world, local_rank)
    if rank == 0:
        line = {
            "metric": "full TinyLlama decoder greedy decode tokens/s (BASELINE config 4 on the whole model; "
                      "row f1: batched decode step)",
            "value": leg["value"],
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": leg["ms_per_step"],
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (random-init TinyLlama weights N(0, 0.02), seeded K/V caches, random token ids)",
            "config": {
                "workload": f"{args.sequences} sequences per GPU, contexts {leg['contexts']}, one greedy token "
                            "each per step through the whole decoder (22 layers + LM head) replayed as one CUDA "
                            "graph, then the batch's tokens gathered over NCCL (N > 1)",
                "parallelism": f"dp{world} (independent sequences, weights replicated, token ids all-gathered)",
                "l2": "inputs larger than L2: 2.2 GB of weights and ~5.7 GB of K/V per step",
            },
            **{k: leg[k] for k in ("e2e", "roofline", "gpu_launches", "clocks", "token_gather")},
            "host_affinity": host_affinity,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = _decoder_cpu_baseline(seed=4)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def _decoder_cpu_baseline(seed: int, context: int = 1024, budget_s: float = 15.0) -> dict:
    """The reference's one-token decode on the host cores, as a serving CPU would run it.

    PagedCore's decode_paged serves each row with single-row F.linear
    projections and its FP32 page loop (decoder.py:156-199, attention.py:32-53);
    the oracle's contiguous decoder performs the same dense.py ops with FP32
    attention over the row's whole history (decoder.py:138-153), the cost of
    that page loop without the page traversal.  One row with a `context`-token
    seeded cache (the middle of the leg's U[1, 2048 - room] contexts), greedy
    steps repeated for about `budget_s` seconds with all of torch's host
    threads; FP16 weights as the reference keeps them.
    """
    import torch

    from oracle.torch_decoder import ContiguousDecoder
    from pagedcore_b200.weights import random_weights

    weights = random_weights(seed, torch.device("cpu"))
    decoder = ContiguousDecoder(weights)
    generator = torch.Generator().manual_seed(seed)
    decoder.layers = [
        (torch.randn(1, 4, context, 64, dtype=torch.float16, generator=generator),
         torch.randn(1, 4, context, 64, dtype=torch.float16, generator=generator))
        for _ in range(LAYERS)
    ]
    ids = torch.randint(0, 32000, (1, 1), generator=generator)
    with torch.inference_mode():
        logits = decoder.decode(ids)  # warm-up
        begin, steps = time.perf_counter(), 0
        while steps == 0 or time.perf_counter() - begin < budget_s:
            ids = logits[:, -1:].argmax(-1)
            logits = decoder.decode(ids)
            steps += 1
        seconds = time.perf_counter() - begin
    return {
        "value": steps / seconds,
        "unit": "tokens/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"one sequence with a {context}-token seeded cache, {steps} greedy decode steps of the "
                  "contiguous FP16 decoder with FP32 attention (the reference's per-row decode arithmetic) in "
                  f"{seconds:.1f}s on the host cores; the GPU line serves 256 such rows per step",
    }


def _prefill_cpu_baseline(weights, host_ids, sample_tokens: int = 128, budget_s: float = 10.0) -> dict:
    """The reference's prefill on the host cores: the dense FP16 forward that
    PagedCore's prefill_paged runs before its append (decoder.py:113-135), as
    restated by ``pagedcore_b200.decoder.prefill`` (bit-exact with it on CPU),
    on the first ``sample_tokens`` tokens of the same prompt, repeated for
    about ``budget_s`` seconds with all of torch's host threads."""
    import dataclasses

    import torch

    from pagedcore_b200.decoder import prefill as dense_prefill

    def host(layer):
        return type(layer)(**{f.name: getattr(layer, f.name).cpu() for f in dataclasses.fields(layer)})

    weights_cpu = type(weights)(embedding=weights.embedding.cpu(), layers=tuple(host(x) for x in weights.layers),
                                final_norm=weights.final_norm.cpu(), lm_head=weights.lm_head.cpu())
    prompt = host_ids[:, :sample_tokens].clone()
    with torch.inference_mode():
        dense_prefill(prompt, weights_cpu)  # warm-up
        begin, repeats = time.perf_counter(), 0
        while repeats == 0 or time.perf_counter() - begin < budget_s:
            dense_prefill(prompt, weights_cpu)
            repeats += 1
    seconds = time.perf_counter() - begin
    tokens = prompt.shape[1]
    return {
        "value": repeats * tokens / seconds,
        "unit": "tokens/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"the first {tokens} tokens of the prompt through the dense FP16 prefill (the reference's "
                  f"prefill_paged forward), {repeats} times in {seconds:.1f}s; a short prompt spends "
                  "relatively less on attention than the full one",
    }


def run_prefill_arm(args: argparse.Namespace) -> None:
    """Row f2: a whole prompt prefilled through the pool (``BatchedDecoder.prefill``).

    Random-init TinyLlama weights, one prompt of ``--prompt`` tokens (default
    2047, the longest that leaves room for a generated token) per GPU and step,
    into an empty request: embedding, 22 x (norm, fused Q/K/V GEMM, K/V write
    with RoPE, causal prefill attention over the block table, output
    projection, norm, gate/up GEMM, SwiGLU product, down projection), final
    norm and LM head for every prompt token.  The roofline is the hand-written
    attention kernel's (``prefill_tc_kernel``), timed alone over the
    same chunk on the same stream: its algorithmic MMA work over the measured
    dense tensor peak.
    """
    import torch
    import torch.distributed as dist

    from pagedcore_b200.decoder import BatchedDecoder
    from pagedcore_b200.engine_types import KVReservation, RequestId
    from pagedcore_b200.kv_cache import KVAllocator
    from pagedcore_b200.weights import random_weights

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    host_affinity = _bind_host_cores(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    seed = 6 + 1000 * rank
    tokens = args.prompt
    if not 1 <= tokens <= 2047:
        raise SystemExit("--prompt must lie in [1, 2047]")
    blocks = -(-tokens // 16)
    pool = torch.empty((LAYERS, 2, blocks + 8, 16, 4, 64), dtype=torch.float16, device=device)
    allocator = KVAllocator(pool, validation="incremental")
    weights = random_weights(seed, device)
    decoder = BatchedDecoder(weights)
    generator = torch.Generator(device="cpu").manual_seed(seed)
    host_ids = torch.randint(0, 32000, (1, tokens), generator=generator).pin_memory()
    ids = host_ids.to(device)
    request = RequestId("prompt")
    stream = torch.cuda.current_stream(device)

    def prefill(prompt):
        allocator.create(KVReservation(request, blocks))
        logits = decoder.prefill(prompt, allocator, request)
        allocator.release_all(request)
        return logits

    def barrier() -> None:
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    with ClockSampler(local_rank) as clocks:
        for _ in range(args.warmup):
            prefill(ids)
        torch.cuda.synchronize(device)
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.begin()
        torch.cuda.nvtx.range_push("timed")  # marks the timed launches for an ncu launch list
        start.record(stream)
        for _ in range(args.steps):
            logits = prefill(ids)
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(device)
        clocks.end()
    step_ms = start.elapsed_time(end) / args.steps
    # End to end through the public call: the prompt ids copied from pinned
    # host memory and the last token's logits read back, every step.
    last = torch.empty((1, 32000), dtype=torch.float16, pin_memory=True)
    torch.cuda.synchronize(device)
    barrier()
    e2e_start, e2e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_start.record(stream)
    for _ in range(args.steps):
        prompt = host_ids.to(device, non_blocking=True)
        last.copy_(prefill(prompt)[0, -1:], non_blocking=True)
    e2e_end.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = e2e_start.elapsed_time(e2e_end) / args.steps
    # The attention kernel alone, one layer of the same chunk, on the same stream.
    allocator.create(KVReservation(request, blocks))
    query = torch.randn(tokens, 32, 64, dtype=torch.float16, device=device)
    key = torch.randn(tokens, 4, 64, dtype=torch.float16, device=device)
    with allocator.prefill_append(request, tokens) as chunk:
        rotated = chunk.write_layer(0, key, key, query)
        out = torch.empty_like(rotated)
        for _ in range(3):
            chunk.attend(0, rotated, out)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            chunk.attend(0, rotated, out)
        b.record(stream)
        torch.cuda.synchronize(device)
    allocator.release_all(request)
    attention_us = a.elapsed_time(b) / args.steps * 1000.0
    allocator.check_device_errors()
    times = torch.tensor([step_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    step_ms, e2e_ms = (float(x) for x in times.tolist())
    if rank == 0:
        peak, peak_kind = _peak_tensor()
        # Token t attends to t + 1 positions: QK^T and PV are 2 x 2 x 64 FLOP
        # per (query head, position) pair.
        flops = 4.0 * 64 * 32 * tokens * (tokens + 1) / 2
        achieved = flops / (attention_us * 1e-6) / 1e12
        line = {
            "metric": "prompt tokens/s, whole TinyLlama prefill through the pool (row f2: paged prefill)",
            "value": world * tokens / (step_ms / 1000.0),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": step_ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (random-init TinyLlama weights N(0, 0.02), random prompt token ids)",
            "config": {
                "workload": f"one {tokens}-token prompt per GPU per step into an empty request, every layer's K/V "
                            "written to the pool and attended through the block table (BatchedDecoder.prefill); "
                            "weights (2.2 GB) larger than L2",
                "parallelism": f"dp{world} (independent prompts, weights replicated, no collective)",
            },
            "e2e": {
                "value": world * tokens / (e2e_ms / 1000.0),
                "unit": "tokens/s",
                "h2d_bytes_per_step": tokens * 8,
                "d2h_bytes_per_step": 32000 * 2,
            },
            "roofline": {
                "bound": "tensor",
                "kernel": "prefill_tc_kernel (tcgen05.mma kind::f16, FP16 in, FP32 accumulate in TMEM)",
                "achieved": achieved,
                "peak": peak,
                "peak_kind": peak_kind,
                "unit": "TFLOP/s",
                "frac": achieved / peak,
                "flops_per_launch": flops,
                "launch_us": attention_us,
                # DRAM bytes of one launch at 2047 tokens from one ncu capture: the
                # rotated Q and the layer's K/V read once, the re-reads hit L2.
                "traffic": PREFILL_DRAM_BYTES_2047 if tokens == 2047 else None,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at 2047 tokens"
                                  if tokens == 2047 else None,
            },
            # This library's kernels per step: per layer two fused norms, the K/V write
            # (Q rotated in place), the prefill attention and the SwiGLU product; then
            # the final norm.  The GEMMs and the embedding are library/torch kernels,
            # except that a one-token prompt's projections (Q/K/V, o, gate/up, down per
            # layer and the LM head) run this library's matrix-vector kernel.
            "gpu_launches": args.steps * _step_launches(tokens),
            "gpu_launches_attention_per_step": LAYERS,
            "logits_finite": bool(torch.isfinite(logits).all().item()),
            "clocks": clocks.summary(),
            "host_affinity": host_affinity,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = _prefill_cpu_baseline(weights, host_ids)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--repeats", type=int, default=3,
                        help="timed regions of --steps steps each (the line reports the median and the spread)")
    parser.add_argument("--no-decoder", action="store_true",
                        help="skip the whole-decoder leg of the default line")
    parser.add_argument("--no-shared", action="store_true",
                        help="skip the shared-batch point (256 / N sequences per GPU) of the default line at N > 1")
    parser.add_argument("--sequences", type=int, default=SEQUENCES,
                        help="sequences per GPU (default: config 4's 256; smaller only for ncu captures)")
    parser.add_argument("--workload", choices=("decode", "stress", "append", "decoder", "prefill"), default="decode",
                        help="decode: config 4 (the headline line); stress: config 5 (allocator churn); "
                             "append: config 2a (prompt K/V appends); decoder: row f1 (whole decoder step); "
                             "prefill: row f2 (a whole prompt through the pool)")
    parser.add_argument("--prompt", type=int, default=2047, help="prompt tokens of the prefill workload")
    parser.add_argument("--stress-iterations", type=int, default=300)
    parser.add_argument("--stress-warmup", type=int, default=200)
    args = parser.parse_args()
    globals()["SEQUENCES"] = args.sequences
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.workload == "stress":
        run_stress_arm(args)
    elif args.workload == "append":
        run_append_arm(args)
    elif args.workload == "decoder":
        run_decoder_arm(args)
    elif args.workload == "prefill":
        run_prefill_arm(args)
    else:
        run_gpu_arm(args)


if __name__ == "__main__":
    main()
