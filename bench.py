"""Benchmark: DWARF-v2 whole-model prefill on 1..8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1)

Workload: DwarfForCausalLM (D=512, L=10, T=2048, vocab 32768, seeded bf16
weights), q6 KV cache in every DSQG layer, global batch 256 uniform-random
token ids in [57, 32768), split by batch rows across the ranks (strong scaling:
the global batch is fixed). One step = prefill of the whole batch to logits
plus an NCCL all-gather of every row's next-token logits to all ranks.

The prefill is launched eagerly (``--graph``: as one CUDA graph per step,
``model.capture_prefill``; measured the same within 0.1%: the step is not
launch-bound).

Printed JSON line (rank 0):
* value    tokens/s with inputs resident in HBM, timed with CUDA events over
           exactly K steps between barriers, max over ranks;
* e2e      the same step through the public API with the host->device copy of
           the token ids (pinned) and the device->host read of the gathered
           next-token logits inside the timed region;
* roofline the dominant engine kernel (dwarf_dsqg_fwd): algorithmic bytes per
           launch / its mean CUDA-event duration (per-launch events in an eager
           run of the same K steps right after the graph's timed region),
           against the measured HBM copy bandwidth; ``fma`` beside it: the
           kernel's FP32 pair FMAs (2 x 64 per valid (query, offset) pair) per
           second against the derived CUDA-core peak (148 SMs x 128 lanes x 2
           x the sampled SM clock);
* device_status the status word of the kernels' bounded waits after the
           timed region (non-zero: a wait ran out and the line is invalid);
* cpu_baseline  the CPU oracle port of the same prefill (oracle/model.py) on
           one 2048-token row, host cores, rank 0 at N=1.
``--impl reference`` times that CPU port alone on the host cores (the
reference's own code is pure PyTorch/Triton under a source tree that is not
present on the GPU box), with the port built once outside the timed steps.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
METRIC = "prefill tok/s (D512 L10 T2048, q6 KV) at 1/2/4/8 B200; kernel HBM % of peak"
GLOBAL_BATCH = 256
SEQ_LEN = 2048
VOCAB = 32768
FALLBACK_HBM_GBS = 6650.0


def _peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _token_ids(rows: slice) -> torch.Tensor:
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(57, VOCAB, (GLOBAL_BATCH, SEQ_LEN), generator=g)
    return ids[rows].contiguous()


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a timed region.

    One process per node: local rank 0 samples every GPU of the job on its node
    (``indices``); the other ranks pass ``None`` and start nothing, so that N
    pollers do not contend with the kernel launches of an N-GPU step. The
    process starts before the warm-up steps (its NVML start-up is heavy driver
    work that must not land in the timed region); ``mark_start`` / ``mark_end``
    bracket the timed region on the host clock, and the summary keeps the
    samples whose nvidia-smi timestamps fall inside it (with one sampling period
    of slack at either end, so that a short region still has samples)."""

    PERIOD_S = 0.1
    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices: list[int] | None):
        self.indices = indices
        self.proc = None
        self.t0 = self.t1 = None

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __enter__(self):
        if not self.indices:
            return self
        ids = ",".join(str(i) for i in self.indices)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={ids}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", str(int(self.PERIOD_S * 1000))], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lo = self.t0 - self.PERIOD_S if self.t0 is not None else None
        hi = self.t1 + self.PERIOD_S if self.t1 is not None else None
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            try:
                stamp = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                if (lo is not None and stamp < lo) or (hi is not None and stamp > hi):
                    continue
                sm.append(float(parts[2]))
                mx = float(parts[3])
            except (ValueError, IndexError):
                continue
            for name, flag in zip(names, parts[6:10]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def _cpu_port():
    """The CPU restatement of the prefill (oracle/model.py), its seeded reference-init
    state dict and the offset lattice; built once, outside any timed region."""
    sys.path.insert(0, str(ROOT))
    from oracle import model as omodel

    from dwarf_v2_b200.dsqg_attention_v22 import ALL_OFFSETS
    from dwarf_v2_b200.model import DwarfForCausalLM

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    with torch.no_grad():
        state = {k: v.clone() for k, v in DwarfForCausalLM().state_dict().items()}
    return omodel, state, ALL_OFFSETS, cores


def _cpu_sample(port, ids) -> float:
    omodel, state, offsets, _ = port
    t0 = time.perf_counter()
    omodel.prefill(state, ids, all_offsets=offsets)
    return time.perf_counter() - t0


def cpu_baseline(sample_rows: int = 1) -> dict:
    """Time the CPU oracle port of the prefill on `sample_rows` rows of the workload
    (model construction outside the timed call)."""
    port = _cpu_port()
    ids = _token_ids(slice(0, sample_rows))
    dt = _cpu_sample(port, ids)
    return {"value": sample_rows * SEQ_LEN / dt, "unit": "tok/s", "cores": port[3], "kind": "port",
            "sample": f"{sample_rows} row(s) x {SEQ_LEN} tokens of the config-5 batch through oracle/model.py "
                      f"(fp32/fp64 CPU restatement of the reference forward), {dt:.1f} s"}


def run_reference(args) -> None:
    world, rank, _ = _dist()
    if rank != 0:
        return
    port = _cpu_port()
    ids = _token_ids(slice(0, 1))
    for _ in range(args.warmup):
        _cpu_sample(port, ids)
    times = [_cpu_sample(port, ids) for _ in range(args.steps)]
    value = SEQ_LEN * len(times) / sum(times)
    r = {"unit": "tok/s", "cores": port[3], "kind": "port",
         "sample": f"each step: 1 row x {SEQ_LEN} tokens of the config-5 batch through oracle/model.py "
                   "(fp32/fp64 CPU restatement of the reference forward; model built once, untimed)"}
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded uniform token ids in [57,32768); seeded reference init)",
            "config": {"workload": "config5: DWARF-v2 prefill, T=2048; each step a 1-row sample on host cores",
                       "global_batch": GLOBAL_BATCH, "seq_len": SEQ_LEN},
            "cpu_baseline": {**r, "value": value},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import torch.distributed as dist

    from dwarf_v2_b200 import _lib
    from dwarf_v2_b200.model import DwarfForCausalLM
    from dwarf_v2_b200.sharding import gather_rows, rows_for_rank

    world, rank, local = _dist()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    mine = rows_for_rank(GLOBAL_BATCH, rank, world)
    rows = mine.stop - mine.start
    model = DwarfForCausalLM(kv_cache="q6").eval().to(torch.bfloat16).to(dev)
    ids_host = _token_ids(mine).pin_memory()
    ids_dev = ids_host.to(dev)
    gathered = torch.empty(GLOBAL_BATCH, VOCAB, dtype=torch.bfloat16, device=dev)
    out_host = torch.empty(GLOBAL_BATCH, VOCAB, dtype=torch.bfloat16).pin_memory()

    # --graph: the prefill as one CUDA graph (model.capture_prefill), the same kernels
    # as the eager forward launched as one graph instead of ~300 host launches; a
    # launch log active during the capture counts the engine kernels of one step.
    capture_log = _lib.LaunchLog()
    _lib.set_launch_log(capture_log)
    try:
        graph = model.capture_prefill(rows, SEQ_LEN) if args.graph else None
    finally:
        _lib.set_launch_log(None)
    launches_per_step = capture_log.count // 2 if graph is not None else None  # warm-up + capture

    def forward(ids):
        return graph(ids) if graph is not None else model(ids)

    def step(ids):
        logits = forward(ids)
        return gather_rows(logits[:, -1].contiguous(), gathered)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    clocks = ClockSampler(list(range(local_world)) if local == 0 else None)
    with torch.no_grad():
        clocks.__enter__()  # started before the warm-up: its start-up stays out of the timed region
        try:
            for _ in range(max(args.warmup, 0)):
                step(ids_dev)
            # device-resident throughput
            log = _lib.LaunchLog(timed=("dwarf_dsqg_fwd",))
            barrier()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            _lib.set_launch_log(log)
            clocks.mark_start()
            start.record()
            for _ in range(args.steps):
                step(ids_dev)
            end.record()
            _lib.set_launch_log(None)
            barrier()
            clocks.mark_end()
        finally:
            clocks.__exit__(None, None, None)
        ms = max_over_ranks(start.elapsed_time(end) / args.steps)
        launches = log.count if graph is None else launches_per_step * args.steps
        if graph is not None:
            # The graph's kernels carry no per-launch events: the DSQG launch time for
            # the roofline comes from the same steps run eagerly right after (the
            # same kernels, arguments and inputs), with CUDA events around each
            # dwarf_dsqg_fwd launch on its stream.
            log = _lib.LaunchLog(timed=("dwarf_dsqg_fwd",))
            barrier()
            _lib.set_launch_log(log)
            for _ in range(args.steps):
                model(ids_dev)
            _lib.set_launch_log(None)
            barrier()
        dsqg_ms = log.mean_ms("dwarf_dsqg_fwd")
        # end to end through the public API: H2D ids, prefill + gather, D2H logits
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            ids_dev.copy_(ids_host, non_blocking=True)
            out = step(ids_dev)
            if rank == 0:
                out_host.copy_(out, non_blocking=True)
        end.record()
        barrier()
        e2e_ms = max_over_ranks(start.elapsed_time(end) / args.steps)

    device_status = _lib.read_and_clear_device_status(dev)
    tokens = GLOBAL_BATCH * SEQ_LEN
    hbm, hbm_kind = _peaks()
    # dwarf_dsqg_fwd algorithmic bytes per launch (one DSQG layer over this rank's rows):
    # Q bf16 + K/V q6 codes+scales + y_pre/z_pre fp32 + content gate bf16 + output bf16.
    per_row = 8 * SEQ_LEN  # (head, token) rows per batch row
    dsqg_bytes = rows * per_row * (64 * 2 + 2 * 50 + 2 * 16 + 64 * 2 + 64 * 2)
    achieved = dsqg_bytes / (dsqg_ms * 1e-3) / 1e9 if dsqg_ms else None
    # FP32 work of one dwarf_dsqg_fwd launch, averaged over the model's DSQG layers:
    # 2 x 64 FMAs (q.k and p.v) per valid (query, offset) pair.
    from dwarf_v2_b200.model import DSQGBlock

    layer_groups = [blk.attn.offsets for blk in model.blocks if isinstance(blk, DSQGBlock)]
    pairs = sum(sum(max(0, SEQ_LEN - d) for d in g) for g in layer_groups) / len(layer_groups)
    dsqg_flops = rows * 8 * pairs * 2 * 64 * 2
    clock = clocks.summary()
    sm_mhz = clock["sm_mhz"] or 1965.0
    fma_peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12
    fma = ({"achieved": dsqg_flops / (dsqg_ms * 1e-3) / 1e12, "peak": fma_peak, "unit": "TFLOP/s",
            "frac": dsqg_flops / (dsqg_ms * 1e-3) / 1e12 / fma_peak, "flops_per_launch": dsqg_flops,
            "peak_kind": "derived: 148 SMs x 128 FP32 lanes x 2 x median sampled SM clock"} if dsqg_ms else None)
    traffic = None
    prof = ROOT / "profiles" / "dsqg_fwd_traffic.json"
    if prof.is_file():
        info = json.loads(prof.read_text())
        traffic = info["dram_bytes_per_row"] * rows
    line = {
        "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded uniform token ids in [57,32768); random-init weights (reference seeded init)",
        "config": {"workload": "config5: full DWARF-v2 prefill D512 L10 T2048, q6 KV, batch rows sharded",
                   "model": "DWARF-v2 55M (10 blocks: 9 DSQG + 1 HISA)", "global_batch": GLOBAL_BATCH,
                   "seq_len": SEQ_LEN, "parallelism": f"dp{world}", "kv_cache": "q6",
                   "l2": "no flush: every step's working set (>= 4 GB of activations per GPU) exceeds L2",
                   "launch": "eager" if graph is None else "one CUDA graph per step (model.capture_prefill)"},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": rows * SEQ_LEN * 8,
                "d2h_bytes_per_step": GLOBAL_BATCH * VOCAB * 2 if rank == 0 else 0},
        "gpu_launches": launches,
        "roofline": {"kernel": "dwarf_dsqg_fwd", "bound": "hbm", "achieved": achieved, "peak": hbm,
                     "peak_kind": hbm_kind, "unit": "GB/s", "frac": (achieved / hbm) if achieved else None,
                     "traffic": traffic, "algorithmic_bytes_per_launch": dsqg_bytes, "mean_launch_ms": dsqg_ms,
                     "fma": fma},
        "clocks": clock,
        "device_status": device_status,
    }
    if device_status != 0:
        line["invalid"] = "a kernel's bounded wait ran out (DWARF_DEVICE_TIMEOUT) during the timed steps"
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    if device_status != 0:
        sys.exit(3)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=None, help="override the global batch (small profiling cases)")
    ap.add_argument("--graph", action="store_true", help="run each step as one CUDA graph (model.capture_prefill)")
    args = ap.parse_args()
    if args.rows:
        global GLOBAL_BATCH
        GLOBAL_BATCH = args.rows
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
