"""Training-throughput benchmark: BS-RoFormer audio-seconds per second on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config config3] [--impl ours|reference]

N > 1 runs under ``torch.distributed.run`` (one rank per GPU, NCCL); every rank
trains on its own seeded synthetic batch (weak scaling) and the captured step
all-reduces the flat gradient buffer over NCCL (mean over ranks).  Rank 0
prints one JSON line:

* ``value``: whole-job audio-seconds/s with inputs resident in HBM (device
  time of K steps, CUDA events, max over ranks);
* ``e2e``: the same through the public step API from pinned host buffers
  (H2D copy of every step's audio and D2H copy of every step's loss inside
  the timed region);
* ``roofline``: the dominant fused op of this package, timed with CUDA events
  around its calls during the timed steps, against the measured peaks;
* ``cpu_baseline``: the CPU oracle (the reference semantics in PyTorch, fp32)
  on a bounded sample of the same workload (the benchmark's batch, five timed
  steps), on this machine's host cores;
* ``clocks``: nvidia-smi samples taken during the timed region.

``--impl reference`` times the reference's CPU implementation of the path
(the oracle port: the reference's CUDA extension has no model, and its model
package pymss-core is not installed) at the benchmark's per-GPU batch, K
timed steps, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch
import torch.distributed as dist

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from pymsst_b200 import _native as nat  # noqa: E402
from pymsst_b200 import roofline as rl  # noqa: E402
from pymsst_b200 import synthetic  # noqa: E402
from pymsst_b200.train import CONFIGS, Trainer, build_model, init_distributed, max_over_ranks  # noqa: E402

METRIC = "BSR train audio-sec/sec"
UNIT = "audio-s/s"
TIMED_ENTRIES = [
    "pmb_rms_norm_forward", "pmb_rms_norm_backward", "pmb_qkv_rotary_split", "pmb_qkv_rotary_merge",
    "pmb_attention_gate_forward", "pmb_attention_gate_backward", "pmb_band_gather_forward",
    "pmb_band_recombine_forward", "pmb_band_recombine_backward", "pmb_band_split_forward",
    "pmb_band_split_backward", "pmb_grouped_linear_forward", "pmb_grouped_linear_backward",
    "pmb_mask_estimator_final_forward", "pmb_mask_estimator_final_backward", "pmb_mask_estimator_tc_forward",
    "pmb_mask_estimator_tc_backward", "pmb_gemm_tc", "pmb_qkv_linear_rotary_forward", "pmb_band_split_tc_forward",
    "pmb_band_split_tc_backward", "pmb_gelu_forward", "pmb_gelu_backward", "pmb_column_sum",
    "pmb_attention_forward", "pmb_attention_backward", "pmb_attention_backward_rotary", "pmb_rms_norm_backward_add",
    "pmb_stft_frames_forward", "pmb_stft_frames_backward", "pmb_spectral_l1_forward", "pmb_spectral_l1_backward",
    "pmb_attention_forward_gated", "pmb_attention_backward_gated", "pmb_istft_overlap_add_forward",
    "pmb_istft_overlap_add_backward",
]


def parse():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--config", default="config3", choices=sorted(CONFIGS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--bucket-mb", type=float, default=1024.0,
                   help="gradient all-reduce bucket size (MB) of --overlap-allreduce and of the eager DDP path; the "
                        "default puts all gradients in one bucket reduced after the backward, which keeps NCCL off "
                        "the SMs while the persistent kernels run")
    p.add_argument("--overlap-allreduce", action="store_true",
                   help="N > 1: all-reduce the flat gradients in buckets launched from gradient hooks during the "
                        "backward (bucket size --bucket-mb) instead of once after it")
    p.add_argument("--eager", action="store_true",
                   help="launch every kernel from Python each step instead of replaying the captured step graph")
    p.add_argument("--profile-range", action="store_true",
                   help="bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    p.add_argument("--traffic-json", default="",
                   help="per-kernel ncu DRAM bytes per launch, {config: {entry: bytes}} (default: the measured "
                        "table in pymsst_b200.roofline)")
    return p.parse_args()


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu_index)], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = [line.split(",") for line in Path(self.file.name).read_text().splitlines() if line.strip()]
        os.unlink(self.file.name)
        sm, reasons, smax = [], set(), None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


def physical_gpu_index(local_rank: int) -> int:
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        ids = [v.strip() for v in visible.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ------------------------------------------------------------ CPU timings
def cpu_oracle_rate(bench, steps: int, warmup: int, batch: int = 1) -> dict:
    """Time the oracle (reference semantics, fp32) training step on the host cores."""
    from oracle import roformer_ref

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    model = roformer_ref.build(bench.model_type, **bench.model)
    opt = torch.optim.Adam(model.parameters(), lr=bench.lr)
    mix, tgt = synthetic.make_batch(batch, bench.chunk, seed=12345, stems=bench.stems)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        opt.zero_grad(set_to_none=True)
        loss = model(mix, tgt)
        loss.backward()
        opt.step()
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    per_step = statistics.median(times)
    audio = batch * bench.chunk / synthetic.SAMPLE_RATE
    cpu_name = ""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                cpu_name = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"value": round(audio / per_step, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{bench.name} architecture, fp32, batch {batch} x {bench.chunk} samples, fwd+bwd+Adam, "
                      f"median of {steps} steps after {warmup} warm-up ({per_step:.2f} s/step); CPU {cpu_name}"}


def bench_config(bench, world: int) -> dict:
    """The ``config`` object of both arms' JSON lines."""
    return {"workload": bench.name, "model": bench.model_type, "global_batch": bench.batch * world,
            "per_gpu_batch": bench.batch, "chunk_samples": bench.chunk, "frames": bench.frames,
            "parallelism": f"dp{world}", "note": bench.notes,
            "l2": "no flush: a step's activations (several GB) exceed the 126 MB L2"}


def run_reference(args, rank: int, world: int):
    """The reference's CPU path of the step (fused backend off: fp32 PyTorch) on this box's host cores, at the
    benchmark's own per-GPU batch; rank 0 only (one CPU sample stands for the job)."""
    if rank != 0:
        return
    bench = CONFIGS[args.config]
    base = cpu_oracle_rate(bench, steps=max(1, args.steps), warmup=min(max(0, args.warmup), 3), batch=bench.batch)
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "config": bench_config(bench, 1),
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- ours
def run_ours(args, rank: int, world: int, local: int):
    bench = CONFIGS[args.config]
    device = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    model = build_model(bench, seed=0)
    trainer = Trainer(model, lr=bench.lr, amp_dtype=bench.amp, distributed=world > 1, device=device,
                      bucket_cap_mb=args.bucket_mb, cuda_graph=not args.eager,
                      overlap_allreduce=args.overlap_allreduce)
    pool = 2
    host = [synthetic.make_batch(bench.batch, bench.chunk, seed=1000 * rank + i, stems=bench.stems) for i in range(pool)]
    host = [(m.pin_memory(), t.pin_memory()) for m, t in host]
    dev = [(m.to(device), t.to(device)) for m, t in host]
    h2d = host[0][0].numel() * host[0][0].element_size() + host[0][1].numel() * host[0][1].element_size()
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    for i in range(args.warmup):
        trainer.step(*dev[i % pool])
    barrier()

    sampler = ClockSampler(physical_gpu_index(local)) if rank == 0 else None
    if sampler:
        sampler.start()
    launches0 = nat.library().pmb_launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    if args.profile_range:
        torch.cuda.cudart().cudaProfilerStart()
    start.record(stream)
    for i in range(args.steps):
        trainer.step(*dev[i % pool])
    end.record(stream)
    barrier()
    if args.profile_range:
        torch.cuda.cudart().cudaProfilerStop()
    if trainer.cuda_graph:
        launches = trainer.launches_per_step * args.steps
    else:
        launches = nat.library().pmb_launch_count() - launches0
    value_ms = start.elapsed_time(end)

    # end to end through the step API from pinned host buffers
    losses = torch.empty(args.steps, dtype=torch.float32).pin_memory()
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for i in range(args.steps):
        trainer.step_host(*host[i % pool], loss_out=losses[i : i + 1])
    e_end.record(stream)
    barrier()
    e2e_ms = e_start.elapsed_time(e_end)
    clocks = sampler.stop() if sampler else None

    # per-kernel durations for the roofline: each entry point bracketed by CUDA events on its stream.  Graph
    # mode: the step's forward/backward captured once more with the events as graph nodes and replayed K times,
    # so the times are device times inside the replayed step; eager mode: the eager forward/backward.
    barrier()
    calls_ms: dict = {}
    if trainer.cuda_graph:
        with nat.time_entries(TIMED_ENTRIES, external=True) as timer:
            prof = trainer.profile_graph()
        for _ in range(args.steps):
            prof.replay()
            for n, (c, ms, a) in timer.result().items():
                tot = calls_ms.setdefault(n, [0, 0.0, []])
                tot[0] += c
                tot[1] += ms
                tot[2] += a
        del prof
    else:
        with nat.time_entries(TIMED_ENTRIES) as timer:
            for i in range(args.steps):
                trainer._zero_grads()
                trainer._forward_backward(*dev[i % pool])
            barrier()
        calls_ms = {n: list(v) for n, v in timer.result().items()}
    barrier()

    trainer.check_kernels()  # no tensor-core wait ran out during the timed or profiled steps
    value_ms, e2e_ms = max_over_ranks([value_ms, e2e_ms], device)
    trainer.close()  # the captured step (with its collectives) goes before the process group does
    audio_job = bench.audio_seconds_per_step * world * args.steps
    result = {n: tuple(v) for n, v in calls_ms.items()}
    if rank != 0:
        return

    peaks = rl.load_peaks()
    traffic = rl.MEASURED_TRAFFIC.get(bench.name, {})
    if args.traffic_json:
        traffic = json.loads(Path(args.traffic_json).read_text()).get(bench.name, {})
    per_entry = {n: round(ms, 3) for n, (c, ms, _) in sorted(result.items(), key=lambda kv: -kv[1][1]) if c}
    top = max(result.items(), key=lambda kv: kv[1][1])
    name, (calls, total_ms, arglist) = top
    roof = rl.roofline(name, calls, total_ms, arglist, peaks, traffic=traffic.get(name), in_step=True)
    roof["timing"] = ("CUDA events as graph nodes around each call, in K replays of the captured step's "
                      "forward/backward" if trainer.cuda_graph else "CUDA events around each call of K eager steps")

    line = {
        "metric": METRIC, "value": round(audio_job / (value_ms / 1e3), 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value_ms / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": {torch.bfloat16: "bf16", torch.float16: "f16", None: "f32"}[bench.amp], "data": "synthetic",
        "config": bench_config(bench, world),
        "e2e": {"value": round(audio_job / (e2e_ms / 1e3), 3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches),
        "step_launch": "cuda graph replay" if trainer.cuda_graph else "eager",
        "roofline": roof,
        "fused_op_ms": per_entry,
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_oracle_rate(bench, steps=5, warmup=1, batch=bench.batch)
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank, world, local = init_distributed()
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
