"""Benchmark of the ZONOS3-Mini hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload ("cfg2"): gated-DeltaNet recurrent decode of 64 streams x 16 heads,
dk = dv = 128, 512 sequential single-token state updates with per-step outputs. One bench step is that whole run.
The 64 MB state of one layer fits in the 126 MB L2, while in the model every GDN layer owns a state and the rest
of the step runs between two updates of it, so the bench keeps LAYERS = 4 independent layer states and updates
them round-robin (256 MB of state, more than L2; no flush needed). An audio token is one decode update of one
stream; value = streams x layers x 512 x K x N / max-over-ranks time.

Multi-GPU: one process per GPU (torchrun), each rank runs its own 64-stream replica (request sharding, no
collective on the data path); the only collectives are the barrier and the max-reduction of the timings.

``--impl reference`` times the reference's CPU implementation of the same path (the per-token recurrence of
model/src/zonos3/reference/lm.py:576-582, restated in oracle/gdn.py) on the host cores, on rank 0 only.
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
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "audio tokens/sec per box"
UNIT = "tokens/s"

# cfg2
STREAMS, HEADS, DK, DV, UPDATES = 64, 16, 128, 128, 512
LAYERS = 4


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        busy = [s for s, r in zip(sm, rows) if float(r[3] or 0) > 200.0] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


# --------------------------------------------------------------------------------------------- distributed


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, local: int):
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        return dist
    return None


def barrier(dist):
    if dist is not None:
        dist.barrier()


def max_over_ranks(dist, value: float) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------------------------- cfg2 workload


def cfg2_inputs(seed: int, device, streams=STREAMS):
    """cfg2 distributions (seeded on CPU, then moved): q, k ~ N(0,1) L2-normalised per head (bf16), v ~ N(0,1)
    (bf16), beta = sigmoid(N(0,1)), g = -softplus(N(0,1)); one [UPDATES] sequence of per-step inputs."""
    gen = torch.Generator().manual_seed(seed)
    shape = (UPDATES, streams, HEADS)
    q = F.normalize(torch.randn(*shape, DK, generator=gen), dim=-1).bfloat16()
    k = F.normalize(torch.randn(*shape, DK, generator=gen), dim=-1).bfloat16()
    v = torch.randn(*shape, DV, generator=gen).bfloat16()
    beta = torch.sigmoid(torch.randn(*shape, generator=gen))
    g = -F.softplus(torch.randn(*shape, generator=gen))
    return [t.to(device) for t in (q, k, v, g, beta)]


def cfg2_state(seed: int, device, streams=STREAMS):
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(streams, HEADS, DV, DK, generator=gen) * 0.01).to(device)


def bytes_per_update(streams=STREAMS) -> int:
    """Algorithmic bytes of one decode update: state read + write (fp32), q, k, v (bf16), g, beta (fp32), out."""
    return streams * HEADS * (2 * DK * DV * 4 + (2 * DK + DV) * 2 + 2 * 4 + DV * 2)


def run_ours(args, dist, rank, world, local):
    pkg = __import__("__graft_entry__").load_package()
    ops = pkg.ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    seed = 1234 + rank
    q, k, v, g, beta = cfg2_inputs(seed, dev)
    states = [cfg2_state(seed + 1 + l, dev) for l in range(LAYERS)]
    outs = torch.empty(LAYERS, UPDATES, STREAMS, HEADS, DV, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.Stream(dev)

    def one_step():
        for t in range(UPDATES):
            for l in range(LAYERS):
                ops.gdn_decode_step(q[t], k[t], v[t], g[t], beta[t], states[l], outs[l, t])

    launches_per_step = UPDATES * LAYERS
    with torch.cuda.stream(stream):
        one_step()  # eager warm-up (loads the library, first launch)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            one_step()
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize(dev)
        barrier(dist)
        torch.cuda.synchronize(dev)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index) as clocks:
            start.record(stream)
            for _ in range(args.steps):
                graph.replay()
            stop.record(stream)
            torch.cuda.synchronize(dev)
        barrier(dist)
        torch.cuda.synchronize(dev)
    elapsed_ms = max_over_ranks(dist, start.elapsed_time(stop))
    del graph

    # end to end through the public op with host buffers: every update copies its inputs from pinned host memory
    # and reads its output back, all inside the timed region
    host = [t.cpu().pin_memory() for t in (q, k, v, g, beta)]
    host_out = torch.empty(UPDATES, STREAMS, HEADS, DV, dtype=torch.bfloat16).pin_memory()
    dq = [torch.empty_like(t[0]) for t in (q, k, v, g, beta)]
    h2d_update = sum(t[0].numel() * t.element_size() for t in host)
    d2h_update = host_out[0].numel() * host_out.element_size()
    e2e_steps = max(1, min(args.steps, 3))
    with torch.cuda.stream(stream):
        def e2e_step():
            for t in range(UPDATES):
                for l in range(LAYERS):
                    for dst, src in zip(dq, host):
                        dst.copy_(src[t], non_blocking=True)
                    o = ops.gdn_decode_step(dq[0], dq[1], dq[2], dq[3], dq[4], states[l], outs[l, t])
                    host_out[t].copy_(o, non_blocking=True)
        e2e_step()
        torch.cuda.synchronize(dev)
        barrier(dist)
        e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e_stop.record(stream)
        torch.cuda.synchronize(dev)
        barrier(dist)
    e2e_ms = max_over_ranks(dist, e_start.elapsed_time(e_stop))

    tokens_per_step = STREAMS * LAYERS * UPDATES
    value = tokens_per_step * args.steps * world / (elapsed_ms / 1e3)
    e2e_value = tokens_per_step * e2e_steps * world / (e2e_ms / 1e3)
    pk = peaks()
    bytes_launch = bytes_per_update()
    launch_s = elapsed_ms / 1e3 / (args.steps * launches_per_step)
    achieved = bytes_launch / launch_s / 1e9
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded cfg2 distributions; random state N(0, 0.01^2))",
        "config": {
            "workload": "cfg2 gated-DeltaNet recurrent decode: 64 streams x 16 heads, dk=dv=128, 512 sequential "
                        "single-token updates with per-step outputs; 4 layer states round-robin",
            "streams_per_gpu": STREAMS, "heads": HEADS, "dk": DK, "dv": DV, "updates_per_step": UPDATES,
            "layer_states": LAYERS, "token": "one decode update of one stream",
            "l2": "state working set 256 MB > 126 MB L2 (no flush)", "graph": "CUDA graph of one step",
            "parallelism": f"replicas x{world} (request-sharded, no collective)",
        },
        "roofline": {
            "kernel": "gdn_decode_kernel<128>", "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
            "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "traffic": None,
            "algorithmic_bytes_per_launch": bytes_launch, "avg_launch_us": launch_s * 1e6,
            "peak_source": pk["source"],
        },
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d_update * LAYERS * UPDATES,
                "d2h_bytes_per_step": d2h_update * LAYERS * UPDATES,
                "path": "ops.gdn_decode_step per update with pinned-host copies in and out"},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clocks.summary(),
    }
    line["roofline"]["traffic"] = profiled_traffic("gdn_decode_cfg2.md")
    return line


def profiled_traffic(summary: str):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) recorded from an ncu capture in the
    committed summary under profiles/, or None."""
    path = ROOT / "profiles" / summary
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return int(line.split(":", 1)[1])
    return None


def cpu_reference(updates: int, streams=STREAMS):
    """Time the CPU recurrence (oracle/gdn.py restating lm.py:576-582) on this host's cores.
    Returns (tokens/s, threads, seconds)."""
    from oracle import gdn as ogdn

    torch.set_num_threads(os.cpu_count() or 1)
    q, k, v, g, beta = cfg2_inputs(99, "cpu", streams)
    state = cfg2_state(98, "cpu", streams)
    ogdn.recurrent_step(state, q[0], k[0], v[0], g[0], beta[0], DK ** -0.5)
    t0 = time.perf_counter()
    for t in range(updates):
        state, _ = ogdn.recurrent_step(state, q[t % UPDATES], k[t % UPDATES], v[t % UPDATES], g[t % UPDATES],
                                       beta[t % UPDATES], DK ** -0.5)
    dt = time.perf_counter() - t0
    return streams * updates / dt, torch.get_num_threads(), dt


def profile_launches(n: int) -> None:
    """n eager cfg2 decode updates cycling the layer states (the bench's own launches, without graphs or timing)."""
    ops = __import__("__graft_entry__").load_package().ops
    dev = torch.device("cuda", 0)
    q, k, v, g, beta = cfg2_inputs(1234, dev)
    states = [cfg2_state(1235 + l, dev) for l in range(LAYERS)]
    out = torch.empty(STREAMS, HEADS, DV, device=dev, dtype=torch.bfloat16)
    for i in range(n):
        ops.gdn_decode_step(q[i % UPDATES], k[i % UPDATES], v[i % UPDATES], g[i % UPDATES], beta[i % UPDATES],
                            states[i % LAYERS], out)
    torch.cuda.synchronize(dev)
    print(f"profile: {n} gdn_decode_step launches done")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cpu-updates", type=int, default=256, help="updates in the CPU-baseline sample")
    ap.add_argument("--profile-launches", type=int, default=0,
                    help="only run this many eager launches of the dominant kernel (for an ncu capture) and exit")
    args = ap.parse_args()
    if args.profile_launches:
        profile_launches(args.profile_launches)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = dist_env()

    if args.impl == "reference":
        if rank != 0:
            return
        per_step_updates = 16
        value, threads, dt = cpu_reference(per_step_updates * (args.steps + args.warmup))
        sample = (f"{per_step_updates} of the 512 updates per step (x{args.steps + args.warmup} steps incl. warm-up), "
                  f"64 streams x 16 heads, {dt:.1f} s")
        line = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded cfg2 distributions)",
            "config": {"workload": "cfg2 gated-DeltaNet recurrent decode: 64 streams x 16 heads, dk=dv=128"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return

    dist = init_dist(world, local)
    try:
        line = run_ours(args, dist, rank, world, local)
        if rank == 0:
            cpu_value, threads, dt = cpu_reference(args.cpu_updates)
            line["cpu_baseline"] = {
                "value": cpu_value, "unit": UNIT, "cores": threads, "kind": "port",
                "sample": f"{args.cpu_updates} sequential updates of 64 streams x 16 heads ({dt:.1f} s), "
                          "oracle/gdn.py restating lm.py:576-582",
            }
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
