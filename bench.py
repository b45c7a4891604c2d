"""Benchmark of the ZONOS3-Mini hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Default workload (the benchmark's config 5, "cfg5"): the decode step of the 24-layer hybrid LM (hidden 2048; 18 gated-
DeltaNet layers of 16 heads at 128/128 and 6 GQA layers of 16 q / 4 kv heads at 128 in the 3:1 pattern; an MoE FFN
of 64 experts, top-8, SwiGLU 768 in every layer; Full AttnRes; a 10-codebook head over 4098 ids) for 256 concurrent
streams per GPU, run through the package's public API: ``Zonos3ForCausalLM`` and its captured ``DecodeGraph``
(embedding -> 49 AttnRes routes and 48 sublayers -> head GEMM -> soft cap + TTS sampler -> the next step's ids).
An audio token is one decode step of one stream (one 10-code frame); value = 256 x K x N / max-over-ranks time.

The 1500-step generation of the config runs from the middle of its cache (878 keys: the 128-token prompt and 750
decode steps) and each replay appends one more key per stream, as a decode loop does. Weights are random-init
(N(0, 0.02)), generated on the device; the KV cache, DeltaNet states and conv histories are random too. Each step
reads 15.6 GB of weights, far more than the 126 MB L2, so no flush is needed between steps.

``value``: graph replays only (ids, metadata, codes stay on the device; each replay feeds its codes back).
``e2e``: ``DecodeGraph.step()`` per step: the ids and the attention metadata copied in from pinned host memory, the
sampled codes copied back and the host synchronised before the next step's ids are built from them.

Multi-GPU: one process per GPU (torchrun), each rank runs its own 256-stream replica (request sharding, no collective
on the data path; weak scaling); the only collectives are the barrier and the max-reduction of the timings.

``--impl reference`` times the reference's CPU implementation of the same step: the oracle port of Zonos3LM.forward
(model/src/zonos3/reference/lm.py:660-735, restated in oracle/lm.py) on the host cores, one stream at a time (the
reference processes one sequence per call) on a 4-layer slice of the cfg5 model and on its 0-layer remainder
(embedding, final route, head), scaled to 24 layers.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "audio tokens/sec per box"
UNIT = "tokens/s"

# cfg5
D5, LAYERS5 = 2048, 24
GDN_H, GDN_D = 16, 128
HQ, HKV, HD = 16, 4, 128
E5, K5, I5 = 64, 8, 768
CODEBOOKS, CODEBOOK_SIZE, TEXT_VOCAB = 10, 4096, 8192
STREAMS5, PROMPT5, DECODE5 = 256, 128, 1500
CONTEXT5 = PROMPT5 + DECODE5 // 2  # keys cached before the first timed step's new row
MAX_LEN5 = PROMPT5 + DECODE5
SAMPLING5 = dict(temperature=0.8, top_k=50, top_p=0.9, min_p=0.0, repetition_window=32, repetition_penalty=1.2)

# cfg2 (operator line)
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



# --------------------------------------------------------------------------------------------- cfg2 inputs


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


# --------------------------------------------------------------------------------------------- cfg5 decode step


def cfg5_model_config(pkg, layers: int = LAYERS5):
    return pkg.config.ModelConfig(
        hidden_size=D5, num_layers=layers, gdn_num_heads=GDN_H, gdn_head_dim=GDN_D, moe_n_experts=E5, moe_topk=K5,
        moe_intermediate_size=I5, moe_start_from_layer=0, norm_topk_prob=True, use_training_router_weights=True,
        attention_pattern="gdn3_global1", num_qo_heads=HQ, num_kv_heads=HKV, head_dim=HD, n_codebooks=CODEBOOKS,
        codebook_size=CODEBOOK_SIZE, text_vocab=TEXT_VOCAB, audio_pad_id=CODEBOOK_SIZE + 1, loss_softcap=15.0)


def cfg5_page_table(streams: int, device, prompt: int = PROMPT5, max_len: int = MAX_LEN5):
    """Slots as a token pool hands them out: each prompt one contiguous block, then every decode step one slot per
    stream (a stream's decode keys sit `streams` slots apart). Returns (page_table [streams, max_len] int32,
    number of slots)."""
    b = torch.arange(streams, dtype=torch.int64)[:, None]
    pos = torch.arange(max_len, dtype=torch.int64)[None, :]
    table = torch.where(pos < prompt, b * prompt + pos, streams * prompt + (pos - prompt) * streams + b)
    return table.to(torch.int32).to(device), streams * max_len


def random_init_(model, seed: int, device) -> None:
    """Seeded random init on the device, as oracle/lm.py random_weights draws it: matrices N(0, 0.02^2), conv
    weights N(0, 0.3^2), norm weights and |temp| 1, A_log = dt_bias = balancing biases = 0."""
    gen = torch.Generator(device=device).manual_seed(seed)
    for name, t in model.state_dict().items():
        if name.endswith(("norm.weight", "rmsnorm_eda.weight", "out_weight", ".temp")):
            t.fill_(1.0)
        elif name.endswith(("A_log", "dt_bias", "balancing_biases")):
            t.zero_()
        elif name.endswith("conv.weight"):
            t.normal_(0.0, 0.3, generator=gen)
        else:
            t.normal_(0.0, 0.02, generator=gen)


def build_cfg5(pkg, dev, streams: int = STREAMS5, layers: int = LAYERS5, seed: int = 0, context: int = CONTEXT5):
    """The cfg5 model with random weights, its caches at `context` cached keys per stream (random KV rows,
    DeltaNet states N(0, 0.01^2), conv histories N(0, 1)), and its captured decode step. Returns (model, graph)."""
    cfg = cfg5_model_config(pkg, layers)
    with torch.device(dev):
        model = pkg.model.Zonos3ForCausalLM(cfg)
    model.to(dev, torch.bfloat16)
    random_init_(model, seed, dev)
    table, kv_slots = cfg5_page_table(streams, dev)
    pool = model.allocate_caches(streams, kv_slots, dev)
    sampling = pkg.model.SamplingConfig(seed=seed, **SAMPLING5)
    graph = pkg.model.DecodeGraph(model, pool, streams, table, sampling=sampling)
    graph.capture()
    gen = torch.Generator(device=dev).manual_seed(seed + 1)
    pool.k_buffer.normal_(generator=gen)
    pool.v_buffer.normal_(generator=gen)
    for gdn in model.gdn_layers():
        gdn._recurrent_state.normal_(0.0, 0.01, generator=gen)
        gdn._conv_state.normal_(generator=gen)
    ids = torch.randint(0, CODEBOOK_SIZE, (streams, CODEBOOKS + 1), generator=gen, device=dev, dtype=torch.int32)
    ids[:, -1] = TEXT_VOCAB  # the text column of a decode row: the text pad id
    graph.load(ids, torch.full((streams,), context, dtype=torch.int32, device=dev),
               torch.full((streams,), context + 1, dtype=torch.int32, device=dev), table[:, context].contiguous())
    torch.cuda.synchronize(dev)
    return model, graph


def cfg5_step_bytes(streams: int, context: int, layers: int = LAYERS5) -> int:
    """Algorithmic bytes of one cfg5 decode step, each read or write counted once: every expert's weights (2048
    routed pairs over 64 experts touch all of them) and the router weights; per DeltaNet layer the in_proj / wo
    weights, the fp32 states and bf16 conv histories read and written; per GQA layer the projection weights and the
    K / V rows of `context` + 1 keys (and their page-table entries); the AttnRes bank (route r reads r + 1 rows and
    writes one); the embedding rows, the head weights and the bf16 logits written and read back."""
    inner = GDN_H * GDN_D
    n_gqa = layers // 4
    n_gdn = layers - n_gqa
    keys = context + 1
    moe = layers * (E5 * 3 * I5 * D5 * 2 + E5 * D5 * 2)
    gdn = n_gdn * (((4 * inner + 2 * GDN_H) * D5 + D5 * inner) * 2 + streams * GDN_H * GDN_D * GDN_D * 4 * 2
                   + streams * 3 * inner * 3 * 2 * 2)
    gqa = n_gqa * (((HQ * HD + 2 * HKV * HD + HQ) * D5 + D5 * HQ * HD) * 2 + streams * keys * (HKV * HD * 2 * 2 + 4))
    routes = 2 * layers + 1
    attnres = sum(r + 2 for r in range(routes)) * streams * D5 * 2
    vocab = CODEBOOKS * (CODEBOOK_SIZE + 2)
    head = streams * (CODEBOOKS + 1) * D5 * 2 + vocab * D5 * 2 + 2 * streams * vocab * 2
    return moe + gdn + gqa + attnres + head


def cfg5_config(world: int) -> dict:
    return {
        "workload": "cfg5 decode step, one CUDA graph: embedding, 24 layers (18 DeltaNet + 6 GQA, MoE 64 x top-8, "
                    "Full AttnRes), head + soft cap, TTS sampler",
        "model": "ZONOS3-Mini cfg5 (random init, 7.9 B params)",
        "streams_per_gpu": STREAMS5, "global_batch": STREAMS5 * world, "seq_len": MAX_LEN5,
        "context_start": CONTEXT5, "layers": LAYERS5, "token": "one decode step of one stream",
        "l2": "no flush (15.6 GB of weights per step)",
        "parallelism": f"replicas x{world}",
    }


def run_ours(args, dist, rank, world, local):
    pkg = __import__("__graft_entry__").load_package()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    model, graph = build_cfg5(pkg, dev, seed=1234 + rank)
    stream = torch.cuda.Stream(dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    total_steps = args.warmup + args.steps + args.warmup + args.e2e_steps
    if CONTEXT5 + 1 + total_steps > MAX_LEN5:
        raise SystemExit(f"{total_steps} steps would run past the {MAX_LEN5}-key cache")
    with torch.cuda.stream(stream):
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
    status = pkg.ops.device_status()

    # end to end through DecodeGraph.step: host ids + metadata in, codes out, host synchronised every step (the
    # next step's ids are the codes just read back)
    pos0 = int(graph.positions[0].item())
    table = graph.page_table.cpu()
    n_e2e = args.e2e_steps
    host_ids = graph.input_ids.cpu().pin_memory()
    host_codes = torch.empty(STREAMS5, CODEBOOKS + 1, dtype=torch.int32).pin_memory()
    meta = []
    for i in range(args.warmup + n_e2e):
        p = pos0 + i
        meta.append((torch.full((STREAMS5,), p, dtype=torch.int32).pin_memory(),
                     torch.full((STREAMS5,), p + 1, dtype=torch.int32).pin_memory(),
                     table[:, p].contiguous().pin_memory()))
    h2d = host_ids.numel() * 4 + sum(t.numel() * 4 for t in meta[0])
    d2h = host_codes.numel() * 4

    def e2e_step(i):
        graph.step(host_ids, host_codes, *meta[i])
        torch.cuda.current_stream(dev).synchronize()
        host_ids.copy_(host_codes[:, : host_ids.shape[1]])
        host_ids[:, -1] = TEXT_VOCAB

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            e2e_step(i)
        barrier(dist)
        torch.cuda.synchronize(dev)
        e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for i in range(n_e2e):
            e2e_step(args.warmup + i)
        e_stop.record(stream)
        torch.cuda.synchronize(dev)
        barrier(dist)
    e2e_ms = max_over_ranks(dist, e_start.elapsed_time(e_stop))

    strong = strong_scaling(pkg, model, graph, dist, rank, world, dev, stream, args) if world > 1 else None

    step_ms = elapsed_ms / args.steps
    context_mid = CONTEXT5 + args.warmup + args.steps // 2
    nbytes = cfg5_step_bytes(STREAMS5, context_mid)
    pk = peaks()
    achieved = nbytes / (step_ms / 1e3) / 1e9
    line = {
        "metric": METRIC,
        "value": STREAMS5 * args.steps * world / (elapsed_ms / 1e3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init weights, random caches, sampled codes fed back)",
        "config": cfg5_config(world),
        "roofline": {
            "kernel": "decode step (one graph)", "bound": "hbm", "achieved": achieved,
            "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
            "traffic": profiled_traffic("decode_step_cfg5.md"), "algorithmic_bytes_per_step": nbytes,
            "peak_source": pk["source"],
        },
        "e2e": {"value": STREAMS5 * n_e2e * world / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms / n_e2e,
                "path": "DecodeGraph.step: host ids in, codes out, sync per step"},
        "strong_scaling": strong,
        "gpu_launches": graph.launches_per_step * args.steps,
        "launches_per_step": graph.launches_per_step,
        "device_status": status,
        "clocks": clocks.summary(),
    }
    del graph, model
    torch.cuda.empty_cache()
    return line


def strong_scaling(pkg, model, graph, dist, rank, world, dev, stream, args) -> dict:
    """The config's 256 streams split over the ranks (replicas.shard: a contiguous share per GPU), each rank's share
    decoded by its own captured step on the same model and caches; timed like the weak-scaling value (max over
    ranks). Under strong scaling every GPU still reads all 15.6 GB of weights per step, so the box throughput grows
    far slower than the GPU count."""
    share = pkg.replicas.shard(STREAMS5, world, rank)
    n = len(share)
    table, _ = cfg5_page_table(n, dev)
    sampling = pkg.model.SamplingConfig(seed=7 + rank, **SAMPLING5)
    sub = pkg.model.DecodeGraph(model, graph.pool, n, table, sampling=sampling)
    sub.capture()
    ids = graph.input_ids[:n].clone()
    pos = graph.positions[:n].clone()
    sub.load(ids, pos, pos + 1, table[torch.arange(n, device=dev), pos.long()].contiguous())
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            sub.replay()
        torch.cuda.synchronize(dev)
        barrier(dist)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            sub.replay()
        b.record(stream)
        torch.cuda.synchronize(dev)
        barrier(dist)
    ms = max_over_ranks(dist, a.elapsed_time(b))
    del sub
    # per GPU: the share's algorithmic bytes (all expert weights are still read) against the HBM copy peak
    step_s = ms / args.steps / 1e3
    nbytes = cfg5_step_bytes(STREAMS5 // world, CONTEXT5)
    pk = peaks()
    return {"streams_total": STREAMS5, "streams_per_gpu": STREAMS5 // world, "ms_per_step": ms / args.steps,
            "value": STREAMS5 * args.steps / (ms / 1e3), "unit": UNIT,
            "per_gpu_roofline": {"bound": "hbm", "bytes_per_step": nbytes, "achieved": nbytes / step_s / 1e9,
                                 "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": nbytes / step_s / 1e9 / pk["hbm_gbs"],
                                 "limiter": "every GPU reads all 15.6 GB of weights per step whatever its share of "
                                            "streams; at small shares the latency of the step's ~240 launches"}}


# --------------------------------------------------------------------------------------------- CPU reference


def cfg5_oracle_config(layers: int):
    from oracle import lm as olm

    return olm.LMConfig(dim=D5, n_layers=layers, gdn_period=4, gdn_heads=GDN_H, gdn_head_dim=GDN_D, n_heads=HQ,
                        n_kv_heads=HKV, head_dim=HD, n_experts=E5, topk=K5, moe_hidden=I5, moe_routed_dim=D5,
                        n_codebooks=CODEBOOKS, codebook_size=CODEBOOK_SIZE, text_rows=TEXT_VOCAB + 1)


def cpu_reference_cfg5(samples: int, seed: int = 99):
    """Time the reference's CPU forward (oracle/lm.py restating Zonos3LM.forward, lm.py:660-735, fp32) for one
    stream's decode step at cfg5 shapes on this host's cores, from a cache of CONTEXT5 keys: `samples` steps of a
    4-layer slice (3 DeltaNet + 1 GQA, one period of the 3:1 pattern) and of the 0-layer remainder (embedding,
    final route, head). One 24-layer stream-step = t0 + 24 x (t4 - t0) / 4. Returns (tokens/s, threads, seconds,
    per-stream-step seconds)."""
    from oracle import lm as olm

    torch.set_num_threads(os.cpu_count() or 1)
    c4 = cfg5_oracle_config(4)
    w4 = olm.random_weights(c4, seed)
    c0 = dataclasses.replace(c4, n_layers=0)
    w0 = {k: v for k, v in w4.items() if not k.startswith("layers.")}
    w0["block_attnres_queries"] = w4["block_attnres_queries"][-1:]
    gen = torch.Generator().manual_seed(seed + 1)

    def cache(c):
        cc = olm.Cache(position=CONTEXT5)
        for layer in range(c.n_layers):
            if c.uses_gdn(layer):
                cc.gdn_state[layer] = 0.01 * torch.randn(GDN_H, GDN_D, GDN_D, generator=gen)
                cc.conv_state[layer] = torch.randn(3 * GDN_H * GDN_D, 3, generator=gen)
            else:
                cc.kv[layer] = (torch.randn(CONTEXT5, HKV, HD, generator=gen), torch.randn(CONTEXT5, HKV, HD, generator=gen))
        return cc

    caches = (cache(c4), cache(c0))
    ids = torch.randint(0, CODEBOOK_SIZE, (1, CODEBOOKS + 1), generator=gen)
    ids[:, -1] = TEXT_VOCAB
    times = [0.0, 0.0]
    t_all = time.perf_counter()
    with torch.no_grad():
        for i in range(samples + 1):  # the first sample of each model is a warm-up
            for j, (c, w) in enumerate(((c4, w4), (c0, w0))):
                t0 = time.perf_counter()
                olm.forward(c, w, ids, caches[j])
                if i:
                    times[j] += time.perf_counter() - t0
    t4, t0 = times[0] / samples, times[1] / samples
    per_step = t0 + LAYERS5 * (t4 - t0) / 4
    return 1.0 / per_step, torch.get_num_threads(), time.perf_counter() - t_all, per_step


# --------------------------------------------------------------------------------------------- cfg2 operator


def bench_gdn_decode_cfg2(ops, dev, stream, reps=3):
    """cfg2: 512 sequential single-token gated-DeltaNet updates of 64 streams x 16 heads at 128/128 with per-step
    outputs, cycling 4 independent layer states (256 MB > L2, as each layer owns its state in the model); one CUDA
    graph of the 2048 launches."""
    q, k, v, g, beta = cfg2_inputs(1234, dev)
    states = [cfg2_state(1235 + l, dev) for l in range(LAYERS)]
    outs = torch.empty(LAYERS, UPDATES, STREAMS, HEADS, DV, device=dev, dtype=torch.bfloat16)

    def run():
        for t in range(UPDATES):
            for l in range(LAYERS):
                ops.gdn_decode_step(q[t], k[t], v[t], g[t], beta[t], states[l], outs[l, t])

    ms = graph_ms(run, stream, reps=reps, warmup=2)
    launches = UPDATES * LAYERS
    launch_s = ms / 1e3 / launches
    nbytes = bytes_per_update()
    pk = peaks()
    return {"workload": "cfg2 gated-DeltaNet recurrent decode: 64 streams x 16 heads, dk=dv=128, 512 updates x 4 "
                        "layer states",
            "ms": ms, "updates_per_s": STREAMS * launches / (ms / 1e3),
            "roofline": {"kernel": "gdn_decode_kernel<128>", "bound": "hbm", "achieved": nbytes / launch_s / 1e9,
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": nbytes / launch_s / 1e9 / pk["hbm_gbs"],
                         "traffic": profiled_traffic("gdn_decode_cfg2.md"), "algorithmic_bytes_per_launch": nbytes,
                         "avg_launch_us": launch_s * 1e6, "peak_source": pk["source"]}}


# --------------------------------------------------------------------------------------------- operator timings


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


class L2Flush:
    """Reads a 256 MB buffer (twice the 126 MB L2) so the next kernel starts from HBM. A read leaves clean lines
    behind, so the timed kernel pays no write-back of the flush (a write-based flush would)."""

    def __init__(self, dev):
        self.buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)
        self.out = torch.empty(1, dtype=torch.float32, device=dev)

    def __call__(self):
        torch.sum(self.buf, dim=0, keepdim=True, out=self.out)


def flush_l2(flush) -> None:
    flush()


def moe_cfg4_inputs(dev, seed=4):
    """cfg4: 4096 tokens x hidden 2048 bf16 N(0,1); router N(0,0.02) [64, 2048]; 64 SwiGLU experts, I=768,
    bf16 weights N(0,0.02)."""
    T, D, E, I = 4096, 2048, 64, 768
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(T, D, generator=gen).bfloat16()
    norm_w = torch.ones(D).bfloat16()
    w_r = (0.02 * torch.randn(E, D, generator=gen)).bfloat16()
    gate_up = (0.02 * torch.randn(E, 2 * I, D, generator=gen)).bfloat16()
    down = (0.02 * torch.randn(E, D, I, generator=gen)).bfloat16()
    return [t.to(dev) for t in (x, norm_w, w_r, gate_up, down)]


def graph_ms(fn, stream, reps=5, warmup=2) -> float:
    """Milliseconds per call of fn() captured in a CUDA graph and replayed `reps` times between two events on
    `stream` (no host work inside the timed region)."""
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            fn()
        for _ in range(warmup):
            graph.replay()
        a, b = _events()
        a.record(stream)
        for _ in range(reps):
            graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
    del graph
    return a.elapsed_time(b) / reps


def flushed_ms(fn, flush, stream, reps=5) -> float:
    """Device time of fn() starting from a cold L2: graph[flush, fn] minus graph[flush]."""
    return graph_ms(lambda: (flush_l2(flush), fn()), stream, reps) - graph_ms(lambda: flush_l2(flush), stream, reps)


def bench_moe_cfg4(ops, dev, stream, steps=10, warmup=3):
    """The MoE layer of cfg4 (router -> permutation -> gather -> GEMM1+SwiGLU -> GEMM2*w -> combine) as one CUDA
    graph, plus each kernel's device time from a cold L2 (graph of [flush, kernel] minus graph of [flush])."""
    x, norm_w, w_r, gate_up, down = moe_cfg4_inputs(dev)
    T, D = x.shape
    E, two_i, _ = gate_up.shape
    I, k = two_i // 2, 8
    ws = ops.MoEWorkspace(T, k, E, D, I, dev)
    out = torch.empty(T, D, device=dev, dtype=torch.bfloat16)
    flush = L2Flush(dev)

    def router():
        ops.moe_router(x, norm_w, 1e-5, w_r, None, k, weights="full_softmax", renormalize=True, ids=ws.ids,
                       topk_weights=ws.weights)

    def permute():
        ops.moe_permute(ws.ids, E, capacity=ws.capacity, out=ws.perm)

    def gather():
        ops.moe_gather(x, ws.perm["sorted_pairs"], k, ws.x_perm)

    def gemm1():
        ops.moe_gemm_swiglu(ws.x_perm, gate_up, ws.perm["offsets"], ws.h, counts=ws.perm["counts"])

    def gemm2():
        ops.moe_gemm_down(ws.h, down, ws.perm["offsets"], ws.perm["sorted_pairs"], ws.weights, ws.y,
                          counts=ws.perm["counts"])

    def combine():
        ops.moe_combine(ws.y, k, out)

    parts = [("router", router), ("permute", permute), ("gather", gather), ("gemm_swiglu", gemm1),
             ("gemm_down", gemm2), ("combine", combine)]

    def layer():
        for _, fn in parts:
            fn()

    layer_ms = graph_ms(layer, stream, reps=steps, warmup=warmup)
    per = {name: flushed_ms(fn, flush, stream) for name, fn in parts}
    status = ops.device_status()
    pk = peaks()
    pairs = T * k
    f1, f2 = 2 * pairs * D * 2 * I, 2 * pairs * I * D
    gemm_ms = per["gemm_swiglu"] + per["gemm_down"]
    tflops = (f1 + f2) / (gemm_ms / 1e3) / 1e12
    return {
        "workload": "cfg4 MoE layer: 4096 tokens x 2048, top-8 of 64 experts, SwiGLU I=768 (router, permutation, "
                    "gather, grouped GEMMs, combine)",
        "ms_per_layer": layer_ms, "tokens_per_s": T / (layer_ms / 1e3),
        "kernel_ms_cold_l2": per,
        "roofline": {"kernel": "moe_gemm_kernel (SwiGLU + Down)", "bound": "tensor", "achieved": tflops,
                     "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": tflops / pk["bf16_tflops"],
                     "flops_per_layer": f1 + f2, "peak_source": pk["source"] + " burst"},
        "cpu_baseline": dict(zip(("ms_per_layer", "cores", "sample"), cpu_moe_cfg4()), kind="port",
                             path="oracle/moe.py router + experts_loop_fp32 (lm.py:610-637)"),
        "gemm_swiglu_tflops": f1 / (per["gemm_swiglu"] / 1e3) / 1e12,
        "gemm_down_tflops": f2 / (per["gemm_down"] / 1e3) / 1e12,
        "device_status": status,
    }


def cpu_moe_cfg4(tokens: int = 64):
    """The reference's CPU MoE layer (lm.py:610-637: router GEMM and top-k, then the per-(token, rank) expert loop,
    restated in oracle/moe.py) on `tokens` of cfg4's 4096 tokens, fp32 on this host's cores; the layer time is
    scaled by 4096 / tokens (tokens are independent). Returns (ms per 4096-token layer, threads, sample)."""
    from oracle import moe as omoe

    torch.set_num_threads(os.cpu_count() or 1)
    x, norm_w, w_r, gate_up, down = [t.float() for t in moe_cfg4_inputs("cpu")]
    x = x[:tokens]
    with torch.no_grad():
        omoe.experts_loop_fp32(x[:1], gate_up, down, torch.zeros(1, 8, dtype=torch.int64), torch.ones(1, 8))
        t0 = time.perf_counter()
        logits = omoe.router_logits(x, norm_w, w_r, 1e-5)
        ids, w = omoe.route(logits, torch.zeros(w_r.shape[0]), 8, weights="full_softmax", renormalize=True)
        omoe.experts_loop_fp32(x, gate_up, down, ids, w)
        dt = time.perf_counter() - t0
    ms = dt * 1e3 * 4096 / tokens
    return ms, torch.get_num_threads(), f"{tokens} of the 4096 tokens ({dt:.2f} s), scaled by {4096 // tokens}"


def bench_attnres_decode(ops, dev, stream, tokens=256, dim=2048, layers=24, reps=3):
    """cfg5's AttnRes schedule for one decode step: 2L+1 routes over a growing bank (S = 1 .. 2L+1 sources) of
    `tokens` rows, each with the following RMSNorm fused, as FusedBlockAttnResContext runs them with the forward's
    queries registered: route r reads the logits of rows < r from the table, computes its current source's (bank
    row r) and, while it mixes, route r+1's logits of rows <= r. Before every route the L2 is flushed (as the
    sublayer between two routes does with its weight streams) and then the current source row is rewritten by a copy
    kernel: in the model that row is the output of the kernel just before the route, so it is in L2 when the route
    starts, while the older bank rows, the logit table and the queries are not. Route time = graph[flush, copy,
    route] minus graph[flush, copy], summed over the 2L+1 routes. The largest route is also timed with nothing in L2
    (`largest_route_cold`)."""
    gen = torch.Generator().manual_seed(7)
    n_src = 2 * layers + 1
    bank = torch.randn(n_src, tokens, dim, generator=gen).bfloat16().to(dev)
    queries = (0.02 * torch.randn(n_src, dim, generator=gen)).bfloat16().to(dev)
    norm_w = torch.ones(dim, dtype=torch.bfloat16, device=dev)
    out = torch.empty(tokens, dim, device=dev, dtype=torch.bfloat16)
    table = torch.zeros(n_src, tokens, (n_src + 3) // 4 * 4, device=dev, dtype=torch.float32)
    inv_rms = torch.zeros(tokens, (n_src + 3) // 4 * 4, device=dev, dtype=torch.float32)
    staging = bank.clone()  # the producer of each route's current source copies its row from here
    flush = L2Flush(dev)

    def route(r):
        ops.attnres_route_tabled(bank, r, bank[r], queries, r, table, inv_rms, 1e-5, source_in_bank=r < n_src - 1,
                                 norm_weight=norm_w, out=out)

    def schedule(with_routes, only=None):
        for r in range(n_src) if only is None else [only]:
            flush_l2(flush)
            bank[r].copy_(staging[r])
            if with_routes:
                route(r)

    schedule(True)  # fills the table as a forward does
    total_ms = graph_ms(lambda: schedule(True), stream, reps) - graph_ms(lambda: schedule(False), stream, reps)
    big_ms = graph_ms(lambda: schedule(True, n_src - 1), stream, 10) - graph_ms(lambda: schedule(False, n_src - 1),
                                                                                  stream, 10)
    big_cold_ms = flushed_ms(lambda: route(n_src - 1), flush, stream, reps=10)

    # algorithmic bytes of route r: r + 1 bank rows read, the output row written, this and the next route's query
    # and the norm weight, per token the r table logits and r inverse RMS read, the next route's r + 1 logits and
    # the source's inverse RMS written
    def route_bytes(r):
        nxt = r + 1 if r + 1 < n_src else 0
        return ((r + 1) * tokens * dim + tokens * dim + 3 * dim) * 2 + (2 * r + nxt + 1) * tokens * 4

    total_bytes = sum(route_bytes(r) for r in range(n_src))
    pk = peaks()
    gbs = total_bytes / (total_ms / 1e3) / 1e9
    big_bytes = route_bytes(n_src - 1)
    return {
        "workload": f"cfg5 AttnRes decode schedule: {n_src} routes over a growing bank, {tokens} tokens x {dim}, "
                    "fused RMSNorm, L2 flushed before each route and the route's current source then written by "
                    "the kernel before it",
        "ms_per_step": total_ms, "bytes_per_step": total_bytes,
        "roofline": {"kernel": "attnres_tabled_kernel", "bound": "hbm", "achieved": gbs,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"], "peak_source": pk["source"]},
        "largest_route": {"sources": n_src, "us": big_ms * 1e3, "gbs": big_bytes / (big_ms / 1e3) / 1e9,
                          "frac": big_bytes / (big_ms / 1e3) / 1e9 / pk["hbm_gbs"]},
        "largest_route_cold": {"us": big_cold_ms * 1e3, "frac": big_bytes / (big_cold_ms / 1e3) / 1e9 / pk["hbm_gbs"]},
    }


def decode_layer_cfg5(pkg, dev, streams=256, bank_rows=24):
    """Builds the cfg5 DeltaNet + MoE decode layer of bench_decode_layer_cfg5; returns (layer, core, batch): call
    layer() inside core.forward_batch(batch)."""
    ops, core = pkg.ops, pkg.core
    D, H, d, E, k, I = 2048, 16, 128, 64, 8, 768
    cfg = pkg.config.ModelConfig(hidden_size=D, gdn_num_heads=H, gdn_head_dim=d, moe_n_experts=E, moe_topk=k,
                                 moe_intermediate_size=I, norm_topk_prob=True, use_training_router_weights=False)
    gen = torch.Generator().manual_seed(11)
    rnd = lambda *shape, s=0.02: (s * torch.randn(*shape, generator=gen)).bfloat16()  # noqa: E731
    inner = H * d
    gdn = pkg.gdn.OriginalGDN(cfg, 1)
    gdn.load_state_dict({"in_proj.weight": rnd(4 * inner + 2 * H, D), "conv.weight": rnd(3 * inner, 1, 4, s=0.3),
                         "out_weight": torch.ones(d).bfloat16(), "A_log": torch.zeros(H), "dt_bias": torch.zeros(H),
                         "wo.weight": rnd(D, inner)})
    gdn.to(dev, torch.bfloat16)
    gdn.allocate_cache(streams, dev, torch.bfloat16)
    slots = torch.arange(streams, device=dev, dtype=torch.int64)
    gdn.enable_graph_decode(slots, pkg.gdn.OriginalGDN.static_tables(dev, [streams]))
    gdn.set_static_mode(True)
    moe = pkg.moe.MoEFeedForward(cfg, 1)
    moe.load_state_dict({"router.router_linear.weight": rnd(E, D), "router.rmsnorm_eda.weight": torch.ones(D).bfloat16(),
                         "router.balancing_biases": torch.zeros(E), "experts.gate_up_proj": rnd(E, 2 * I, D),
                         "experts.down_proj": rnd(E, D, I)})
    moe.to(dev, torch.bfloat16)
    bank = torch.randn(bank_rows + 2, streams, D, generator=gen).bfloat16().to(dev)
    # the layer's two routes are routes bank_rows and bank_rows + 1 of a forward of 2 * bank_rows + 1 routes (the
    # middle layer of a 2 x bank_rows-sublayer stack), the route queries registered up front
    n_routes = 2 * bank_rows + 1
    queries = (0.02 * torch.randn(n_routes, D, generator=gen)).bfloat16().to(dev)
    norm_w = torch.ones(D, dtype=torch.bfloat16, device=dev)
    table = torch.zeros(n_routes, streams, (n_routes + 3) // 4 * 4, device=dev, dtype=torch.float32)
    inv_rms = torch.ones(streams, (n_routes + 3) // 4 * 4, device=dev, dtype=torch.float32)
    h = torch.empty(streams, D, device=dev, dtype=torch.bfloat16)
    batch = core.Batch(reqs=[core.Req(i, 1, cached_len=100) for i in range(streams)], is_decode=True,
                       padded_size=streams)

    def layer():
        ops.attnres_route_tabled(bank, bank_rows, bank[bank_rows], queries, bank_rows, table, inv_rms, 1e-5,
                                 source_in_bank=True, norm_weight=norm_w, out=h)
        a = gdn.forward(h)
        ops.attnres_route_tabled(bank, bank_rows + 1, a, queries, bank_rows + 1, table, inv_rms, 1e-5,
                                 append_to=bank[bank_rows + 1], norm_weight=norm_w, out=h)
        out, _ = moe.forward(h)
        return out

    return layer, core, batch


def bench_decode_layer_cfg5(pkg, dev, stream, streams=256, bank_rows=24, reps=5):
    """cfg5 decode step of one DeltaNet + MoE layer through the drop-in modules, for `streams` concurrent streams
    (one new row each): AttnRes route (bank of `bank_rows` sources + the layer input, attention_norm fused) ->
    OriginalGDN.forward in its static decode mode (in_proj GEMM, prologue, recurrent update of 256 slot states,
    gated norm, wo GEMM) -> AttnRes route (ffn_norm fused) -> MoEFeedForward.forward (router, permutation,
    grouped GEMMs over 604 MB of expert weights, combine). Hidden 2048, GDN 16 x 128/128, 64 experts top-8, I=768;
    bf16 random-init weights (N(0, 0.02)); captured in one CUDA graph. The L2 is not flushed: the expert weights
    alone exceed it."""
    D, E, I = 2048, 64, 768
    layer, core, batch = decode_layer_cfg5(pkg, dev, streams, bank_rows)
    with core.forward_batch(batch):
        ms = graph_ms(layer, stream, reps)
    return {
        "workload": f"cfg5 DeltaNet + MoE layer decode step: {streams} streams x hidden {D}; AttnRes route over "
                    f"{bank_rows + 1} sources before each sublayer; GDN 16 x 128/128 recurrent update; MoE 64 experts "
                    "top-8, I=768 (604 MB of expert weights); CUDA graph of one layer",
        "layer_ms": ms, "layer_tokens_per_s": streams / (ms / 1e3),
        "expert_weight_bytes": E * 3 * I * D * 2,
    }



def bench_sampler_cfg5(ops, dev, stream, streams=256, codebooks=10, vocab=4098, reps=5):
    """The TTS sampler for a cfg5 decode step: fp32 logits [256, 10, 4098] (N(0, 3)), temperature 0.8, top-k 50,
    top-p 0.9, a 32-step repetition window with penalty 1.2; one row per CTA. The 42 MB of logits stay in L2 between
    replays (as the head GEMM leaves them there)."""
    gen = torch.Generator().manual_seed(8)
    logits = (3 * torch.randn(streams, codebooks, vocab, generator=gen)).to(dev)
    rep = torch.randint(0, vocab, (streams, codebooks, 32), generator=gen, dtype=torch.int32).to(dev)
    pen = torch.full((streams,), 1.2, device=dev)
    stop = torch.full((streams,), vocab - 2, dtype=torch.int32, device=dev)
    temps = torch.full((streams,), 0.8)
    temps_d = temps.to(dev)
    out = torch.empty(streams, codebooks + 1, device=dev, dtype=torch.int32)

    def sample():
        ops.sample_tts(logits, temps, [50], [0.9], [0.0], codebook_size=vocab - 2, audio_pad_id=vocab - 1,
                       stop_token_ids=stop, repetition_token_ids=rep, repetition_penalties=pen, seed=1, out=out,
                       device_temperatures=temps_d)

    ms = graph_ms(sample, stream, reps)
    return {"workload": f"TTS sampler: {streams} streams x {codebooks} codebooks x {vocab} ids, fp32 logits, "
                        "temperature 0.8, top-k 50, top-p 0.9, repetition window 32",
            "us": ms * 1e3, "rows_per_s": streams * codebooks / (ms / 1e3)}


def vocoder_inputs(streams: int, frames: int, seed: int = 12):
    """Head frames of the codec's two iSTFT branches (n_fft 736 / 2208, hop 184): log-magnitudes N(-3, 1.5), phases
    U(-pi, pi), float32 [streams, frames, n + 2]; periodic Hann windows, a 127-tap mixer, the 44160 -> 44100 Hz sinc
    kernel."""
    from oracle.istft import sinc_resample_kernel  # the kernel's construction only; nothing timed runs the oracle

    rng = np.random.default_rng(seed)
    ys = []
    for n in (736, 2208):
        bins = n // 2 + 1
        ys.append(np.concatenate([rng.normal(-3.0, 1.5, (streams, frames, bins)),
                                  rng.uniform(-np.pi, np.pi, (streams, frames, bins))], -1).astype(np.float32))
    windows = [torch.hann_window(n, periodic=True).numpy() for n in (736, 2208)]
    mixer = rng.normal(0, 0.05, (2, 127)).astype(np.float32)
    mixer[0, 63] += 1.0
    kernel, width, orig, new = sinc_resample_kernel(44160, 44100, 16, 0.99)
    return ys, windows, mixer, (kernel, orig, new, width)


def bench_vocoder_tail(pkg, dev, streams=256, frames=240, chunk=4, reps=3):
    """The codec's DSP tail (two-branch iSTFT head + FIR mixer + 44.1 kHz resampler, float64) for 256 lock-step streams
    and one second of audio each (240 head frames): pushed at once, and pushed 4 frames at a time as a streaming decode
    does (also end to end as the codec's stream runs: the frames are the trunk's output on the device, each push's
    samples are read back to the host); fresh streams each rep, timed with CUDA events from the first push to the
    flush."""
    voc = pkg.vocoder
    ys, windows, mixer, (kernel, orig, new, width) = vocoder_inputs(streams, frames)
    y0, y1 = (torch.from_numpy(y).to(dev) for y in ys)

    def run(step, host=False):
        head = voc.IstftHeadStream((736, 2208), 184, windows, mixer, math.log(100.0), dev, streams=streams,
                                   max_cols=step)
        res = voc.ResamplerStream(kernel, orig, new, width, dev, streams=streams)
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        n, outs = 0, []
        for c0 in range(0, frames, step):
            o = res.push(head.push(y0[:, c0:c0 + step], y1[:, c0:c0 + step]))
            outs.append(o.to("cpu", non_blocking=True) if host else o)  # e2e: each push's samples read back
        outs += [res.push(head.flush()), res.flush()]
        if host:
            outs[-2:] = [o.to("cpu", non_blocking=True) for o in outs[-2:]]
        end.record()
        torch.cuda.synchronize(dev)
        n = sum(o.shape[1] for o in outs)
        return start.elapsed_time(end), n

    out = {"workload": f"codec DSP tail: {streams} streams x {frames} head frames (1 s of 44.1 kHz audio each), "
                       "n_fft 736 + 2208, hop 184, 127-tap mixer, 736 -> 735 sinc resampler (770 taps), float64"}
    for label, step in (("bulk", frames), ("stream4", chunk)):
        run(step)
        ms = min(run(step)[0] for _ in range(reps))
        samples = run(step)[1]
        out[label] = {"ms": ms, "samples_per_s": streams * samples / (ms / 1e3),
                      "realtime_x": streams * samples / 44100 / (ms / 1e3)}
    run(chunk, host=True)
    ms = min(run(chunk, host=True)[0] for _ in range(reps))
    samples = run(chunk, host=True)[1]
    out["stream4_e2e"] = {"ms": ms, "samples_per_s": streams * samples / (ms / 1e3),
                          "realtime_x": streams * samples / 44100 / (ms / 1e3),
                          "h2d_bytes": 0, "d2h_bytes": streams * samples * 4}
    out["ms"] = out["bulk"]["ms"]
    out["cpu_baseline"] = cpu_vocoder_tail(ys, windows, mixer, (kernel, orig, new, width), streams)
    return out


def cpu_vocoder_tail(ys, windows, mixer, res_args, streams, sample_streams=4):
    """The oracle's whole-signal decode (NumPy float64: irfft per frame, overlap-add, mixer, resampler) of a few of the
    same streams, timed on one host thread and scaled to all streams."""
    from oracle import istft

    kernel, orig, new, width = res_args
    t0 = time.perf_counter()
    for s in range(sample_streams):
        full = istft.istft_decode(ys[0][s], ys[1][s], (736, 2208), 184, windows, mixer, math.log(100.0))
        istft.resample(full.astype(np.float32), kernel, orig, new, width, -(-new * len(full) // orig))
    dt = time.perf_counter() - t0
    return {"ms_per_layer": dt / sample_streams * streams * 1e3, "sample_streams": sample_streams, "cores": 1,
            "kind": "port"}


def gqa_cfg5_inputs(dev, streams=256, prompt=128, context=1628, Hq=16, Hkv=4, hd=128, seed=5):
    """cfg5 global-attention decode at the end of the run: `streams` requests, each with `context` cached keys
    (the 128-token prompt, then 1500 decode steps). Slots as a token pool hands them out: each prompt a contiguous
    block, then every decode step one slot per request (so a request's decode keys sit `streams` slots apart).
    K/V N(0,1) bf16; q N(0,1) bf16."""
    gen = torch.Generator().manual_seed(seed)
    slots = streams * context
    b = torch.arange(streams, dtype=torch.int64)[:, None]
    pos = torch.arange(context, dtype=torch.int64)[None, :]
    table = torch.where(pos < prompt, b * prompt + pos, streams * prompt + (pos - prompt) * streams + b)
    k_cache = torch.randn(slots, Hkv, hd, generator=gen).bfloat16().to(dev)
    v_cache = torch.randn(slots, Hkv, hd, generator=gen).bfloat16().to(dev)
    q = torch.randn(streams, Hq, hd, generator=gen).bfloat16().to(dev)
    seq = torch.full((streams,), context, dtype=torch.int32, device=dev)
    return q, k_cache, v_cache, table.to(torch.int32).to(dev), seq


def bench_gqa_decode_cfg5(ops, dev, stream, reps=5):
    """cfg5 GQA decode attention (16 q / 4 kv heads at 128) for 256 streams at 1628 cached keys: 853 MB of K/V per
    call, above L2, so replays need no flush. Unsplit (the reference's setting for this model) and with the
    automatic split."""
    streams, context, Hq, Hkv, hd = 256, 1628, 16, 4, 128
    q, kc, vc, table, seq = gqa_cfg5_inputs(dev, streams, 128, context, Hq, Hkv, hd)
    out = torch.empty_like(q)
    nbytes = streams * context * Hkv * hd * 2 * 2 + table.numel() * 4 + 2 * q.numel() * 2
    pk = peaks()
    res = {"workload": f"cfg5 GQA decode attention: {streams} streams x {context} cached keys, {Hq} q / {Hkv} kv "
                       f"heads at {hd}; slot-indexed cache (prompt blocks, then interleaved decode slots)",
           "algorithmic_bytes": nbytes}
    for name, splits in (("unsplit", 1), ("auto", 0), ("split2", 2)):
        s, _ = ops.gqa_splits(streams, Hkv, context, splits, hd)
        ws = torch.empty(streams * Hq * s * (hd + 2), device=dev, dtype=torch.float32)
        ms = graph_ms(lambda: ops.gqa_decode(q, kc, vc, table, seq, num_splits=splits, out=out, workspace=ws),
                      stream, reps)
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"splits": s, "us": ms * 1e3, "achieved_gbs": gbs, "frac": gbs / pk["hbm_gbs"]}
    res["roofline"] = {"kernel": "gqa_decode_tc_kernel", "bound": "hbm", "achieved": res["unsplit"]["achieved_gbs"],
                       "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": res["unsplit"]["frac"],
                       "peak_source": pk["source"]}
    return res


def bench_gdn_prefill_cfg3(ops, dev, stream, reps=5):
    """cfg3: chunked prefill of B=8 sequences x T=2048 tokens, 16 heads, dk=dv=128, zero initial state, bf16 out and
    fp32 final state. Inputs (201 MB of q/k/v) exceed L2, so no flush is needed between replays."""
    B, T, H, d = 8, 2048, 16, 128
    gen = torch.Generator().manual_seed(3)
    N = B * T
    q = F.normalize(torch.randn(N, H, d, generator=gen), dim=-1).bfloat16().to(dev)
    k = F.normalize(torch.randn(N, H, d, generator=gen), dim=-1).bfloat16().to(dev)
    v = torch.randn(N, H, d, generator=gen).bfloat16().to(dev)
    beta = torch.sigmoid(torch.randn(N, H, generator=gen)).to(dev)
    g = (-F.softplus(torch.randn(N, H, generator=gen))).to(dev)
    cu = torch.arange(0, N + 1, T, dtype=torch.int32, device=dev)
    out = torch.empty(N, H, d, device=dev, dtype=torch.bfloat16)
    final = torch.empty(B, H, d, d, device=dev, dtype=torch.float32)
    ws = torch.empty(ops.gdn_chunk_prefill_workspace_bytes(N, B, H, d), device=dev, dtype=torch.uint8)
    ms = graph_ms(lambda: ops.gdn_chunk_prefill(q, k, v, g, beta, cu, final_state=final, out=out, workspace=ws),
                  stream, reps)
    nbytes = N * H * (3 * d * 2 + 2 * 4 + d * 2) + B * H * d * d * 4
    chunk_heads = B * H * (T // 64)
    flops = chunk_heads * 2 * (64 * 64 * (3 * d + 2 * d) + 3 * 64 * d * d + 64 ** 3 // 3)
    pk = peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    return {
        "workload": "cfg3 GDN chunked prefill: B=8 x T=2048, 16 heads, dk=dv=128, chunk 64, zero initial state",
        "ms": ms, "tokens_per_s": N / (ms / 1e3),
        "roofline": {"kernel": "gdn_prefill_prep_kernel + gdn_prefill_state_kernel", "bound": "hbm", "achieved": gbs,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"], "algorithmic_bytes": nbytes,
                     "peak_source": pk["source"]},
        "tensor": {"algorithmic_flops": flops, "tflops": flops / (ms / 1e3) / 1e12,
                   "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / pk["bf16_tflops"]},
    }




# --------------------------------------------------------------------------------------------- summaries


def profiled_traffic(summary: str):
    """DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) recorded from an ncu capture in the committed
    summary under profiles/ (the line ``traffic_bytes_per_launch: N`` or ``traffic_bytes_per_step: N``), or None."""
    path = ROOT / "profiles" / summary
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith(("traffic_bytes_per_launch:", "traffic_bytes_per_step:")):
            return int(line.split(":", 1)[1])
    return None


def operator_lines(pkg, dev) -> dict:
    """Every other hot-path operator on its own config (N=1): cfg2 DeltaNet decode, cfg4 MoE layer, the cfg5 AttnRes
    schedule, cfg3 chunked prefill, cfg5 GQA decode attention, the cfg5 sampler and one cfg5 DeltaNet + MoE layer."""
    ops = pkg.ops
    stream = torch.cuda.Stream(dev)
    return {
        "gdn_decode_cfg2": bench_gdn_decode_cfg2(ops, dev, stream),
        "moe_cfg4": bench_moe_cfg4(ops, dev, stream),
        "attnres_cfg5_decode": bench_attnres_decode(ops, dev, stream),
        "gdn_prefill_cfg3": bench_gdn_prefill_cfg3(ops, dev, stream),
        "gqa_decode_cfg5": bench_gqa_decode_cfg5(ops, dev, stream),
        "sampler_cfg5": bench_sampler_cfg5(ops, dev, stream),
        "decode_layer_cfg5": bench_decode_layer_cfg5(pkg, dev, stream),
        "vocoder_tail": bench_vocoder_tail(pkg, dev),
    }


def operator_summary(ops_: dict) -> dict:
    """The figure each operator is judged on, in a few keys."""
    out = {}
    for name, r in ops_.items():
        item = {}
        for key in ("ms", "ms_per_layer", "ms_per_step", "layer_ms", "us"):
            if key in r:
                item[key] = round(r[key], 4)
        roof = r.get("roofline")
        if roof:
            item["achieved"] = round(roof["achieved"], 1)
            item["unit"] = roof["unit"]
            item["frac"] = round(roof["frac"], 3)
        if "tensor" in r:
            item["tensor_frac"] = round(r["tensor"]["frac_of_bf16_peak"], 3)
        if "largest_route" in r:
            item["largest_route_frac"] = round(r["largest_route"]["frac"], 3)
        if "cpu_baseline" in r:
            item["cpu_ms"] = round(r["cpu_baseline"]["ms_per_layer"], 1)
        for key in ("bulk", "stream4", "stream4_e2e"):
            if key in r:
                item[key] = {"ms": round(r[key]["ms"], 3), "realtime_x": round(r[key]["realtime_x"])}
        out[name] = item
    return out


def profile_launches(n: int, workload: str = "decode_step", layers: int = LAYERS5, streams: int = 0) -> None:
    """n runs of a workload's kernels (the bench's own launches, without timing): cfg5 decode steps (graph replays of
    the headline step; ``layers`` shrinks the model for a small ncu case), cfg2 decode updates cycling the layer
    states, cfg4 MoE layers, the largest cfg5 AttnRes route, cfg3 prefill, cfg5 DeltaNet + MoE decode layers, cfg5
    GQA decode attention, cfg5 sampler calls (eager launches) or the vocoder DSP tail's two bench cases."""
    pkg = __import__("__graft_entry__").load_package()
    ops = pkg.ops
    dev = torch.device("cuda", 0)
    if workload == "decode_step":
        model, graph = build_cfg5(pkg, dev, layers=layers)
        for _ in range(n):
            graph.replay()
        torch.cuda.synchronize(dev)
        print(f"profile: {n} cfg5 decode steps ({layers} layers, {graph.launches_per_step} library launches each) "
              f"done, status {ops.device_status()}")
        return
    if workload == "vocoder_tail":
        voc = pkg.vocoder
        S = streams or 256
        ys, windows, mixer, (kernel, orig, new, width) = vocoder_inputs(S, 240)
        y0, y1 = (torch.from_numpy(y).to(dev) for y in ys)
        for _ in range(n):
            for step in (240, 4):  # one push of the whole second, then 4-frame pushes
                head = voc.IstftHeadStream((736, 2208), 184, windows, mixer, math.log(100.0), dev, streams=S,
                                           max_cols=step)
                res = voc.ResamplerStream(kernel, orig, new, width, dev, streams=S)
                for c0 in range(0, 240, step):
                    res.push(head.push(y0[:, c0:c0 + step], y1[:, c0:c0 + step]))
                res.push(head.flush())
                res.flush()
        torch.cuda.synchronize(dev)
        print(f"profile: {n} x (one 240-frame push + 60 four-frame pushes) of {S} vocoder streams done")
        return
    if workload == "moe":
        x, norm_w, w_r, gate_up, down = moe_cfg4_inputs(dev)
        T, D = x.shape
        E, two_i, _ = gate_up.shape
        ws = ops.MoEWorkspace(T, 8, E, D, two_i // 2, dev)
        out = torch.empty(T, D, device=dev, dtype=torch.bfloat16)
        for _ in range(n):
            ids, w = ops.moe_router(x, norm_w, 1e-5, w_r, None, 8, weights="full_softmax", renormalize=True,
                                    ids=ws.ids, topk_weights=ws.weights)
            ops.moe_experts(x, gate_up, down, ids, w, ws, out=out)
        torch.cuda.synchronize(dev)
        print(f"profile: {n} cfg4 MoE layers done, status {ops.device_status()}")
        return
    if workload == "decode_layer":
        layer, core, batch = decode_layer_cfg5(__import__("__graft_entry__").load_package(), dev)
        with core.forward_batch(batch):
            for _ in range(n):
                layer()
        torch.cuda.synchronize(dev)
        print(f"profile: {n} cfg5 DeltaNet + MoE decode layers done")
        return
    if workload == "prefill":
        B, T, H, d = 8, 2048, 16, 128
        N = B * T
        gen = torch.Generator().manual_seed(3)
        q = F.normalize(torch.randn(N, H, d, generator=gen), dim=-1).bfloat16().to(dev)
        k = F.normalize(torch.randn(N, H, d, generator=gen), dim=-1).bfloat16().to(dev)
        v = torch.randn(N, H, d, generator=gen).bfloat16().to(dev)
        beta = torch.sigmoid(torch.randn(N, H, generator=gen)).to(dev)
        g = (-F.softplus(torch.randn(N, H, generator=gen))).to(dev)
        cu = torch.arange(0, N + 1, T, dtype=torch.int32, device=dev)
        for _ in range(n):
            ops.gdn_chunk_prefill(q, k, v, g, beta, cu)
        torch.cuda.synchronize(dev)
        print(f"profile: {n} cfg3 chunked prefills done")
        return
    if workload == "sampler":
        gen = torch.Generator().manual_seed(8)
        logits = (3 * torch.randn(256, 10, 4098, generator=gen)).to(dev)
        rep = torch.randint(0, 4098, (256, 10, 32), generator=gen, dtype=torch.int32).to(dev)
        for i in range(n):
            ops.sample_tts(logits, [0.8] * 256, [50], [0.9], [0.0], codebook_size=4096, audio_pad_id=4097,
                           stop_token_ids=[4096] * 256, repetition_token_ids=rep,
                           repetition_penalties=torch.full((256,), 1.2), seed=1, offset=i)
        torch.cuda.synchronize(dev)
        print(f"profile: {n} cfg5 sampler calls done")
        return
    if workload == "gqa_decode":
        q, kc, vc, table, seq = gqa_cfg5_inputs(dev)
        out = torch.empty_like(q)
        for _ in range(n):
            ops.gqa_decode(q, kc, vc, table, seq, out=out)
        torch.cuda.synchronize(dev)
        print(f"profile: {n} cfg5 GQA decode attention calls done")
        return
    if workload == "attnres":
        gen = torch.Generator().manual_seed(7)
        bank = torch.randn(49, 256, 2048, generator=gen).bfloat16().to(dev)
        queries = (0.02 * torch.randn(49, 2048, generator=gen)).bfloat16().to(dev)
        norm_w = torch.ones(2048, dtype=torch.bfloat16, device=dev)
        table = torch.zeros(49, 256, 52, device=dev, dtype=torch.float32)
        inv_rms = torch.zeros(256, 52, device=dev, dtype=torch.float32)
        for r in range(48):  # the earlier routes of the forward fill the logit table
            ops.attnres_route_tabled(bank, r, bank[r], queries, r, table, inv_rms, 1e-5, source_in_bank=True,
                                     norm_weight=norm_w)
        flush = L2Flush(dev)
        for i in range(n):  # alternately the last route with a look-ahead (47) and the largest route (48)
            r = 47 + i % 2
            flush_l2(flush)
            ops.attnres_route_tabled(bank, r, bank[r], queries, r, table, inv_rms, 1e-5, source_in_bank=r < 48,
                                     norm_weight=norm_w)
        torch.cuda.synchronize(dev)
        print(f"profile: {n} AttnRes routes (49 sources x 256 tokens x 2048) done")
        return
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
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--e2e-steps", type=int, default=10, help="timed steps of the end-to-end loop")
    ap.add_argument("--cpu-samples", type=int, default=3, help="stream-steps in the CPU-baseline sample")
    ap.add_argument("--profile-launches", type=int, default=0,
                    help="only run this many steps / launches of a workload (for an ncu capture) and exit")
    ap.add_argument("--profile-workload", default="decode_step",
                    choices=("decode_step", "gdn_decode", "moe", "attnres", "prefill", "decode_layer", "gqa_decode",
                             "sampler", "vocoder_tail"),
                    help="workload whose launches --profile-launches runs")
    ap.add_argument("--profile-layers", type=int, default=LAYERS5, help="layers of the decode_step profile model")
    ap.add_argument("--profile-streams", type=int, default=0, help="streams of the vocoder_tail profile (0: 256)")
    ap.add_argument("--operators", type=int, default=1,
                    help="also time the other hot-path operators on their own configs at N=1")
    args = ap.parse_args()
    if args.profile_launches:
        profile_launches(args.profile_launches, args.profile_workload, args.profile_layers, args.profile_streams)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = dist_env()

    if args.impl == "reference":
        if rank != 0:
            return
        samples = args.steps + args.warmup
        value, threads, dt, per_step = cpu_reference_cfg5(samples)
        sample = (f"{samples} stream-steps of a 4-layer slice (3 DeltaNet + 1 GQA) and of the 0-layer remainder of "
                  f"the cfg5 model at {CONTEXT5} cached keys, one stream per call, scaled to 24 layers "
                  f"({per_step * 1e3:.0f} ms per stream-step; {dt:.1f} s of timed forwards)")
        line = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * STREAMS5 * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random-init weights N(0, 0.02); random cache)", "config": cfg5_config(world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return

    dist = init_dist(world, local)
    try:
        line = run_ours(args, dist, rank, world, local)
        if rank == 0:
            value, threads, dt, per_step = cpu_reference_cfg5(args.cpu_samples)
            line["cpu_baseline"] = {
                "value": value, "unit": UNIT, "cores": threads, "kind": "port",
                "sample": f"{args.cpu_samples} stream-steps of oracle/lm.py (fp32; 4-layer slice + remainder, "
                          f"scaled to 24 layers): {per_step * 1e3:.0f} ms each",
            }
            if args.operators and world == 1:
                pkg = __import__("__graft_entry__").load_package()
                full = operator_lines(pkg, torch.device("cuda", local))
                print("operators (full): " + json.dumps(full), file=sys.stderr, flush=True)
                line["operators"] = operator_summary(full)
                for name, item in line["operators"].items():
                    print(f"operator {name}: {json.dumps(item)}", flush=True)
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
