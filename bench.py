#!/usr/bin/env python
"""Benchmark of the sm_100a Chronos MoE feed-forward layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|prefill|ep]

Prints ONE JSON line (rank 0).  Workloads (synthetic data, seeded; weights
N(0, 0.02), hidden states N(0, 1)):

* ``decode`` (default): the DeepSeek-MoE-16B-shaped layer (d_model 2048, 64
  routed experts top-6 + 2 shared, d_ff 1408, bf16) with availability mask
  Bernoulli(0.9) (unavailable experts are placeholders served by the shared
  fallback).  One step = one layer call at each decode batch 1, 8, 32 and 64
  tokens (105 tokens).  ``value`` = tokens/s of the layer with inputs resident
  in HBM (each call a CUDA-graph replay, L2 flushed before every call).
* ``prefill``: the same layer on 8192 tokens, router logits offset by a
  Zipf(s=1.1) per-expert bias, all experts available.  One step = one call.

* ``e2e_decode`` (sub-object): the MoE FFNs of an 8-layer decode (d_model 1024,
  16 experts top-2 + 1 shared, d_ff 2048, batch 32, 512-token prompt, 256
  steps, availability Bernoulli(0.85) per step and layer, ready flags on).
* ``ep``: the DeepSeek-V3-shaped layer (d_model 7168, 256 routed experts
  top-8 + 1 shared, d_ff 2048, bf16), 4096 tokens per GPU, routed experts
  sharded evenly over the GPUs with NCCL all-to-all dispatch/combine (one
  GPU: all experts local, no exchange).  One step = one layer call per rank.

All workloads are measured in every run; ``--workload`` picks the one the
headline ``value`` reports, the others appear as sub-objects.  ``e2e``
drives the public module (``ChronosMOEFeedForward``) with pinned host inputs:
H2D copy, layer, D2H copy inside the timed region.  ``roofline`` is the
dominant kernel of the headline workload, timed per launch with CUDA events
around that kernel (stage events inside the extension).  ``cpu_baseline``
(rank 0, N=1) is the CPU oracle port of the layer on a bounded sample.

``--impl reference`` times the CPU implementation of the path (the oracle
port: router restated in C, experts in numpy/BLAS with every host thread) on
the same workload and prints the same metric with "impl": "reference".

Multi-GPU (torchrun, one process per GPU): decode and prefill run an
independent replica per rank (those layers do not shard); ``ep`` shards the
experts over the ranks.  ``value`` = tokens of all ranks / max-over-ranks
device time.
"""
from __future__ import annotations

import argparse
import datetime
import gc
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

DECODE_BATCHES = (1, 8, 32, 64)
PREFILL_TOKENS = 8192
FLUSH_BYTES = 256 << 20  # > 126 MB L2
METRIC_DECODE = "MoE-layer tokens/s (decode, batches 1/8/32/64)"
METRIC_PREFILL = "MoE-layer tokens/s (prefill, 8192 tokens)"


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return dict(hbm_gbs=float(d["hbm_gbs"]), bf16_tflops=float(d["bf16_tflops"]),
                    bf16_tflops_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                    source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0,
                source="fallback")


def committed_traffic():
    p = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        busy = [r for r in rows if (num(r[4]) or 0.0) >= 50.0] or rows
        sm = [num(r[1]) for r in busy if num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in busy for i in range(4) if r[6 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": num(rows[0][2]), "reasons": reasons, "samples": len(rows),
                "busy_samples": len(busy)}


class Dist:
    def __init__(self):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False

    def init(self):
        if self.world > 1:
            import torch.distributed as dist
            torch.cuda.set_device(self.local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local_rank))
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            import torch.distributed as dist
            dist.destroy_process_group()


def decode_config(shape):
    return dict(hidden_size=shape.hidden, num_experts=shape.num_experts,
                num_experts_per_tok=shape.top_k, moe_intermediate_size=shape.ffn,
                num_shared_experts=shape.num_shared, norm_topk_prob=shape.norm_topk,
                router_aux_loss_coef=5e-4, hidden_act="silu", dropout=0.0,
                fallback_mask_prob=0.0, intermediate_size=shape.ffn)


def algorithmic_bytes(stage: str, shape, n_tokens: int, experts_applied: int, slots: int,
                      elem: int = 2) -> float:
    """HBM bytes one launch of a stage must move at minimum, the numerator of the
    decode roofline (each weight byte read once per call):
    gate/up: gate+up weights of every expert applied (routed + shared), the
    token rows read and the hidden rows written; down: down weights of every
    expert applied, hidden rows read, fp32 output accumulator written."""
    H, F = shape.hidden, shape.ffn
    if stage == "gateup":
        return experts_applied * 2 * F * H * elem + slots * H * elem + slots * F * elem
    if stage == "down":
        return experts_applied * F * H * elem + slots * F * elem + n_tokens * H * 4
    raise ValueError(stage)


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------

def run_ours(args, dist: Dist):
    from project_chronos_b200 import LazyExpertPlaceholder, ops, synthetic as syn
    from project_chronos_b200.moe import ChronosMOEFeedForward
    import types

    dev = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(dev)
    peaks = measured_peaks()
    sampler = ClockSampler(dist.local_rank)
    sampler.start()

    spec = syn.WORKLOADS["decode"]
    shape = spec["shape"]
    wl = syn.make_workload(shape, max(DECODE_BATCHES), seed=1234 + dist.rank,
                           dtype=torch.bfloat16, device=dev, avail_p=spec["avail_p"])
    w = wl.weights
    mask_host = wl.mask.cpu()
    cfg = types.SimpleNamespace(**decode_config(shape))
    module = ChronosMOEFeedForward.from_stacked(cfg, w.router, w.gate, w.up, w.down, w.sh_gate,
                                                w.sh_up, w.sh_down).eval()
    for e in range(shape.num_experts):
        if not bool(mask_host[e]):
            module.experts[e] = LazyExpertPlaceholder(shape.hidden, shape.ffn, torch.bfloat16)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    xs = {b: wl.x[:b].contiguous().view(1, b, shape.hidden) for b in DECODE_BATCHES}

    # ---------------- decode: warm-up, graphs, timed region ----------------
    with torch.no_grad():
        for _ in range(max(1, args.warmup)):
            for b in DECODE_BATCHES:
                module(xs[b], mask_host)
        torch.cuda.synchronize()
        graphs, gouts, launches_per_graph = {}, {}, {}
        for b in DECODE_BATCHES:
            g = torch.cuda.CUDAGraph()
            before = ops.kernel_launches()
            with torch.cuda.graph(g):
                gouts[b] = module(xs[b], mask_host)
            launches_per_graph[b] = ops.kernel_launches() - before
            graphs[b] = g
        for _ in range(2):
            for b in DECODE_BATCHES:
                graphs[b].replay()
        torch.cuda.synchronize()
        # graph output equals the eager output
        for b in DECODE_BATCHES:
            ref = module(xs[b], mask_host)
            graphs[b].replay()
            torch.cuda.synchronize()
            if not torch.allclose(ref.float(), gouts[b].float(), rtol=1e-2, atol=1e-2):
                raise RuntimeError("graph replay disagrees with the eager layer call")

        K = args.steps
        ev = {b: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(K)] for b in DECODE_BATCHES}
        dist.barrier()
        torch.cuda.synchronize()
        for i in range(K):
            for b in DECODE_BATCHES:
                flush.zero_()
                ev[b][i][0].record()
                graphs[b].replay()
                ev[b][i][1].record()
        torch.cuda.synchronize()
        dist.barrier()
        dec_ms = {b: sum(s.elapsed_time(e) for s, e in ev[b]) for b in DECODE_BATCHES}
        dec_total_ms = dist.max(sum(dec_ms.values()))
        dec_launches = K * sum(launches_per_graph.values())

        # per-stage kernel times (queue backed up behind a sleep so events
        # bracket kernels, not host launch gaps)
        ops.profile_begin(K * len(DECODE_BATCHES))
        dec_apps = {}
        for i in range(K):
            for b in DECODE_BATCHES:
                flush.zero_()
                torch.cuda._sleep(1_000_000)
                module(xs[b], mask_host)
        prof_dec = ops.profile_end()
        for b in DECODE_BATCHES:
            r = ops.moe_route(xs[b].view(b, -1), w.router, shape.top_k, shape.norm_topk)
            sel = set(r["topk_idx"].cpu().numpy().ravel().tolist())
            avail_sel = [e for e in sel if bool(mask_host[e])]
            slots_routed = int(sum(int((r["topk_idx"] == e).sum()) for e in avail_sel))
            dec_apps[b] = dict(experts=len(avail_sel) + shape.num_shared,
                               slots=slots_routed + b * shape.num_shared)
        ops.check_status(dev)

        # ---------------- prefill ----------------
        pwl_g = syn.make_generator(99 + dist.rank, dev)
        xp = syn.make_hidden(PREFILL_TOKENS, shape.hidden, pwl_g, dtype=torch.bfloat16, device=dev)
        bias = syn.make_zipf_bias(shape.num_experts, 1.1, pwl_g, dev)

        def prefill_call():
            return ops.moe_forward(xp, w.router, w.gate, w.up, w.down, w.sh_gate, w.sh_up,
                                   w.sh_down, shape.top_k, shape.norm_topk, router_bias=bias,
                                   want_probs=True)

        for _ in range(max(1, args.warmup)):
            prefill_call()
        torch.cuda.synchronize()
        KP = max(3, min(args.steps, 20))
        pev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(KP)]
        launches0 = ops.kernel_launches()
        dist.barrier()
        torch.cuda.synchronize()
        for i in range(KP):
            flush.zero_()
            pev[i][0].record()
            prefill_call()
            pev[i][1].record()
        torch.cuda.synchronize()
        dist.barrier()
        pre_launches = ops.kernel_launches() - launches0
        pre_ms = dist.max(sum(s.elapsed_time(e) for s, e in pev)) / KP
        ops.profile_begin(KP)
        for i in range(KP):
            flush.zero_()
            torch.cuda._sleep(1_000_000)
            out = prefill_call()
        prof_pre = ops.profile_end()
        ops.check_status(dev)
        pre_slots_routed = PREFILL_TOKENS * shape.top_k
        pre_flops = syn.layer_flops(shape, PREFILL_TOKENS)
        counts = torch.bincount(out["topk_idx"].reshape(-1).long(), minlength=shape.num_experts)
        imbalance = float(counts.max()) / float(counts.float().mean())

        # ---------------- e2e through the public module ----------------
        x_host = {b: xs[b].cpu().pin_memory() for b in DECODE_BATCHES}
        y_host = {b: torch.empty_like(x_host[b]).pin_memory() for b in DECODE_BATCHES}
        x_dev = {b: torch.empty_like(xs[b]) for b in DECODE_BATCHES}
        compute = torch.cuda.current_stream(dev)
        h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        ev_in = {b: torch.cuda.Event() for b in DECODE_BATCHES}
        ev_out = {b: torch.cuda.Event() for b in DECODE_BATCHES}

        def e2e_step():
            # a serving loop's copies on their own streams: the step's inputs go up
            # while the first call runs, each result comes back while the next runs
            h2d_s.wait_stream(compute)
            with torch.cuda.stream(h2d_s):
                for b in DECODE_BATCHES:
                    x_dev[b].copy_(x_host[b], non_blocking=True)
                    ev_in[b].record(h2d_s)
            for b in DECODE_BATCHES:
                compute.wait_event(ev_in[b])
                y = module(x_dev[b], mask_host)
                ev_out[b].record(compute)
                d2h_s.wait_event(ev_out[b])
                with torch.cuda.stream(d2h_s):
                    y.record_stream(d2h_s)
                    y_host[b].copy_(y, non_blocking=True)
            compute.wait_stream(d2h_s)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        # more steps than the device-timed loop: one host pause (another process
        # on the host, the OS) then moves the mean by a fraction, and the
        # per-step distribution shows whether the mean is such a pause
        KE = max(K, E2E_MIN_STEPS)
        eev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(KE)]
        dist.barrier()
        torch.cuda.synchronize()
        # the timed steps include host-side Python: a full collection before them
        # and none inside them (as timeit does)
        gc.collect()
        gc.disable()
        try:
            for i in range(KE):
                # a serving loop consumes each result: the host waits for step i - 2's
                # copies before issuing step i (one step of slack keeps the GPU fed,
                # and the host never runs hundreds of launches ahead)
                if i >= 2:
                    eev[i - 2][1].synchronize()
                flush.zero_()
                eev[i][0].record()
                e2e_step()
                eev[i][1].record()
        finally:
            gc.enable()
        torch.cuda.synchronize()
        if not torch.allclose(y_host[DECODE_BATCHES[-1]].float(), gouts[DECODE_BATCHES[-1]].float().cpu(),
                              rtol=1e-2, atol=1e-2):
            raise RuntimeError("end-to-end output disagrees with the graph-replayed layer")
        dist.barrier()
        e2e_steps_ms = np.array([s.elapsed_time(e) for s, e in eev])
        e2e_ms = dist.max(float(e2e_steps_ms.sum())) / KE
        h2d = sum(x_host[b].numel() * x_host[b].element_size() for b in DECODE_BATCHES)
        d2h = sum(y_host[b].numel() * y_host[b].element_size() for b in DECODE_BATCHES)

        # ---------------- expert parallel (DeepSeek-V3 shape) ----------------
        ep = run_ep(args, dist, dev, peaks, flush)
        # ---------------- 8-layer decode, MoE FFNs (e2e workload) ----------------
        e2e_dec = run_model_decode(args, dist, dev, peaks)
        e2e_dec["moe_layers_alone"] = run_moe_layers_decode(args, dist, dev, peaks)

    clocks = sampler.stop()

    # ---------------- assemble ----------------
    tokens_step = sum(DECODE_BATCHES)
    dec_ms_step = dec_total_ms / K
    dec_value = tokens_step * dist.world / (dec_ms_step / 1e3)
    per_batch = {}
    for b in DECODE_BATCHES:
        t_ms = dec_ms[b] / K
        lb = syn.decode_bytes(shape, b, dec_apps[b]["experts"] - shape.num_shared)
        per_batch[str(b)] = dict(us_per_call=round(t_ms * 1e3, 2),
                                 us_per_token=round(t_ms * 1e3 / b, 3),
                                 layer_bytes=int(lb),
                                 layer_gbs=round(lb / (t_ms / 1e3) / 1e9, 1),
                                 layer_hbm_frac=round(lb / (t_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                                 experts_read=dec_apps[b]["experts"])
    # dominant decode kernel and its roofline
    stage_ms = {s: prof_dec[s][0] for s in ("gateup", "down")}
    dom = max(stage_ms, key=stage_ms.get)
    dom_bytes = sum(algorithmic_bytes(dom, shape, b, dec_apps[b]["experts"], dec_apps[b]["slots"])
                    for b in DECODE_BATCHES) * K
    dom_launches = prof_dec[dom][1]
    dom_avg_ms = prof_dec[dom][0] / max(1, dom_launches)
    dec_achieved = dom_bytes / (prof_dec[dom][0] / 1e3) / 1e9
    traffic = committed_traffic()
    dec_roof = dict(kernel=f"tc_grouped_gemm ({dom}) decode", bound="hbm",
                    achieved=round(dec_achieved, 1), peak=peaks["hbm_gbs"], unit="GB/s",
                    frac=round(dec_achieved / peaks["hbm_gbs"], 4),
                    traffic=traffic.get(f"decode_{dom}_bytes_per_launch"),
                    algorithmic_bytes_per_launch=round(dom_bytes / max(1, dom_launches)),
                    avg_launch_us=round(dom_avg_ms * 1e3, 2), launches=dom_launches,
                    peak_source=peaks["source"])
    # prefill
    pre_gateup_ms = prof_pre["gateup"][0] / max(1, prof_pre["gateup"][1])
    pre_gateup_flops = 2.0 * 2 * shape.ffn * shape.hidden * (pre_slots_routed
                                                              + PREFILL_TOKENS * shape.num_shared)
    pre_gu_tflops = pre_gateup_flops / (pre_gateup_ms / 1e3) / 1e12
    pre_roof = dict(kernel="tc_gateup_tm (gate/up, token-major) prefill", bound="tensor",
                    achieved=round(pre_gu_tflops, 1), peak=peaks["bf16_tflops"], unit="TFLOP/s",
                    frac=round(pre_gu_tflops / peaks["bf16_tflops"], 4),
                    traffic=traffic.get("prefill_gateup_bytes_per_launch"),
                    algorithmic_flops_per_launch=pre_gateup_flops,
                    avg_launch_us=round(pre_gateup_ms * 1e3, 1), launches=prof_pre["gateup"][1],
                    peak_source=peaks["source"])
    pre_layer_tflops = pre_flops / (pre_ms / 1e3) / 1e12
    prefill = dict(metric=METRIC_PREFILL, value=round(PREFILL_TOKENS * dist.world / (pre_ms / 1e3), 1),
                   unit="tokens/s", ms_per_step=round(pre_ms, 4), steps=KP,
                   layer_tflops=round(pre_layer_tflops, 1),
                   layer_tc_frac=round(pre_layer_tflops / peaks["bf16_tflops"], 4),
                   flops_per_call=pre_flops, expert_load_max_over_mean=round(imbalance, 2),
                   gpu_launches=pre_launches, roofline=pre_roof,
                   stages_ms_per_call={s: round(prof_pre[s][0] / KP, 4) for s in prof_pre
                                       if s != "calls"})
    decode = dict(metric=METRIC_DECODE, value=round(dec_value, 1), unit="tokens/s",
                  ms_per_step=round(dec_ms_step, 4), per_batch=per_batch, roofline=dec_roof,
                  gpu_launches=dec_launches,
                  stages_ms_per_step={s: round(prof_dec[s][0] / K, 4) for s in prof_dec
                                      if s != "calls"})
    e2e = dict(value=round(tokens_step * dist.world / (e2e_ms / 1e3), 1), unit="tokens/s",
               h2d_bytes_per_step=int(h2d), d2h_bytes_per_step=int(d2h),
               ms_per_step=round(e2e_ms, 4), steps=int(KE),
               median_ms=round(float(np.median(e2e_steps_ms)), 4),
               p90_ms=round(float(np.percentile(e2e_steps_ms, 90)), 4),
               max_ms=round(float(e2e_steps_ms.max()), 4),
               # where the slow steps were: index of the slowest, and the steps over 5x the median
               max_step=int(e2e_steps_ms.argmax()),
               steps_over_5x_median=[int(i) for i in np.nonzero(e2e_steps_ms > 5 * np.median(e2e_steps_ms))[0][:8]],
               mean_without_those_ms=round(float(e2e_steps_ms[e2e_steps_ms <= 5 * np.median(e2e_steps_ms)].mean()), 4),
               over_device_step=round(e2e_ms / dec_ms_step, 3),
               path=("ChronosMOEFeedForward.forward (eager), pinned host x -> device -> host y, "
                     "copies on their own streams"))

    head = {"decode": decode, "prefill": prefill, "ep": ep}[args.workload]
    line = {
        "metric": head["metric"], "value": head["value"], "unit": head["unit"],
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, N(0,0.02) weights)",
        "config": bench_config(args, dist.world),
        "roofline": {"decode": dec_roof, "prefill": pre_roof, "ep": ep["roofline"]}[args.workload],
        "e2e": e2e,
        "clocks": clocks,
        "gpu_launches": head["gpu_launches"],
        "decode": decode if args.workload != "decode" else {k: v for k, v in decode.items()
                                                            if k not in ("metric", "value", "unit")},
        "prefill": prefill if args.workload != "prefill" else {k: v for k, v in prefill.items()
                                                               if k not in ("metric", "value", "unit")},
        "ep": ep if args.workload != "ep" else {k: v for k, v in ep.items()
                                                 if k not in ("metric", "value", "unit")},
        "e2e_decode": e2e_dec,
    }
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"], line["parity"] = cpu_baseline(
            w, wl.x, mask_host, shape, args.workload, xp_dev=xp, bias=bias,
            gpu_out={b: gouts[b].view(b, -1) for b in DECODE_BATCHES})
    return line


WORKLOAD_DESC = {
    "decode": ("decode: MoE layer d_model 2048, 64 experts top-6 + 2 shared, d_ff 1408 "
               "(DeepSeek-MoE-16B shape), batches 1/8/32/64, availability Bernoulli(0.9)"),
    "prefill": "prefill: same layer, 8192 tokens, Zipf(1.1) router bias, all available",
    "ep": ("expert parallel: MoE layer d_model 7168, 256 experts top-8 + 1 shared, d_ff 2048 "
           "(DeepSeek-V3 shape), 4096 tokens per GPU, experts sharded evenly over the GPUs, "
           "NCCL all-to-all dispatch/combine"),
}


def bench_config(args, world: int) -> dict:
    """The ``config`` of both arms' JSON lines (same workload, same keys)."""
    return {
        "workload": WORKLOAD_DESC[args.workload],
        "l2": "flushed before every timed call (256 MB write)",
        "graphs": "decode calls replayed as CUDA graphs" if args.workload == "decode" else "eager",
        "parallelism": (f"ep{world} (experts sharded)" if args.workload == "ep"
                        else f"replicas x{world} (decode/prefill), ep{world} (ep)"),
    }


E2E_MIN_STEPS = 2000  # ~1.2 s: one ~100 ms host pause (seen once in 500 steps) moves the mean by ~8 %
E2E_BATCH = 32
E2E_LAYERS = 8
E2E_PROMPT = 512
E2E_STEPS = 256




def _model_step_bytes(cfg, B: int, ctx: int, experts_read: float) -> float:
    """Algorithmic HBM bytes of one decode step of the model (bf16): every weight
    the step reads once (attention projections, the router, the shared expert and
    the experts read (selected and available, summed over layers), the lookahead
    router, the tied LM head), the caches read (MLA latent and rope keys of
    ``ctx`` positions, sliding-window keys and values of min(ctx, window) slots)."""
    H, nh, nkv, D = cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    L, R, W, E, F = cfg["kv_latent_dim"], cfg["rope_dim"], cfg["sliding_window_size"], cfg["num_experts"], \
        cfg["moe_intermediate_size"]
    nope = D - R
    mla_w = H * (nh * (nope + R) + L) + L * nkv * (nope + R + D) + nh * D * H
    sw_w = H * (nh + 2 * nkv) * D + nh * D * H
    n_layers = cfg["num_hidden_layers"]
    n_mla = (n_layers + 1) // 2
    attn_w = n_mla * mla_w + (n_layers - n_mla) * sw_w
    moe_w = n_layers * (E * H + cfg["num_shared_experts"] * 3 * H * F) + experts_read * 3 * H * F
    look_w = H * (H // 4) + (H // 4) * E * (cfg["lookahead_steps"] + 1)
    head_w = cfg["vocab_size"] * H
    caches = B * (n_mla * ctx * (L + nkv * R) + (n_layers - n_mla) * min(ctx, W) * nkv * D * 2)
    return 2.0 * (attn_w + moe_w + look_w + head_w + caches)


def run_model_decode(args, dist: Dist, dev, peaks) -> dict:
    """The 8-layer Chronos model decode: d_model 1024, 8 heads (2 kv heads),
    MLA on even and sliding-window attention on odd layers, MoE blocks of 16
    experts top-2 + 1 shared with d_ff 2048, the lookahead router and the tied
    LM head; bf16, random-init weights, batch 32, a 512-token random prompt
    then 256 greedy decode steps.  Each layer's expert availability is a fresh
    Bernoulli(0.85) draw per step (the experts drawn unavailable are treated as
    not resident: their selections go to the shared expert), device ready flags
    gate every selected expert.  Each step is one CUDA-graph replay of the whole
    model step (embedding, 8 blocks, lookahead router, LM head, greedy pick);
    the step's masks are copied into the graph's buffer before it."""
    import types
    from project_chronos_b200 import ops
    from project_chronos_b200.model import ChronosForCausalLM, GraphedDecoder

    from project_chronos_b200 import synthetic as syn
    cfg = types.SimpleNamespace(**syn.DECODE_MODEL)
    B, P, T = E2E_BATCH, E2E_PROMPT, E2E_STEPS
    lm = ChronosForCausalLM.on_device(cfg, dev, torch.bfloat16)
    syn.init_model_(lm, 8800 + dist.rank, dev)
    lm = lm.eval()
    g = torch.Generator(device=dev)
    g.manual_seed(8900 + dist.rank)
    L, E = cfg.num_hidden_layers, cfg.num_experts
    flags = torch.ones(E, dtype=torch.int32, device=dev)
    for blk in lm.model.layers:
        blk.mlp.mask_semantics = "residency"
        blk.mlp.expert_ready_flags = flags
        blk.mlp.expert_ready_epoch = 1
    ids = torch.randint(0, cfg.vocab_size, (B, P), generator=g, device=dev)
    masks = (torch.rand(T + 32, L, E, generator=g, device=dev) < 0.85).float()
    pa, pb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.no_grad():
        lm(ids, use_cache=True, cache_capacity=P + T + 40)          # warm-up prompt
        torch.cuda.synchronize()
        pa.record()
        out, _ = lm(ids, use_cache=True, cache_capacity=P + T + 40)
        pb.record()
        cache = out.past_key_values
        gd = GraphedDecoder(lm, cache)
        gd.ids.copy_(torch.argmax(out.logits[:, -1], dim=-1).view(-1, 1))
        launches0 = ops.kernel_launches()
        gd.masks.copy_(masks[0])
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for t in range(T):
            gd.masks.copy_(masks[t])
            gd.step()
        b.record()
        torch.cuda.synchronize()
        dist.barrier()
        del launches0
        # experts read per step, sampled on further (untimed) steps through the
        # statistics buffers the captured MoE calls write
        pend = [blk.mlp._stats_pending for blk in lm.model.layers]
        reads = []
        for t in range(T, T + 16):
            gd.masks.copy_(masks[t])
            gd.step()
            torch.cuda.synchronize()
            reads.append(sum(int(((pd["counts"] > 0) & (pd["a"] > 0)).sum()) for pd in pend
                             if pd is not None and isinstance(pd.get("a"), torch.Tensor)))
    ops.check_status(dev)
    ms = dist.max(a.elapsed_time(b)) / T
    prompt_ms = pa.elapsed_time(pb)
    experts_read = float(np.mean(reads)) if reads else float("nan")
    step_bytes = _model_step_bytes(syn.DECODE_MODEL, B, P + T // 2, experts_read)
    gbs = step_bytes / (ms / 1e3) / 1e9
    return dict(metric="Chronos model decode tokens/s (8 layers, hybrid attention + MoE, batch 32)",
                value=round(B * dist.world / (ms / 1e3), 1), unit="tokens/s",
                us_per_step=round(ms * 1e3, 2), steps=T, prompt_tokens=B * P,
                prompt_ms=round(prompt_ms, 3),
                prompt_tokens_per_s=round(B * P / (prompt_ms / 1e3), 1),
                experts_read_per_step=round(experts_read, 2),
                step_bytes_mid_sequence=int(step_bytes), step_gbs=round(gbs, 1),
                hbm_frac=round(gbs / peaks["hbm_gbs"], 4),
                cache_bytes=int(cache.nbytes()),
                gpu_launches_per_step=int(gd.launches_per_step),
                gpu_launches=int(gd.launches_per_step) * T,
                note=("ChronosForCausalLM: attention decode kernels (MLA latent cache, sliding-window ring), "
                      "MoE kernels, lookahead kernel, cuBLAS projections and LM head; greedy; "
                      "availability Bernoulli(0.85) per step and layer, ready flags on; one CUDA graph "
                      "replay per step"))


def run_moe_layers_decode(args, dist: Dist, dev, peaks) -> dict:
    """The MoE layers ALONE of the 8-layer decode (for the MoE share of the model
    step): d_model 1024, 16 experts top-2 + 1 shared, d_ff 2048, bf16, batch 32,
    a 512-token prompt then 256 steps; each layer's availability a fresh
    Bernoulli(0.85) draw per step, device ready flags on; each layer call gets
    fresh N(0, 1) hidden states; one CUDA-graph replay per step."""
    from project_chronos_b200 import ops, synthetic as syn

    spec = syn.WORKLOADS["e2e"]
    shape = spec["shape"]
    B = spec["tokens"]
    E, L = shape.num_experts, E2E_LAYERS
    layers = [syn.make_workload(shape, 1, seed=5000 + 17 * l, dtype=torch.bfloat16, device=dev).weights
              for l in range(L)]
    g = syn.make_generator(6000 + dist.rank, dev)
    prompt = syn.make_hidden(B * E2E_PROMPT, shape.hidden, g, dtype=torch.bfloat16, device=dev)
    inputs = syn.make_hidden(E2E_STEPS * L * B, shape.hidden, g, dtype=torch.bfloat16,
                             device=dev).view(E2E_STEPS, L, B, shape.hidden)
    masks = (torch.rand(E2E_STEPS, L, E, generator=g, device=dev) < spec["avail_p"]).float()
    flags = torch.ones(E, dtype=torch.int32, device=dev)
    cur = torch.ones(L, E, dtype=torch.float32, device=dev)
    ws = {}

    def layer(l, x, avail):
        w = layers[l]
        key = x.shape[0]
        if key not in ws:
            ws[key] = torch.empty(ops.workspace_bytes(key, shape.hidden, E, shape.top_k, shape.ffn,
                                                      shape.num_shared, torch.bfloat16),
                                  dtype=torch.uint8, device=dev)
        return ops.moe_forward(x, w.router, w.gate, w.up, w.down, w.sh_gate, w.sh_up, w.sh_down,
                               shape.top_k, shape.norm_topk, avail=avail, ready_flags=flags,
                               ready_epoch=1, want_probs=False, workspace=ws[key])["y"]

    # prompt: the 8 layers on B*512 tokens (all experts available)
    def prefill():
        for l in range(L):
            layer(l, prompt, None)

    for _ in range(2):
        prefill()
    torch.cuda.synchronize()
    pa, pb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pa.record()
    prefill()
    pb.record()
    torch.cuda.synchronize()
    prompt_ms = pa.elapsed_time(pb)

    # decode step graph
    xin = torch.empty(L, B, shape.hidden, dtype=torch.bfloat16, device=dev)

    def step():
        for l in range(L):
            layer(l, xin[l], cur[l])

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    before = ops.kernel_launches()
    with torch.cuda.graph(graph):
        step()
    launches_per_step = ops.kernel_launches() - before
    for t in range(3):
        cur.copy_(masks[t])
        xin.copy_(inputs[t])
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for t in range(E2E_STEPS):
        cur.copy_(masks[t])
        xin.copy_(inputs[t])
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    dist.barrier()
    ops.check_status(dev)
    ms = dist.max(a.elapsed_time(b)) / E2E_STEPS
    # algorithmic bytes per step: per layer the router weight, the shared expert and
    # every selected expert that is available, each read once (mean over 16 steps)
    ebytes = syn.expert_bytes(shape)
    tot = 0
    sample = range(0, E2E_STEPS, E2E_STEPS // 16)
    for t in sample:
        for l in range(L):
            r = ops.moe_route(inputs[t, l], layers[l].router, shape.top_k, shape.norm_topk,
                              want_probs=False)
            sel = set(r["topk_idx"].view(-1).tolist())
            avail_sel = [e for e in sel if masks[t, l, e] > 0]
            tot += ebytes * (len(avail_sel) + shape.num_shared) + E * shape.hidden * 2
    tot //= len(sample)
    hbm = tot / (ms / 1e3) / 1e9
    return dict(metric="MoE FFN time per decode step, 8 layers alone",
                us_per_step=round(ms * 1e3, 2), tokens_per_s_moe_only=round(B * dist.world / (ms / 1e3), 1),
                step_bytes=int(tot), step_gbs=round(hbm, 1), hbm_frac=round(hbm / peaks["hbm_gbs"], 4),
                prompt_ms=round(prompt_ms, 3), prompt_tokens=B * E2E_PROMPT, steps=E2E_STEPS,
                gpu_launches_per_step=launches_per_step,
                note=("MoE layers only, fresh inputs per layer call; masks Bernoulli(0.85) per step and "
                      "layer; device ready flags on; one CUDA graph replay per step"))


def run_ep(args, dist: Dist, dev, peaks, flush) -> dict:
    """Expert-parallel layer, DeepSeek-V3 shape, 4096 tokens per rank, experts
    sharded over the ranks (one rank: all 256 experts local, no exchange)."""
    import types
    from project_chronos_b200 import ops, synthetic as syn
    from project_chronos_b200.ep import ExpertParallelMoE

    spec = syn.WORKLOADS["ep"]
    shape = spec["shape"]
    n = spec["tokens"]
    w = syn.make_ep_weights(shape, dist.rank, dist.world, seed=4321, dtype=torch.bfloat16, device=dev)
    x = syn.make_hidden(n, shape.hidden, syn.make_generator(777 + dist.rank, dev), dtype=torch.bfloat16,
                        device=dev)
    cfg = types.SimpleNamespace(hidden_size=shape.hidden, num_experts=shape.num_experts,
                                num_experts_per_tok=shape.top_k, moe_intermediate_size=shape.ffn,
                                num_shared_experts=shape.num_shared, norm_topk_prob=shape.norm_topk)
    m = ExpertParallelMoE.from_stacked(cfg, w.router, w.gate, w.up, w.down, w.sh_gate, w.sh_up,
                                       w.sh_down, local=True)
    # fixed all-to-all segments (equal splits, no host read of the split sizes) where a
    # token reaches nearly every rank: expected segment fill 1 - (1 - 1/G)^k of at least
    # 88 % (top-8: 2 and 4 ranks; 8 ranks would fill 66 %)
    # (2 GPUs: 5.03-5.16 ms per step against 5.05-5.37 with the counts read on the host)
    if dist.world > 1 and (1.0 - 1.0 / dist.world) ** shape.top_k <= 0.12:
        m.segment_rows = n
    for _ in range(max(1, args.warmup)):
        m(x)
    torch.cuda.synchronize()
    K = max(3, min(args.steps, 10))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    launches0 = ops.kernel_launches()
    dist.barrier()
    torch.cuda.synchronize()
    for i in range(K):
        flush.zero_()
        evs[i][0].record()
        m(x)
        evs[i][1].record()
    torch.cuda.synchronize()
    dist.barrier()
    launches = ops.kernel_launches() - launches0
    ms = dist.max(sum(a.elapsed_time(b) for a, b in evs) / K)
    ops.check_status(dev)
    # phases of a few more (untimed) calls: the exchange waits vs the expert GEMMs
    phases = None
    if dist.world > 1:
        m.phase_events = []
        for _ in range(3):
            m(x)
        torch.cuda.synchronize()
        names = ["start", "dispatched", "counts_exchanged", "shared_done", "rows_arrived", "experts_done",
                 "rows_returned", "combined"]
        per = {f"{a}->{b}": float(np.median([pe[a].elapsed_time(pe[b]) for pe in m.phase_events]))
               for a, b in zip(names[:-1], names[1:])}
        m.phase_events = None
        phases = {k2: round(dist.max(v), 4) for k2, v in per.items()}
    H, F, E, k, S = shape.hidden, shape.ffn, shape.num_experts, shape.top_k, shape.num_shared
    flops = 2.0 * n * (H * E + 3 * H * F * (k + S))          # per rank
    tflops = flops / (ms / 1e3) / 1e12
    sc = m.read_send_counts() or [n * k]
    remote_rows = sum(c for g, c in enumerate(sc) if g != dist.rank)
    if m.segment_rows:   # every segment travels whole, padding rows included
        remote_rows = m.segment_rows * (dist.world - 1)
    a2a_bytes = remote_rows * H * 2
    # the floor that binds: the rank's expert weights read once (HBM) or its FLOPs
    # at the sustained tensor peak (a seconds-long step sequence)
    weight_bytes = 2.0 * (3 * H * F * (E // dist.world + S) + H * E)
    t_hbm = weight_bytes / (peaks["hbm_gbs"] * 1e9)
    t_tc = flops / (peaks["bf16_tflops_sustained"] * 1e12)
    if t_hbm >= t_tc:
        gbs = weight_bytes / (ms / 1e3) / 1e9
        roof = dict(kernel="expert-parallel layer (all kernels + all-to-all), per GPU", bound="hbm",
                    achieved=round(gbs, 1), peak=peaks["hbm_gbs"], unit="GB/s",
                    frac=round(gbs / peaks["hbm_gbs"], 4), traffic=None,
                    algorithmic_bytes_per_step=weight_bytes, peak_source=peaks["source"])
    else:
        roof = dict(kernel="expert-parallel layer (all kernels + all-to-all), per GPU", bound="tensor",
                    achieved=round(tflops, 1), peak=peaks["bf16_tflops_sustained"], unit="TFLOP/s",
                    frac=round(tflops / peaks["bf16_tflops_sustained"], 4), traffic=None,
                    algorithmic_flops_per_step=flops, peak_source=peaks["source"] + " (sustained)")
    roof["floors_ms"] = dict(weights_over_hbm=round(t_hbm * 1e3, 3), flops_over_tc=round(t_tc * 1e3, 3))
    return dict(metric="MoE-layer tokens/s (expert parallel, DeepSeek-V3 shape, 4096 tokens/GPU)",
                value=round(n * dist.world / (ms / 1e3), 1), unit="tokens/s", ms_per_step=round(ms, 4),
                steps=K, ranks=dist.world, experts_per_rank=E // dist.world,
                layer_tflops_per_gpu=round(tflops, 1),
                a2a_bytes_per_gpu_per_direction=int(a2a_bytes),
                a2a_gbs_if_serial=round(a2a_bytes / (ms / 1e3) / 1e9, 1),
                phases_ms=phases,
                # the return exchange overlaps nothing (one chunk): bytes / its time
                a2a_return_gbs=(None if not phases else round(
                    a2a_bytes / (phases["experts_done->rows_returned"] / 1e3 + 1e-12) / 1e9, 1)),
                send_counts_rank0=sc, gpu_launches=launches, roofline=roof,
                exchange=("fixed segments of %d rows" % m.segment_rows if m.segment_rows
                          else ("counts read on the host" if dist.world > 1 else "none")))


# ---------------------------------------------------------------------------
# CPU: the oracle port (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------

def _cpu_weights(w):
    f = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    return dict(router=f(w.router), gate=f(w.gate), up=f(w.up), down=f(w.down),
                sh_gate=f(w.sh_gate), sh_up=f(w.sh_up), sh_down=f(w.sh_down))


def _threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else 1
    except Exception:
        return os.cpu_count() or 1


def _oracle_call(cw, x, avail, shape, bias=None):
    from oracle import moe_oracle as O
    return O.moe_forward(x, cw["router"], cw["gate"], cw["up"], cw["down"], cw["sh_gate"],
                         cw["sh_up"], cw["sh_down"], shape.top_k, shape.norm_topk, avail=avail,
                         bias=bias)


def _published_literal_mismatches() -> dict:
    """Literal bf16 reference routing vs the routing contract, per golden case
    (counts and their classification as committed in tests/golden/cases.json)."""
    try:
        with open(os.path.join(REPO, "tests", "golden", "cases.json")) as f:
            cases = json.load(f)["cases"]
    except OSError:
        return {}
    return {c["name"]: {k: c["literal_bf16_routing"][k] for k in
                        ("tokens", "mismatched_tokens", "bf16_tie", "logit_rounding", "other")}
            for c in cases if "literal_bf16_routing" in c}


def _decode_parity(x, w, cw, avail, shape, oracle_out, gpu_out) -> dict:
    """The timed layer's decode outputs against the oracle on the same inputs:
    top-k indices (bit-exact contract) and rel-L2 of the output."""
    from oracle import moe_oracle as O
    from project_chronos_b200 import ops
    res = {}
    for b in DECODE_BATCHES:
        y_o, idx_o, _, _ = oracle_out[b]
        r = ops.moe_route(x[:b], w.router, shape.top_k, shape.norm_topk, want_probs=False)
        idx = r["topk_idx"].cpu().numpy()
        res[str(b)] = dict(index_mismatches=int((idx != idx_o).any(axis=1).sum()),
                           rel_l2=float(f"{O.rel_l2(gpu_out[b].float().cpu().numpy(), y_o):.3e}"))
    return dict(decode_vs_oracle=res, tolerance="indices bit-exact, rel-L2 <= 1e-2 (bf16)",
                literal_bf16_reference_vs_contract=_published_literal_mismatches())


def cpu_baseline(w, x_dev, mask_host, shape, workload, xp_dev=None, bias=None, budget_s=15.0,
                 gpu_out=None):
    """(the timed oracle port on the host cores, parity of the GPU results on the
    same inputs)."""
    cw = _cpu_weights(w)
    avail = mask_host.numpy().astype(np.float32)
    parity = None
    if workload == "decode":
        x = x_dev.float().cpu().numpy()
        t0 = time.perf_counter()
        reps = 0
        first = {}
        while True:
            for b in DECODE_BATCHES:
                out = _oracle_call(cw, x[:b], avail, shape)
                if b not in first:
                    first[b] = out
            reps += 1
            if time.perf_counter() - t0 > budget_s or reps >= 5:
                break
        dt = time.perf_counter() - t0
        if gpu_out is not None:
            parity = _decode_parity(x_dev, w, cw, avail, shape, first, gpu_out)
        return dict(value=round(reps * sum(DECODE_BATCHES) / dt, 2), unit="tokens/s",
                    cores=_threads(), kind="port",
                    sample=f"{reps} decode step(s) (batches 1/8/32/64) of the oracle port "
                           "(C router + numpy/BLAS fp32 experts)"), parity
    x = xp_dev[:512].float().cpu().numpy()
    b = bias.float().cpu().numpy()
    t0 = time.perf_counter()
    _oracle_call(cw, x, None, shape, bias=b)
    dt = time.perf_counter() - t0
    return dict(value=round(512 / dt, 2), unit="tokens/s", cores=_threads(), kind="port",
                sample="512 of the 8192 prefill tokens through the oracle port"), parity


def run_reference(args, dist: Dist):
    from project_chronos_b200 import synthetic as syn
    spec = syn.WORKLOADS["decode"]
    shape = spec["shape"]
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    wl = syn.make_workload(shape, max(DECODE_BATCHES), seed=1234, dtype=torch.bfloat16,
                           device=dev, avail_p=spec["avail_p"])
    cw = _cpu_weights(wl.weights)
    mask = wl.mask.cpu().numpy().astype(np.float32)
    x = wl.x.float().cpu().numpy()
    if args.workload == "prefill":
        g = syn.make_generator(99, dev)
        xp = syn.make_hidden(PREFILL_TOKENS, shape.hidden, g, dtype=torch.bfloat16, device=dev)
        bias = syn.make_zipf_bias(shape.num_experts, 1.1, g, dev).float().cpu().numpy()
        sample_tokens = 256
        xs = xp[:sample_tokens].float().cpu().numpy()

        def step():
            _oracle_call(cw, xs, None, shape, bias=bias)
        tokens = sample_tokens
        metric = METRIC_PREFILL
        sample = f"{sample_tokens} of the 8192 prefill tokens per step"
    else:
        def step():
            for b in DECODE_BATCHES:
                _oracle_call(cw, x[:b], mask, shape)
        tokens = sum(DECODE_BATCHES)
        metric = METRIC_DECODE
        sample = "one decode step (batches 1/8/32/64) per step"
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = tokens * args.steps / dt
    cores = _threads()
    return {
        "impl": "reference", "metric": metric, "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(args, dist.world),
        "host_side": "the oracle port on the host cores (rank 0 only), fp32",
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("decode", "prefill", "ep"), default="decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    dist = Dist()
    if args.impl == "reference":
        if dist.rank != 0:
            return 0
        print(json.dumps(run_reference(args, dist)), flush=True)
        return 0
    if not torch.cuda.is_available():
        print(json.dumps({"error": "no CUDA device"}))
        return 1
    dist.init()
    try:
        line = run_ours(args, dist)
    finally:
        torch.cuda.synchronize()
        dist.close()
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
