"""Benchmark: ragged decode tokens/s of the hybrid Qwen MoE (4-bit) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: Qwen3-Next-80B-A3B-shaped random-init
weights (48 layers = 12 x [3 Gated-DeltaNet, 1 gated attention], each with a
512-expert top-10 + shared-expert MoE; 4-bit affine g64, bf16 scale/bias),
64 ragged decode sequences with contexts log-uniform over [128, 32768] (seed
0), KV pages of 16 tokens. The prefix state of every sequence is seeded
synthetic state (rs_qwen_device_synthetic_state) standing in for a prefill.
One step = one greedy decode token for every sequence through
rs_qwen_device_step_ragged (the C ABI), parents consumed in place.

Multi-GPU (--gpus N under torchrun): sequence-sharded independent replicas,
64 sequences per GPU, no data-path collective; timing is the max over ranks.
"""
from __future__ import annotations

import argparse
import importlib
import json
import re
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
PKG_NAME = "rust-ts-tokio-inference-engine_b200"

N_SEQ = 64
CTX_LO, CTX_HI = 128, 32768
SEED = 0
METRIC = "ragged decode tokens/s (hybrid Qwen MoE 4-bit) at 1/2/4/8 B200; p50 step ms"
W4_BYTES_PER_PARAM = 0.5625  # 4-bit + bf16 scale + bf16 bias per 64


def contexts(n, seed):
    rng = np.random.default_rng(seed)
    return np.floor(np.exp(rng.uniform(math.log(CTX_LO), math.log(CTX_HI), size=n))).astype(np.int64)


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled during the timed region.
    Sampling starts before the warm-up (nvidia-smi takes a while to print its
    first line); summary() keeps the samples read between begin() and end()."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu, self.rows, self.proc = gpu_index, [], None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.perf_counter(), [x.strip() for x in line.split(",")]))

    def begin(self):
        self.t0 = time.perf_counter()

    def end(self):
        self.t1 = time.perf_counter()
        time.sleep(0.15)  # the sample covering the last timed step
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        lo, hi = self.t0 or 0.0, (self.t1 or float("inf")) + 0.15
        rows = [r for t, r in self.rows if lo <= t <= hi]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) > 8 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def stage_bytes(cfg, ctx, routing, expert_range=None):
    """Algorithmic HBM bytes per step for each operator stage (device-layout bytes).
    With expert_range = (lo, hi) (expert parallelism) the MoE terms count the
    experts of that block hit by `routing` (every rank's tokens) and the rows
    routed to them."""
    H, E, I = cfg.hidden, cfg.experts, cfg.intermediate
    n_attn = cfg.layers // cfg.interval
    n_gdn = cfg.layers - n_attn
    B = len(ctx)
    kd, vd = cfg.key_heads * cfg.key_dim, cfg.value_heads * cfg.value_dim
    cd = 2 * kd + vd
    gdn_in = cd + vd + 2 * cfg.value_heads
    attn_in = cfg.q_heads * 2 * cfg.head_dim + 2 * cfg.kv_heads * cfg.head_dim
    w = W4_BYTES_PER_PARAM
    out = {}
    out["RecurrentProjection"] = n_gdn * (gdn_in * H * w + B * H * 2 + B * gdn_in * 4)
    out["RecurrentUpdate"] = n_gdn * B * (cfg.value_heads * cfg.value_dim * cfg.key_dim * 4 * 2 +
                                          (cfg.conv - 1) * cd * 4 * 2 + gdn_in * 4 + vd * 2)
    out["RecurrentOutput"] = n_gdn * (H * vd * w + B * vd * 2 + B * H * 4)
    out["AttentionProjection"] = n_attn * (attn_in * H * w + B * H * 2 + B * attn_in * 4)
    kv_per_tok = 2 * cfg.kv_heads * cfg.head_dim * 2
    out["AttentionReduction"] = n_attn * (float(np.sum(ctx + 1)) * kv_per_tok + B * attn_in * 4)
    out["AttentionOutput"] = n_attn * (H * cfg.q_heads * cfg.head_dim * w + B * H * 4)
    out["MoeRouting"] = cfg.layers * ((E + 1) * H * w + B * H * 2)
    rows = cfg.layers * B * (cfg.top + 1)
    if expert_range is not None:
        lo, hi = expert_range
        distinct = [len(np.unique(r[(r >= lo) & (r < hi)])) for r in routing]
        rows = float(sum(np.count_nonzero((r >= lo) & (r < hi)) for r in routing)) + cfg.layers * B
    elif routing is not None:
        distinct = [len(np.unique(routing[layer])) for layer in range(routing.shape[0])]
    else:
        distinct = [E * (1 - (1 - cfg.top / E) ** B)] * cfg.layers
    ue = np.array(distinct, np.float64) + 1  # + shared expert
    out["MoeUpGate"] = float(np.sum(ue * 2 * I * H * w)) + rows * (H * 2 + I * 2)
    out["MoeDown"] = float(np.sum(ue * H * I * w)) + rows * (I * 2 + H * 4)
    out["FinalProjection"] = cfg.vocab * H * w + B * cfg.vocab * 4
    return out, float(np.mean(ue))


STAGES = ["Embedding", "InputNorm", "RecurrentProjection", "RecurrentPrepare", "RecurrentUpdate",
          "RecurrentOutput", "AttentionProjection", "AttentionReduction", "AttentionOutput", "ResidualNorm",
          "MoeRouting", "MoeUpGate", "MoeDown", "MoeMixture", "MoeShared", "MoeMerge", "LayerOutput",
          "FinalProjection", "StateValidation"]


def dist_setup(n_gpus):
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world != n_gpus and world > 1:
        raise SystemExit(f"WORLD_SIZE {world} != --gpus {n_gpus}")
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        # NCCL between GPU ranks (one process per GPU), gloo when there is no GPU;
        # a short timeout so a rank that never arrives ends the others with an error
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    return rank, world, local


def max_over_ranks(value, world):
    """The largest value over all ranks (timings are max over ranks)."""
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# Launches per 48-layer step of each stage's dominant kernel.
LAUNCHES_PER_STEP = {"MoeUpGate": 48, "MoeDown": 48, "RecurrentUpdate": 36, "AttentionReduction": 12}
# ncu DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum), read from the committed
# profile summary of that stage's kernel on the same per-layer shapes.
PROFILE_FILES = {"MoeUpGate": "qgemm_tc_moe_gateup_cfg1.md", "MoeDown": "qgemm_tc_moe_down_cfg1.md"}


def profiled_traffic(stage):
    f = Path(__file__).resolve().parent / "profiles" / PROFILE_FILES.get(stage, "-")
    if not f.is_file():
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


def cpu_reference(cfg_kw, ctx, steps, warmup, cores_note=None):
    """The oracle port timed on the host cores: one sequence's decode token
    through a 4-layer slice of the configs[1] model (3 DeltaNet + 1 attention
    layer, each + MoE) at the workload's mean context, scaled to 48 layers.
    Weights the sample touches are generated before timing."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    O.build()
    L = int(np.mean(ctx))
    ocfg = O.config1(layers=4, context=L + 8)
    model = O.Model(ocfg, SEED)
    rng = np.random.default_rng(1)
    state = (rng.standard_normal(model.state_count()) * 0.02).astype(np.float32)
    tok = [1234]
    model.forward(tok, L, old_state=state)  # generate the touched weights
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        model.forward(tok, L, old_state=state)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    per_tok_48 = statistics.median(times) * (cfg_kw["layers"] / 4)
    cores = os.cpu_count() or 1
    return {"value": 1.0 / per_tok_48, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"1 decode token of 1 sequence at context {L} through a 4-layer configs[1] slice "
                      f"(FP64 oracle, {cores} threads), median of {steps}, x{cfg_kw['layers'] // 4} to 48 layers"}, times


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--ep", action="store_true",
                    help="expert parallelism: routed experts split over the ranks, rows stored straight into the "
                         "owner's window over NVLink")
    ap.add_argument("--ep-nccl", action="store_true", help="expert parallelism with NCCL send/recv stages instead")
    args = ap.parse_args()
    rank, world, local = dist_setup(args.gpus)
    cfg_kw = dict(layers=args.layers)
    config = {"workload": "configs[1]: 64 ragged decode seqs, contexts logU[128,32768], 48L Qwen3-Next-80B-A3B "
                          "shapes, 4-bit g64", "seqs_per_gpu": N_SEQ, "page_tokens": 16,
              "parallelism": (f"ep{args.gpus}-nccl" if args.ep_nccl else f"ep{args.gpus}") if args.ep or args.ep_nccl
              else f"replicas{args.gpus}",
              "l2": "inputs larger than L2 (44.8 GB weights per step)"}

    if args.impl == "reference":
        if rank != 0:
            return
        ctx = contexts(N_SEQ, SEED)
        base, times = cpu_reference(cfg_kw, ctx, args.steps, args.warmup)
        line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "tokens/s",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": statistics.median(times) * 1e3 * (args.layers / 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
                "data": "synthetic", "config": config, "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch
    torch.cuda.set_device(local)
    pkg = importlib.import_module(PKG_NAME)
    cfg = pkg.config1(**cfg_kw)
    ctx = contexts(N_SEQ, SEED + rank)
    store = pkg.WeightStore().synthetic(cfg, SEED)
    gdn_slot = (cfg.layers - cfg.layers // cfg.interval) * (
        cfg.value_heads * cfg.value_dim * cfg.key_dim + (cfg.conv - 1) * (
            2 * cfg.key_heads * cfg.key_dim + cfg.value_heads * cfg.value_dim)) * 4
    page_bytes = (cfg.layers // cfg.interval) * 2 * cfg.kv_heads * 16 * cfg.head_dim * 2
    total_steps = args.warmup + args.steps + 2 + 5  # + capture step + 5 profiled steps
    pages = int(sum((L + total_steps + 15) // 16 + 1 for L in ctx)) + 64
    slots = N_SEQ + 8
    budget = slots * gdn_slot + pages * page_bytes
    sess = pkg.DeviceSession(store, cfg, slots=slots, budget_bytes=budget)
    args.ep = args.ep or args.ep_nccl
    if args.ep:  # every rank joins before its first step; all ranks then step in lockstep
        import torch.distributed as dist
        if args.ep_nccl:
            obj = [pkg.ep_unique_id() if rank == 0 else None]
            if world > 1:
                dist.broadcast_object_list(obj, src=0)
            sess.ep_init(world, rank, obj[0], N_SEQ)
        else:
            handle = sess.ep_window(world, rank, N_SEQ)
            handles = [handle]
            if world > 1:
                handles = [None] * world
                dist.all_gather_object(handles, handle)
            sess.ep_connect(handles)
    parents = [sess.synthetic_state(int(L), 1000 + s) for s, L in enumerate(ctx)]
    pos = ctx.astype(np.uint32).copy()
    rng = np.random.default_rng(SEED)
    tokens = rng.integers(0, cfg.vocab, size=N_SEQ).astype(np.uint32)
    ones = np.ones(N_SEQ, np.uint32)
    flags = pkg.RAGGED_SAMPLED | pkg.RAGGED_CONSUME
    sampled = np.zeros(N_SEQ, np.uint32)

    def one_step():
        nonlocal parents, tokens, pos
        outs, s, _ = sess.step_ragged(parents, pos, ones, tokens, flags=flags, sampled_out=sampled)
        parents, tokens, pos = outs, s.copy(), pos + 1

    clocks = ClockSampler(local).start()
    for _ in range(args.warmup):
        one_step()
    # Timed region: whole-step CUDA events only (per-stage events would sit
    # between kernels and serialise programmatic launches).
    sess.set_profile(False)
    _, total0, n0, _ = sess.timing()
    step_ms = []
    launches0 = sess.stats()[16]
    barrier(world)
    torch.cuda.synchronize()
    clocks.begin()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
        step_ms.append(sess.timing()[0])
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clocks.end()
    barrier(world)
    launches = int(sess.stats()[16] - launches0)
    _, total1, n1, _ = sess.timing()
    # Stage breakdown from a few more steps with per-stage events.
    prof_steps = 5
    sess.set_profile(True)
    _, _, _, stage0 = sess.timing()
    for _ in range(prof_steps):
        one_step()
    _, _, _, stage1 = sess.timing()
    sess.set_profile(False)
    sess.set_capture(True)
    one_step()
    routing = sess.debug_routing(N_SEQ)
    sess.set_capture(False)
    expert_range = None
    if args.ep:  # this rank's expert block is hit by every rank's tokens
        if world > 1:
            import torch.distributed as dist
            t = torch.from_numpy(np.ascontiguousarray(routing)).to("cuda")
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            routing = np.concatenate([x.cpu().numpy() for x in parts], axis=1)
        per = cfg.experts // world
        expert_range = (rank * per, (rank + 1) * per)
    dev_s = (total1 - total0) / 1e3
    dev_s = max_over_ranks(dev_s, world)
    wall = max_over_ranks(wall, world)
    tokens_total = N_SEQ * args.steps * world
    value = tokens_total / dev_s
    e2e = tokens_total / wall
    stage_ms = [(b - a) / prof_steps for a, b in zip(stage0, stage1)]
    barrier(world)  # every rank has finished its steps (expert-parallel windows stay valid until here)
    if rank != 0:
        return
    hbm, tflops, peak_kind = measured_peaks()
    bytes_per, mean_ue = stage_bytes(cfg, ctx, routing, expert_range)
    dom = max(bytes_per, key=lambda k: stage_ms[STAGES.index(k)])
    dom_ms = stage_ms[STAGES.index(dom)]
    achieved = bytes_per[dom] / (dom_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_s * 1e3 / args.steps,
        "p50_step_ms": statistics.median(step_ms), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights, synthetic prefix state)",
        "config": config,
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": N_SEQ * (4 + 48) + N_SEQ * 4,
                "d2h_bytes_per_step": N_SEQ * 4 + 4},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": profiled_traffic(dom), "peak_source": peak_kind,
                     "bytes_per_step": bytes_per[dom], "ms_per_step": dom_ms,
                     "algorithmic_bytes_per_launch": bytes_per[dom] / LAUNCHES_PER_STEP.get(dom, 1)},
        "stage_ms": {k: round(v, 4) for k, v in zip(STAGES, stage_ms) if v > 0},
        "stage_gbs": {k: round(bytes_per[k] / (stage_ms[STAGES.index(k)] / 1e3) / 1e9, 1)
                      for k in bytes_per if stage_ms[STAGES.index(k)] > 0},
        "step_bytes_gb": round(sum(bytes_per.values()) / 1e9, 3), "mean_distinct_experts": round(mean_ue, 1),
        "clocks": clocks.summary(),
    }
    line["roofline_step"] = {"achieved": sum(bytes_per.values()) / (dev_s / args.steps) / 1e9, "peak": hbm,
                             "frac": sum(bytes_per.values()) / (dev_s / args.steps) / 1e9 / hbm}
    if not args.no_cpu_baseline and world == 1:
        base, _ = cpu_reference(cfg_kw, ctx, 3, 1)
        line["cpu_baseline"] = base
    print(json.dumps(line))


if __name__ == "__main__":
    try:
        main()
    finally:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()
