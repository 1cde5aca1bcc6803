"""Benchmark: ragged decode tokens/s of the hybrid Qwen MoE (4-bit) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg1|cfg2|cfg3|cfg4] [--parallel auto|replicas|ep|ep-nccl]

Model: Qwen3-Next-80B-A3B-shaped random-init
weights (48 layers = 12 x [3 Gated-DeltaNet, 1 gated attention], each with a
512-expert top-10 + shared-expert MoE; 4-bit affine g64), KV pages of 16
tokens. Prefix states are seeded synthetic state (rs_qwen_device_synthetic_state)
standing in for prefills; no dataset is involved. Workloads:

  cfg1 (default)  64 ragged decode sequences per GPU, contexts logU[128, 32768]
                  (seed 0); one step = one greedy token per sequence through
                  rs_qwen_device_step_ragged, parents consumed in place.
  cfg2            configs[2]: 120 decode sequences, contexts logU[256, 16384],
                  plus 8 prompts U[512, 4096] chunk-prefilled first come first
                  served under a 2048-token budget, all packed into one ragged
                  step (a finished prompt is replaced by a new one).
  cfg3            configs[3]: 128 sequences, contexts logU[128, 8192]; one step =
                  speculative verify + accept of 3 drafts per sequence through
                  rs_qwen_device_mtp_verify_accept; each draft is the target's
                  greedy token with probability 0.7, else uniform (seeded). The
                  greedy continuation is computed before timing; drafting itself
                  is not timed.
  cfg4            configs[4]: 512 decode sequences in total (logU[128, 32768])
                  split over the N GPUs (strong scaling).

Multi-GPU (--gpus N under torchrun, one process per GPU): --parallel auto is
expert parallelism over direct NVLink stores (routed experts split over the
ranks, MoE rows stored into the owner's window); replicas (sequence-sharded,
no collective) and NCCL send/recv expert parallelism are selectable. Device
time is taken with CUDA events and the maximum over ranks is reported.

--impl reference times the CPU restatement of the same step (oracle/fp32_step.cpp,
fp32, all host threads) on a bounded sample: the workload's batch through a
4-layer slice of the model (3 DeltaNet + 1 attention layer with their MoE,
exactly 1/12 of the 48 layers) plus the final norm and vocabulary projection,
scaled to 48 layers. The reference's own implementation (Apple MLX + Metal,
Rust) cannot run on this machine.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import re
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
W4_BYTES_PER_PARAM = 0.5625  # 4-bit + 16-bit scale + 16-bit bias per 64
PREFILL_BUDGET = 2048

WORKLOADS = {
    "cfg1": "configs[1]: 64 ragged decode seqs per GPU, contexts logU[128,32768], Qwen3-Next-80B-A3B shapes, 4-bit g64",
    "cfg2": "configs[2]: 120 decode seqs logU[256,16384] + 8 prompts U[512,4096] chunk-prefilled under a 2048-token "
            "budget, one packed ragged step",
    "cfg3": "configs[3]: 128 seqs logU[128,8192], speculative verify+accept of 3 drafts (p=0.7 target argmax)",
    "cfg4": "configs[4]: 512 ragged decode seqs in total over the GPUs, contexts logU[128,32768]",
}


def contexts(n, seed, lo=CTX_LO, hi=CTX_HI):
    rng = np.random.default_rng(seed)
    return np.floor(np.exp(rng.uniform(math.log(lo), math.log(hi), size=n))).astype(np.int64)


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


def gdn_slot_bytes(cfg):
    """Bytes of one sequence's DeltaNet state over all DeltaNet layers (fp32
    recurrent state + conv history): the session's per-version slot."""
    n_gdn = cfg.layers - cfg.layers // cfg.interval
    cd = 2 * cfg.key_heads * cfg.key_dim + cfg.value_heads * cfg.value_dim
    return n_gdn * (cfg.value_heads * cfg.value_dim * cfg.key_dim + (cfg.conv - 1) * cd) * 4


def kv_page_bytes(cfg):
    """Bytes of one 16-token KV page over all attention layers (bf16 K and V)."""
    return (cfg.layers // cfg.interval) * 2 * cfg.kv_heads * 16 * cfg.head_dim * 2


def stage_bytes(cfg, ctx, routing, expert_range=None, counts=None):
    """Algorithmic HBM bytes per step for each operator stage (device-layout
    bytes). ctx: each sequence's context before the step; counts: its new
    tokens (default 1). Per sequence and layer the recurrent state is read and
    written once and the K/V of its whole context are read once; per token the
    projection rows move once; each distinct expert's weights are read once per
    layer. With expert_range = (lo, hi) (expert parallelism) the MoE terms count
    the experts of that block hit by `routing` and the rows routed to them."""
    H, E, I = cfg.hidden, cfg.experts, cfg.intermediate
    n_attn = cfg.layers // cfg.interval
    n_gdn = cfg.layers - n_attn
    ctx = np.asarray(ctx, np.int64)
    counts = np.ones_like(ctx) if counts is None else np.asarray(counts, np.int64)
    B, T = len(ctx), int(counts.sum())
    kd, vd = cfg.key_heads * cfg.key_dim, cfg.value_heads * cfg.value_dim
    cd = 2 * kd + vd
    gdn_in = cd + vd + 2 * cfg.value_heads
    attn_in = cfg.q_heads * 2 * cfg.head_dim + 2 * cfg.kv_heads * cfg.head_dim
    w = W4_BYTES_PER_PARAM
    out = {}
    out["RecurrentProjection"] = n_gdn * (gdn_in * H * w + T * H * 2 + T * gdn_in * 4)
    out["RecurrentUpdate"] = n_gdn * (B * (cfg.value_heads * cfg.value_dim * cfg.key_dim * 4 * 2 +
                                           (cfg.conv - 1) * cd * 4 * 2) + T * (gdn_in * 4 + vd * 2))
    out["RecurrentOutput"] = n_gdn * (H * vd * w + T * vd * 2 + T * H * 4)
    out["AttentionProjection"] = n_attn * (attn_in * H * w + T * H * 2 + T * attn_in * 4)
    kv_per_tok = 2 * cfg.kv_heads * cfg.head_dim * 2
    out["AttentionReduction"] = n_attn * (float(np.sum(ctx + counts)) * kv_per_tok + T * attn_in * 4)
    out["AttentionOutput"] = n_attn * (H * cfg.q_heads * cfg.head_dim * w + T * H * 4)
    out["MoeRouting"] = cfg.layers * ((E + 1) * H * w + T * H * 2)
    rows = cfg.layers * T * (cfg.top + 1)
    if expert_range is not None:
        lo, hi = expert_range
        distinct = [len(np.unique(r[(r >= lo) & (r < hi)])) for r in routing]
        rows = float(sum(np.count_nonzero((r >= lo) & (r < hi)) for r in routing)) + cfg.layers * T
    elif routing is not None:
        distinct = [len(np.unique(routing[layer])) for layer in range(routing.shape[0])]
    else:
        distinct = [E * (1 - (1 - cfg.top / E) ** T)] * cfg.layers
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


def sum_over_ranks(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# Launches per 48-layer step of each stage's dominant kernel.
def launches_per_step(stage, cfg):
    """Launches of a stage's main kernel per step: one per layer of its kind."""
    n_attn = cfg.layers // cfg.interval
    return {"MoeUpGate": cfg.layers, "MoeDown": cfg.layers, "RecurrentUpdate": cfg.layers - n_attn,
            "AttentionReduction": n_attn}.get(stage, 1)


# ncu DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum), read from the committed
# profile summary of that stage's kernel on the same per-layer shapes.
PROFILE_FILES = {"MoeUpGate": "qgemm_tc_moe_gateup_cfg1.md", "MoeDown": "qgemm_tc_moe_down_cfg1.md"}


def profiled_traffic(stage):
    f = ROOT / "profiles" / PROFILE_FILES.get(stage, "-")
    if not f.is_file():
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


def workload_label(workload, layers):
    label = WORKLOADS[workload]
    if layers != 48:
        label += f" [{layers}-layer slice: NOT the 48-layer configs[1] model]"
    return label


# ------------------------------------------------------------- CPU baseline --

def cpu_sample_batch(workload, rank=0):
    """The decode batch the CPU sample runs (contexts), per workload."""
    if workload == "cfg2":
        return contexts(120, SEED, 256, 16384)
    if workload == "cfg3":
        return contexts(128, SEED, 128, 8192)
    if workload == "cfg4":
        return contexts(512, SEED)[:64]  # a 64-sequence sample of the 512
    return contexts(N_SEQ, SEED + rank)


def cpu_reference(workload, layers, steps, warmup):
    """The fp32 CPU restatement (oracle/fp32_step.cpp) timed on all host
    threads: the workload's decode batch, one token per sequence, through a
    4-layer slice of the model (3 DeltaNet + 1 attention layer with their MoE
    = 1/12 of the 48 layers) and the final projection; 48-layer step time =
    12 x slice + head. Weights and prefix states are generated before timing."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    O.build()
    ctx = cpu_sample_batch(workload)
    cfg = O.config1(layers=4, context=int(ctx.max()) + warmup + steps + 16)
    model = O.F32Step(cfg, SEED)
    model.set_batch(ctx, None, seed=SEED + 17, extra=warmup + steps + 8)
    tok = np.random.default_rng(SEED).integers(0, cfg.vocab, size=len(ctx)).astype(np.uint32)
    per_step, walls, stages = [], [], []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        tok, _, t_layers, t_head = model.step(tok)
        wall = time.perf_counter() - t0
        if i >= warmup:
            per_step.append((layers / 4) * t_layers + t_head)
            walls.append(wall)
            stages.append(model.stage_seconds())
    step_s = statistics.median(per_step)
    gdn, attn, moe = (statistics.median(s[i] for s in stages) for i in range(3))
    sample = (f"{len(ctx)} decode seqs of {workload} (contexts as the workload), one token each, through a 4-layer "
              f"slice of the configs[1] model + final projection, fp32, {model.threads} threads; 48-layer step = "
              f"{layers // 4} x slice + head; median of {steps}")
    info = {"value": len(ctx) / step_s, "unit": "tokens/s", "cores": model.threads, "kind": "port",
            "dtype": "f32", "sample": sample, "step_s_48L": step_s, "sample_s": statistics.median(walls),
            "per_layer_s": {"deltanet": gdn / 3, "attention": attn, "moe": moe / 4}}
    return info, walls


# ----------------------------------------------------------------- drivers --

class TimedCalls:
    """Runs a driver's timed C-ABI call and keeps its accounting: kernel
    launches and host-to-device bytes of timed calls only (the session's own
    counters, rs_qwen_device_stats words 16 and 3), device ms (CUDA events
    around the step on the session stream) and the call's wall seconds."""

    def __init__(self, sess):
        self.sess, self.launches, self.h2d = sess, 0, 0

    def run(self, fn):
        st0 = self.sess.stats()
        t0 = time.perf_counter()
        out = fn()
        wall = time.perf_counter() - t0
        st1 = self.sess.stats()
        self.launches += st1[16] - st0[16]
        self.h2d += st1[3] - st0[3]
        return out, self.sess.timing()[0], wall


class Cfg1Driver:
    """Decode steps for a fixed batch (cfg1 / cfg4): one token per sequence."""

    CALLS_PER_STEP = 1  # session steps per driver step (stage profiles are divided by it)

    def __init__(self, pkg, sess, cfg, ctx, seeds0):
        self.pkg, self.sess, self.cfg = pkg, sess, cfg
        self.n = len(ctx)
        self.parents = [sess.synthetic_state(int(L), seeds0 + s) for s, L in enumerate(ctx)]
        self.pos = np.asarray(ctx, np.uint32).copy()
        self.ctx0 = np.asarray(ctx, np.int64)
        self.tokens = np.random.default_rng(SEED).integers(0, cfg.vocab, size=self.n).astype(np.uint32)
        self.ones = np.ones(self.n, np.uint32)
        self.sampled = np.zeros(self.n, np.uint32)
        self.flags = pkg.RAGGED_SAMPLED | pkg.RAGGED_CONSUME
        self.calls = TimedCalls(sess)

    def step(self):
        (outs, s, _), dev_ms, wall = self.calls.run(lambda: self.sess.step_ragged(
            self.parents, self.pos, self.ones, self.tokens, flags=self.flags, sampled_out=self.sampled))
        self.parents, self.tokens, self.pos = outs, s.copy(), self.pos + 1
        return self.n, {"decode_tokens": self.n}, dev_ms, wall

    def bytes_ctx(self):
        return self.pos.astype(np.int64), None

    def d2h(self):
        return self.n * 4 + 4


class Cfg2Driver:
    """Mixed steps: 120 decode sequences + 8 prompts chunk-prefilled first come
    first served under a 2048-token budget, packed into one ragged step."""

    CALLS_PER_STEP = 1

    def __init__(self, pkg, sess, cfg, rank):
        self.pkg, self.sess, self.cfg = pkg, sess, cfg
        dctx = contexts(120, SEED + 2 + rank, 256, 16384)
        self.rng = np.random.default_rng(SEED + 3 + rank)
        self.dec = [sess.synthetic_state(int(L), 3000 + s) for s, L in enumerate(dctx)]
        self.dpos = dctx.astype(np.uint32).copy()
        self.dtok = self.rng.integers(0, cfg.vocab, size=120).astype(np.uint32)
        self.prompts = [self._new_prompt() for _ in range(8)]
        self.flags = pkg.RAGGED_SAMPLED | pkg.RAGGED_CONSUME
        self.calls = TimedCalls(sess)
        self.last_ctx, self.last_counts = None, None
        self.prefill_done = 0

    def _new_prompt(self):
        n = int(self.rng.integers(512, 4097))
        return {"tokens": self.rng.integers(0, self.cfg.vocab, size=n).astype(np.uint32), "done": 0, "state": None}

    def step(self):
        budget = PREFILL_BUDGET
        chunks = []
        for p in self.prompts:  # first come first served
            if budget == 0:
                break
            c = min(budget, len(p["tokens"]) - p["done"])
            chunks.append((p, c))
            budget -= c
        parents = [p["state"] for p, _ in chunks] + self.dec
        positions = [p["done"] for p, _ in chunks] + list(self.dpos)
        counts = [c for _, c in chunks] + [1] * 120
        toks = np.concatenate([p["tokens"][p["done"]:p["done"] + c] for p, c in chunks] + [self.dtok])
        self.last_ctx = np.array(positions, np.int64)
        self.last_counts = np.array(counts, np.int64)
        (outs, sampled, _), dev_ms, wall = self.calls.run(
            lambda: self.sess.step_ragged(parents, positions, counts, toks, flags=self.flags))
        n_pf = len(chunks)
        for i, (p, c) in enumerate(chunks):
            p["state"], p["done"] = outs[i], p["done"] + c
        self.dec, self.dtok, self.dpos = outs[n_pf:], sampled[n_pf:].copy(), self.dpos + 1
        for i, p in enumerate(self.prompts):  # a finished prompt is replaced by a new one
            if p["done"] == len(p["tokens"]):
                self.sess.release(p["state"])
                self.prompts[i] = self._new_prompt()
                self.prefill_done += 1
        pf = int(sum(c for _, c in chunks))
        return pf + 120, {"decode_tokens": 120, "prefill_tokens": pf}, dev_ms, wall

    def bytes_ctx(self):
        return self.last_ctx, self.last_counts

    def d2h(self):
        return int(len(self.last_counts)) * 4 + 4


class Cfg3Driver:
    """Speculative verify + accept of 3 drafts for 128 sequences; each draft is
    the target's greedy token with probability 0.7, else uniform. The target's
    greedy tokens for the next three positions come from three untimed verify
    passes that feed the tokens found so far (a row depends only on the tokens
    before it, so the timed pass computes the same rows); only the fourth,
    timed pass counts."""

    P_ACCEPT, DRAFTS = 0.7, 3
    CALLS_PER_STEP = 4  # three greedy passes + the timed pass, all of the same shape

    def __init__(self, pkg, sess, cfg, rank):
        self.pkg, self.sess, self.cfg = pkg, sess, cfg
        ctx = contexts(128, SEED + 4 + rank, 128, 8192)
        self.n = 128
        self.rng = np.random.default_rng(SEED + 5 + rank)
        self.parents = [sess.synthetic_state(int(L), 5000 + s) for s, L in enumerate(ctx)]
        self.pos = ctx.astype(np.uint32).copy()
        self.seeds = self.rng.integers(0, cfg.vocab, size=self.n).astype(np.uint32)
        self.calls = TimedCalls(sess)
        self.accepted = []
        self.ctx = ctx

    def _greedy_drafts(self):
        g = np.zeros((self.n, self.DRAFTS), np.uint32)
        for j in range(self.DRAFTS):
            outs, _, emitted = self.sess.verify_accept(self.parents, self.seeds, [list(g[s]) for s in range(self.n)])
            for o in outs:
                self.sess.release(o)
            g[:, j] = [e[j] for e in emitted]  # drafts 0..j-1 are the greedy tokens, so row j was emitted
        return g

    def step(self):
        g = self._greedy_drafts()
        keep = self.rng.random((self.n, self.DRAFTS)) < self.P_ACCEPT
        rnd = self.rng.integers(0, self.cfg.vocab, size=(self.n, self.DRAFTS)).astype(np.uint32)
        drafts = np.where(keep, g, rnd)
        (outs, acc, emitted), dev_ms, wall = self.calls.run(
            lambda: self.sess.verify_accept(self.parents, self.seeds, [list(d) for d in drafts]))
        for o in self.parents:
            self.sess.release(o)
        self.parents = outs
        ne = np.array([len(x) for x in emitted], np.int64)
        self.pos += (np.array(acc, np.int64) + 1).astype(np.uint32)
        self.seeds = np.array([e[-1] for e in emitted], np.uint32)
        self.accepted.extend(acc)
        return int(ne.sum()), {"emitted_tokens": int(ne.sum()), "fed_tokens": self.n * (self.DRAFTS + 1)}, dev_ms, wall

    def bytes_ctx(self):
        return self.pos.astype(np.int64), np.full(self.n, self.DRAFTS + 1, np.int64)

    def d2h(self):  # accepted count, 9 emitted-token words (8 drafts + 1), emitted count per sequence; status word
        return self.n * (4 + 9 * 4 + 4) + 4


def setup_parallel(sess, mode, world, rank, cap_tokens, pkg):
    """Expert-parallel group set-up (every rank joins before its first step)."""
    if mode not in ("ep", "ep-nccl"):
        return
    import torch.distributed as dist
    if mode == "ep-nccl":
        obj = [pkg.ep_unique_id() if rank == 0 else None]
        if world > 1:
            dist.broadcast_object_list(obj, src=0)
        sess.ep_init(world, rank, obj[0], cap_tokens)
    else:
        handle = sess.ep_window(world, rank, cap_tokens)
        handles = [handle]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle)
        sess.ep_connect(handles)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg1", choices=sorted(WORKLOADS))
    ap.add_argument("--parallel", default="auto", choices=["auto", "replicas", "ep", "ep-nccl"],
                    help="multi-GPU mode; auto = expert parallelism over NVLink stores when N > 1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=48)
    args = ap.parse_args()
    rank, world, local = dist_setup(args.gpus)
    mode = args.parallel
    if mode == "auto":
        mode = "ep" if world > 1 and args.workload in ("cfg1", "cfg4") else "replicas"
    if mode != "replicas" and args.workload in ("cfg2", "cfg3"):
        raise SystemExit("cfg2 / cfg3 run as replicas only")
    strong = args.workload == "cfg4"
    config = {"workload": workload_label(args.workload, args.layers), "layers": args.layers, "page_tokens": 16,
              "parallelism": f"{mode}{args.gpus}" if args.gpus > 1 else "single",
              "l2": "inputs larger than L2 (44.8 GB of weights and the KV/state read per step)"}

    if args.impl == "reference":
        if rank != 0:
            return
        base, walls = cpu_reference(args.workload, args.layers, args.steps, args.warmup)
        line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "tokens/s",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": statistics.median(walls) * 1e3,
                "ms_per_step_note": "wall time of one timed sample step (4-layer slice + head); the 48-layer step "
                                    "the value is computed from is step_s_48L",
                "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic", "config": config, "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch
    torch.cuda.set_device(local)
    pkg = importlib.import_module(PKG_NAME)
    cfg = pkg.config1(layers=args.layers)
    store = pkg.WeightStore().synthetic(cfg, SEED)
    steps_all = args.warmup + args.steps + 8
    if args.workload == "cfg2":
        n_seq, tokens_cap = 128, 120 + PREFILL_BUDGET
        pages = int(sum((L + steps_all + 15) // 16 + 1 for L in contexts(120, SEED + 2 + rank, 256, 16384)))
        pages += 8 * (4096 // 16 + 2) * 2
        slots = 128 + 16
    elif args.workload == "cfg3":
        n_seq, tokens_cap = 128, 128 * 4
        horizon = 4 * (args.warmup + args.steps + 8) + 4
        ctx3 = contexts(128, SEED + 4 + rank, 128, 8192)
        # a verify step holds each parent and one candidate version per fed token
        # (5 per sequence); every version is charged its own page list
        pages = 5 * int(sum((L + horizon + 15) // 16 + 2 for L in ctx3))
        slots = 128 * 5 + 16
    else:
        if strong:
            allc = contexts(512, SEED)
            per = 512 // world
            ctx = allc[rank * per:(rank + 1) * per]
        else:
            ctx = contexts(N_SEQ, SEED + rank)
        n_seq, tokens_cap = len(ctx), len(ctx)
        pages = int(sum((L + steps_all + 15) // 16 + 1 for L in ctx)) + 64
        slots = n_seq + 8
    budget = slots * gdn_slot_bytes(cfg) + pages * kv_page_bytes(cfg)
    sess = pkg.DeviceSession(store, cfg, slots=slots, budget_bytes=budget)
    setup_parallel(sess, mode, world, rank, tokens_cap, pkg)
    if args.workload == "cfg2":
        drv = Cfg2Driver(pkg, sess, cfg, rank)
    elif args.workload == "cfg3":
        drv = Cfg3Driver(pkg, sess, cfg, rank)
    else:
        drv = Cfg1Driver(pkg, sess, cfg, ctx, 1000 if not strong else 1000 + rank * (512 // world))

    clocks = ClockSampler(local).start()
    for _ in range(args.warmup):
        drv.step()
    # Timed region: whole-step CUDA events only (per-stage events would sit
    # between kernels and serialise programmatic launches). Each driver step
    # returns its timed call's device milliseconds (CUDA events around the
    # step on the session stream) and the wall seconds of that C-ABI call;
    # untimed helper calls of a driver (cfg3's greedy passes) are excluded.
    sess.set_profile(False)
    step_ms, extras, walls = [], {}, []
    drv.calls.launches = drv.calls.h2d = 0
    barrier(world)
    torch.cuda.synchronize()
    clocks.begin()
    tokens_local = 0
    for _ in range(args.steps):
        n_tok, ex, ms, w = drv.step()
        tokens_local += n_tok
        for k, v in ex.items():
            extras[k] = extras.get(k, 0) + v
        step_ms.append(ms)
        walls.append(w)
    torch.cuda.synchronize()
    clocks.end()
    barrier(world)
    launches = int(drv.calls.launches)
    h2d = drv.calls.h2d / args.steps
    # Stage breakdown from a few more steps with per-stage events.
    prof_steps = 3
    sess.set_profile(True)
    _, _, _, stage0 = sess.timing()
    for _ in range(prof_steps):
        drv.step()
    _, _, _, stage1 = sess.timing()
    sess.set_profile(False)
    bctx, bcounts = drv.bytes_ctx()
    sess.set_capture(True)
    drv.step()
    t_cap = int(np.sum(bcounts)) if bcounts is not None and args.workload != "cfg2" else None
    if args.workload == "cfg2":
        bctx, bcounts = drv.bytes_ctx()
        t_cap = int(np.sum(bcounts))
    routing = sess.debug_routing(t_cap if t_cap else n_seq)
    sess.set_capture(False)
    expert_range = None
    if mode in ("ep", "ep-nccl") and world > 1:  # this rank's expert block is hit by every rank's tokens
        import torch.distributed as dist
        t = torch.from_numpy(np.ascontiguousarray(routing)).to("cuda")
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        routing = np.concatenate([x.cpu().numpy() for x in parts], axis=1)
        per_rank = cfg.experts // world
        expert_range = (rank * per_rank, (rank + 1) * per_rank)
    dev_s = max_over_ranks(sum(step_ms) / 1e3, world)
    wall = max_over_ranks(sum(walls), world)
    tokens_total = sum_over_ranks(tokens_local, world)
    extras = {k: sum_over_ranks(v, world) for k, v in extras.items()}
    value = tokens_total / dev_s
    e2e = tokens_total / wall
    stage_ms = [(b - a) / (prof_steps * drv.CALLS_PER_STEP) for a, b in zip(stage0, stage1)]
    d2h = drv.d2h()
    barrier(world)  # every rank has finished its steps (expert-parallel windows stay valid until here)
    if rank != 0:
        return
    hbm, tflops, peak_kind = measured_peaks()
    bytes_per, mean_ue = stage_bytes(cfg, bctx, routing, expert_range, bcounts)
    dom = max(bytes_per, key=lambda k: stage_ms[STAGES.index(k)])
    dom_ms = stage_ms[STAGES.index(dom)]
    achieved = bytes_per[dom] / (dom_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_s * 1e3 / args.steps,
        "p50_step_ms": statistics.median(step_ms), "step_ms": [round(x, 3) for x in step_ms],
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f16",
        "dtype_note": "projection operands IEEE half (4-bit weights dequantised with one rounding to 11 significant "
                      "bits, activations likewise), fp32 accumulation, fp32 recurrent state, bf16 KV cache",
        "data": "synthetic (seeded random-init weights, synthetic prefix state)", "config": config,
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": profiled_traffic(dom) if args.workload == "cfg1" else None,
                     "peak_source": peak_kind, "bytes_per_step": bytes_per[dom], "ms_per_step": dom_ms,
                     "algorithmic_bytes_per_launch": bytes_per[dom] / launches_per_step(dom, cfg)},
        "stage_ms": {k: round(v, 4) for k, v in zip(STAGES, stage_ms) if v > 0},
        "stage_gbs": {k: round(bytes_per[k] / (stage_ms[STAGES.index(k)] / 1e3) / 1e9, 1)
                      for k in bytes_per if stage_ms[STAGES.index(k)] > 0},
        "step_bytes_gb": round(sum(bytes_per.values()) / 1e9, 3), "mean_distinct_experts": round(mean_ue, 1),
        "clocks": clocks.summary(),
    }
    line["roofline_step"] = {"achieved": sum(bytes_per.values()) / (dev_s / args.steps) / 1e9, "peak": hbm,
                             "frac": sum(bytes_per.values()) / (dev_s / args.steps) / 1e9 / hbm}
    if extras:
        line["tokens"] = {k: v / dev_s for k, v in extras.items()}
        line["tokens"]["unit"] = "tokens/s by kind"
    if args.workload == "cfg3":
        acc = np.array(drv.accepted, np.float64)
        line["accept"] = {"mean_accepted_drafts": float(acc.mean()), "drafts": 3, "p_draft_correct": 0.7}
    if args.workload == "cfg2":
        line["prompts_completed"] = drv.prefill_done
    if not args.no_cpu_baseline and world == 1:
        base, _ = cpu_reference(args.workload, args.layers, 3, 1)
        line["cpu_baseline"] = base
    print(json.dumps(line))


if __name__ == "__main__":
    try:
        main()
    finally:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()
