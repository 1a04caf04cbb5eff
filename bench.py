#!/usr/bin/env python3
"""Qwen3-0.6B B=1 greedy decode on B200 - the benchmark of the reference's headline metric.

Workload (the reference's `--raw --benchmark 64` run): Qwen3-0.6B, bf16 weights random-init
N(0, 0.02) from seed 0 (norms 1.0) in Qwen3.bin layout, context 512, a 16-token prompt of
uniform random IDs in [0, 151936) (seed 0), then greedy decode steps. One bench step is one
greedy decode token at batch 1; the prompt is prefilled (untimed) before every run of 64 steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints one JSON line. Under torchrun (N > 1) every rank runs an independent replica (decode at
B=1 does not shard across replicas without a collective; the data-parallel configuration runs
independent sequences per GPU), the timed region is bracketed by barriers and the max time over
ranks is taken.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qwen3.cpp_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

METRIC = "decode tok/s (B=1, Qwen3-0.6B bf16)"
UNIT = "tok/s"
CTX = 512
PROMPT_LEN = 16
RUN_STEPS = 64
VOCAB = 151936
WEIGHT_BYTES = 1_191_968_768          # 28 layers + tied lm_head, bf16
KV_BYTES_PER_POS = 2 * 28 * 1024 * 2  # K and V rows of every layer
LM_HEAD_BYTES = VOCAB * 1024 * 2
# DRAM traffic of one fused decode step (dram__bytes_read.sum + dram__bytes_write.sum), from an
# `ncu --set full` capture of a one-step launch of `bench.py --legs decode --steps 8 --warmup 3`
# (kv_len ~17): 1.227272 GB read + 6.184704 MB written (the read includes the ~30 MB of the first
# layer's rows that a launch prefetches into L2 for the next one at its end). Re-captured whenever
# the kernel changes.
FUSED_TRAFFIC_PER_STEP = 1_233_456_704
# Long-prompt prefill: 2048 seeded prompt IDs (seed 2) at context 4096, batched on the tensor cores.
PREFILL_LEN = 2048
PREFILL_CTX = 4096
PREFILL_RUNS = 5


# Data-parallel batched decode: 64 sequences with context lengths uniform in [128, 4096] (seed 3)
# and seeded random prompts of those lengths, 16-token KV pages, 128 greedy steps each, the
# sequences split evenly over the ranks (strong scaling: the total work is fixed).
DP_SEQS = 64
DP_STEPS = 128
DP_WARMUP = 2


def dp_workload(n=DP_SEQS):
    """The first n (of 64) sequences of the seeded batched-decode workload."""
    import numpy as np
    rng = np.random.default_rng(3)
    lens = rng.integers(128, 4097, DP_SEQS)
    prompts = [rng.integers(0, VOCAB, int(n)).astype(np.int32) for n in lens]
    return lens[:n], prompts[:n]


# Tensor-parallel single-stream decode: context 32768, a 32000-token prompt of seeded random IDs
# (seed 4) prefilled on every rank, then 128 greedy steps with heads / MLP split over the ranks.
TP_ARM_COLLECTIVE = {
    "fused": "tagged words pushed to every rank from inside the persistent kernel's phases",
    "graph": "this library's one-shot all-reduce kernel after o_proj and down_proj, one CUDA "
             "graph per step",
    "graph_nccl": "ncclAllReduce after o_proj and down_proj and ncclAllGather of the greedy "
                  "candidates, captured in the same per-step CUDA graph",
}
TP_CTX = 32768
TP_PROMPT = 32000
TP_STEPS = 128
TP_WARMUP = 2


def prefill_flops(n: int) -> float:
    """Algorithmic FLOPs of a prefill of n tokens: the layer contractions (2 * n * 440,401,920),
    causal attention (4 * head_dim * n_heads * n_layers * n(n+1)/2) and the lm_head of the last
    token (2 * 151936 * 1024)."""
    return 2.0 * n * 440_401_920 + 4.0 * 128 * 16 * 28 * n * (n + 1) / 2 + 2.0 * VOCAB * 1024


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def prompt_ids():
    import numpy as np
    return np.random.default_rng(0).integers(0, VOCAB, PROMPT_LEN).astype(np.int32)


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def max_over_ranks(v: float, world: int, device: str = "cuda") -> float:
    """The largest of every rank's v (a time: the slowest rank's); v itself on one rank. A
    collective: every rank calls it at the same point."""
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dp_share(n_seqs: int, rank: int, world: int) -> list[int]:
    """This rank's sequences of the data-parallel workload: every world-th one from its rank
    (the ranks' shares are disjoint and cover all sequences; no collective on the data path)."""
    return list(range(rank, n_seqs, world))


def gather_handles(handle: bytes, world: int) -> list:
    """Every rank's exchange-buffer handle, in rank order (the tensor-parallel set-up)."""
    if world == 1:
        return [handle]
    import torch.distributed as dist
    handles = [None] * world
    dist.all_gather_object(handles, handle)
    return handles


class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(gpu_index), "-lms", "20"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.p = None
        # nvidia-smi takes a moment to start: wait (up to 3 s) for its first sample, so that the
        # timed region that follows is sampled.
        t0 = time.perf_counter()
        while self.p is not None and time.perf_counter() - t0 < 3.0:
            self.f.flush()
            if Path(self.f.name).stat().st_size > 0:
                break
            time.sleep(0.01)

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        self.p.wait(timeout=10)
        self.f.flush()
        text = Path(self.f.name).read_text()
        os.unlink(self.f.name)
        return self.summarize(text)

    @staticmethod
    def summarize(text: str) -> dict:
        """Median SM clock, maximum SM clock, the throttle reasons seen Active and the sample
        count of nvidia-smi CSV rows in FIELDS order (no header, no units)."""
        rows = [r.split(",") for r in text.splitlines() if r.strip()]
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip() == "Active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(rows)}


# ------------------------------------------------------------------ reference arm / CPU baseline

def ref_build() -> tuple[bool, str]:
    """Which build of the reference engine this host times: its -march=native build for the GPU
    hosts' CPU when this CPU has those instructions, else the portable AVX2 build."""
    import oracle
    native = oracle.REF_NATIVE_LIB.exists() and oracle.host_runs_native_build()
    return native, ("-O3 -march=sapphirerapids (the reference's -march=native on this host's "
                    "CPU)" if native else "-O3 -mavx2 -mfma (portable)")


def reference_decode(model_path: str, steps: int, warmup: int, threads: int,
                     with_prefill: bool = False, native: bool = False):
    """The reference engine (oracle/_ref, built from the reference sources) on the host cores:
    prefill of the 16-token prompt, then greedy steps (Qwen3::Generate's loops with
    `--benchmark` semantics), timed with its steady_clock marks. Returns (tok/s, decode s), plus
    its prefill tok/s when with_prefill."""
    import oracle
    m = oracle.RefModel(model_path, CTX, native=native)
    p = prompt_ids()
    if warmup:
        m.generate_ids(p, min(warmup, RUN_STEPS))
    done, secs, pre_secs, pre_tokens = 0, 0.0, 0.0, 0
    while done < steps:
        n = min(RUN_STEPS, steps - done)
        _, ps, ds = m.generate_ids(p, n)
        secs += ds
        pre_secs += ps
        pre_tokens += len(p)
        done += n
    if with_prefill:
        return steps / secs, secs, pre_tokens / pre_secs
    return steps / secs, secs


def reference_positions(m, positions) -> float:
    """Mean seconds of one Qwen3::ForwardToken call of the reference engine at each of the given
    positions (one call each after a warm-up call). The reference prefills and decodes one
    ForwardToken per token; a call's cost depends on its position (attention over kv_len =
    pos + 1 cached rows, src/inference.cpp:1017-1058) and not on what the cache holds, so calls
    at positions spread over a workload sample its per-token cost without replaying the tokens
    before them."""
    m.forward(1, int(positions[0]))
    t0 = time.perf_counter()
    for i, pos in enumerate(positions):
        m.forward((7919 * i) % VOCAB, int(pos))
    return (time.perf_counter() - t0) / len(positions)


def cpu_baselines(model_path: str, threads: int) -> dict:
    """The reference engine on the host cores for the long-prompt, batched and tensor-parallel
    configurations, each on a bounded sample (about a second of CPU work or less each)."""
    import oracle
    native, build = ref_build()
    # One engine at the largest context serves every sample (below the context the positions'
    # costs do not depend on it).
    m = oracle.RefModel(model_path, TP_CTX, native=native)
    out = {}
    pre_pos = [int((i + 0.5) * PREFILL_LEN / 16) for i in range(16)]
    s = reference_positions(m, pre_pos)
    out["prefill"] = {"value": round(1.0 / s, 3), "unit": "tok/s", "cores": threads,
                      "kind": "reference", "build": build,
                      "sample": "16 ForwardToken calls at positions spread uniformly over the "
                                f"{PREFILL_LEN}-token prompt (positions {pre_pos[0]}..{pre_pos[-1]}); "
                                "the reference prefills one token per call"}
    lens, _ = dp_workload(DP_SEQS)
    pick = list(range(0, DP_SEQS, 8))
    dp_pos = [int(lens[i]) + DP_WARMUP + DP_STEPS // 2 for i in pick]
    s = reference_positions(m, dp_pos)
    out["dp_decode"] = {"value": round(1.0 / s, 3), "unit": "tok/s", "cores": threads,
                        "kind": "reference", "build": build,
                        "sample": f"ForwardToken of sequences {pick[0]}, {pick[1]}, ..., "
                                  f"{pick[-1]} of the 64 at the middle of their 128 decode steps "
                                  "(the reference serves one sequence at a time)"}
    tp_pos = [TP_PROMPT + TP_WARMUP + TP_STEPS // 2 + k for k in range(3)]
    s = reference_positions(m, tp_pos)
    out["tp_decode"] = {"value": round(1.0 / s, 3), "unit": "tok/s", "cores": threads,
                        "kind": "reference", "build": build,
                        "sample": f"3 ForwardToken calls at positions {tp_pos[0]}..{tp_pos[-1]}, "
                                  "the middle of the 128 decode steps"}
    return out


def run_reference_arm(args):
    world, rank, _ = dist_info()
    if rank != 0:
        return
    import gen_weights
    threads = os.cpu_count() or 1
    path = gen_weights.cached_model(0)
    native, build = ref_build()
    tps, secs = reference_decode(str(path), args.steps, args.warmup, threads, native=native)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tps, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 * secs / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "Qwen3-0.6B B=1 greedy decode, ctx 512, 16-token prompt, "
                               "64-step runs (reference CPU engine)",
                   "threads": threads, "build": build},
        "cpu_baseline": {"value": round(tps, 3), "unit": UNIT, "cores": threads,
                         "kind": "reference", "build": build,
                         "sample": f"{args.steps} greedy decode steps in runs of {RUN_STEPS} after "
                                   f"a {PROMPT_LEN}-token prefill, OMP_NUM_THREADS={threads}"},
        "e2e": {"value": round(tps, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ B200 arm

def time_lm_head_gemv(torch, q3, iters=20):
    """Average duration of the tied lm_head GEMV kernel (151936 x 1024 bf16 weights, fp32 in/out)
    with CUDA events on the launching stream."""
    w = torch.randn(VOCAB, 1024, device="cuda").to(torch.bfloat16)
    x = torch.randn(1024, device="cuda")
    out = torch.empty(VOCAB, device="cuda")
    s = torch.cuda.current_stream()
    for _ in range(3):
        q3.matmul(out.data_ptr(), x.data_ptr(), w.data_ptr(), VOCAB, 1024, s.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        q3.matmul(out.data_ptr(), x.data_ptr(), w.data_ptr(), VOCAB, 1024, s.cuda_stream)
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters / 1e3


def run_b200_arm(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    from torch.cuda import nvtx

    import gen_weights
    import q3b200

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    path = gen_weights.cached_model(0)
    if world > 1:
        dist.barrier()
    legs = set(args.legs.split(","))
    unknown = legs - {"decode", "prefill", "dp", "tp"}
    if unknown:
        raise SystemExit(f"unknown --legs entries: {sorted(unknown)}")
    total_ms = e2e_tps = 0.0
    kv_pos_sum = 0
    fused = False
    clk = None
    if "decode" in legs:
        model = q3b200.Qwen3(path, CTX, device=local)
        if args.path != "auto":
            model.decode_path = model.PATH_FUSED if args.path == "fused" else model.PATH_LAYERWISE
        ext = torch.cuda.ExternalStream(model.stream)
        p = prompt_ids()

        # Warm-up: W decode steps after a prefill.
        _, nxt = model.prefill(p, 0, want_logits=False)
        model.decode_greedy(nxt, PROMPT_LEN, max(args.warmup, 3))
        torch.cuda.synchronize()

        clocks = Clocks(local)
        total_ms = 0.0
        done = 0
        kv_pos_sum = 0
        while done < args.steps:
            n = min(RUN_STEPS, args.steps - done)
            _, nxt = model.prefill(p, 0, want_logits=False)   # untimed
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(ext)
            nvtx.range_push("q3.decode")  # NVTX ranges name each leg's timed work for ncu filters
            model.decode_greedy(nxt, PROMPT_LEN, n)
            nvtx.range_pop()
            e1.record(ext)
            torch.cuda.synchronize()
            total_ms += e0.elapsed_time(e1)
            kv_pos_sum += sum(PROMPT_LEN + i + 1 for i in range(n))
            done += n
        total_ms = max_over_ranks(total_ms, world)
        clk = clocks.stop()

        # End to end through the public API with host buffers: ForwardToken + Sampler::Greedy
        # per step (q3_forward_token_greedy: token and position in; the 151936 fp32 logits and
        # their greedy token out to host) - the two calls of each step of Qwen3::Generate.
        model.reset()
        _, nxt = model.prefill(p, 0, want_logits=False)
        e2e_steps = min(args.steps, RUN_STEPS)
        tok = nxt
        for i in range(3):  # warm-up calls (positions rewritten below)
            model.forward_token_greedy(tok, PROMPT_LEN + i)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            lg, tok = model.forward_token_greedy(tok, PROMPT_LEN + i)
        e2e_s = time.perf_counter() - t0
        e2e_tps = world * e2e_steps / e2e_s

        fused = model.decode_path == model.PATH_FUSED
        model.close()

    # Prefill of the long prompt through q3_prefill (ids in from host, next token out), timed with
    # CUDA events on the model's stream; the max over ranks.
    pm = q3b200.Qwen3(path, PREFILL_CTX, device=local)
    p_ms = 0.0
    batched = False
    if "prefill" in legs:
        pext = torch.cuda.ExternalStream(pm.stream)
        pp = np.random.default_rng(2).integers(0, VOCAB, PREFILL_LEN).astype(np.int32)
        for _ in range(2):
            pm.prefill(pp, 0, want_logits=False)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        p_ms = 0.0
        for _ in range(PREFILL_RUNS):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(pext)
            nvtx.range_push("q3.prefill")
            pm.prefill(pp, 0, want_logits=False)
            nvtx.range_pop()
            e1.record(pext)
            torch.cuda.synchronize()
            p_ms += e0.elapsed_time(e1)
        p_ms /= PREFILL_RUNS
        p_ms = max_over_ranks(p_ms, world)
        batched = pm.prefill_path == pm.PREFILL_BATCHED

    # Data-parallel batched decode: this rank's share of the 64 sequences in one batch.
    dp_ms = dp_gbs = dp_bytes_step = 0.0
    dp_prefill_ms, dp_prefill_tokens = 0.0, 0
    mine = []
    if "dp" in legs:
        lens, prompts = dp_workload(args.dp_seqs)
        mine = dp_share(args.dp_seqs, rank, world)
        batch = q3b200.Batch(pm, len(mine), int(max(lens[i] for i in mine)) + DP_WARMUP + DP_STEPS)
        bext = torch.cuda.ExternalStream(batch.stream)
        # This rank's prompts go in together (one varlen tensor-core pass per 4096-token chunk),
        # timed on the batch's stream.
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(bext)
        nvtx.range_push("q3.dp_prefill")
        batch.add_many([prompts[i] for i in mine])
        nvtx.range_pop()
        e1.record(bext)
        torch.cuda.synchronize()
        dp_prefill_ms = max_over_ranks(e0.elapsed_time(e1), world)
        dp_prefill_tokens = int(sum(int(lens[i]) for i in range(args.dp_seqs)))
        batch.decode(DP_WARMUP)  # warm-up (graph capture); positions advance by DP_WARMUP
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(bext)
        nvtx.range_push("q3.dp_decode")
        batch.decode(DP_STEPS)
        nvtx.range_pop()
        e1.record(bext)
        torch.cuda.synchronize()
        dp_ms = e0.elapsed_time(e1)
        dp_ms = max_over_ranks(dp_ms, world)
        # Bytes per step on this rank: the weights once + every sequence's KV rows at its length.
        kv_tokens = sum(int(lens[i]) + DP_WARMUP + DP_STEPS / 2 for i in mine)
        dp_bytes_step = WEIGHT_BYTES + KV_BYTES_PER_POS * kv_tokens
        dp_gbs = dp_bytes_step * DP_STEPS / (dp_ms / 1e3) / 1e9
        batch.close()

    pm.close()

    # Tensor-parallel decode of one long-context stream over all ranks: the default path (the
    # fused persistent kernel with its in-kernel exchange) timed first, then two comparison arms
    # continuing the same stream: the per-step graph with this library's all-reduce kernels, and
    # the same graph with NCCL's all-reduce / all-gather captured in their place.
    tp_ms = tp_gbs = tp_bytes_gpu = 0.0
    tp_arms = {}
    tp_default = None
    tp_failed = {}
    if "tp" in legs:
        tm = q3b200.Qwen3(path, TP_CTX, device=local)
        tprompt = np.random.default_rng(4).integers(0, VOCAB, TP_PROMPT).astype(np.int32)
        _, tnext = tm.prefill(tprompt, 0, want_logits=False)
        tp = q3b200.TpDecoder(tm, rank, world)
        tp.connect(gather_handles(tp.ipc_handle(), world))
        tpx = torch.cuda.ExternalStream(tp.stream)
        uid = [q3b200.TpDecoder.nccl_unique_id() if rank == 0 else None]
        if world > 1:
            dist.broadcast_object_list(uid, src=0)
        tp.nccl_connect(uid[0])
        pos, tok = TP_PROMPT, tnext
        names = {q3b200.TpDecoder.FUSED: "fused", q3b200.TpDecoder.GRAPH: "graph",
                 q3b200.TpDecoder.GRAPH_NCCL: "graph_nccl"}
        arms = [tp.path] + [a for a in (q3b200.TpDecoder.GRAPH, q3b200.TpDecoder.GRAPH_NCCL)
                            if a != tp.path]
        for arm in arms:
            # A decode that raises (a bounded wait gave up) leaves the arm out of the line; every
            # rank still takes the same collective steps, agrees on the outcome and resets.
            ok, why, out = True, "", None
            tp.path = arm
            try:
                warm = tp.decode(tok, pos, TP_WARMUP)
            except q3b200.Q3Error as e:
                ok, why = False, str(e)
            pos += TP_WARMUP
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(tpx)
            nvtx.range_push("q3.tp_" + names[arm])
            if ok:
                try:
                    out = tp.decode(int(warm[-1]), pos, TP_STEPS)
                except q3b200.Q3Error as e:
                    ok, why = False, str(e)
            nvtx.range_pop()
            e1.record(tpx)
            torch.cuda.synchronize()
            pos += TP_STEPS
            ms = max_over_ranks(e0.elapsed_time(e1), world)
            if max_over_ranks(0.0 if ok else 1.0, world) > 0:
                tp_failed[names[arm]] = why or "failed on another rank"
                tp.reset()
                if world > 1:
                    dist.barrier()
                continue
            tok = int(out[-1])
            tp_arms[names[arm]] = ms
        tp_default = next((names[a] for a in arms if names[a] in tp_arms), None)
        tp_ms = tp_arms.get(tp_default, float("inf"))
        tp_kv = TP_PROMPT + TP_WARMUP + TP_STEPS / 2
        tp_bytes_gpu = (WEIGHT_BYTES + KV_BYTES_PER_POS * tp_kv) / world
        tp_gbs = tp_bytes_gpu * TP_STEPS / (tp_ms / 1e3) / 1e9
        tp.close()
        tm.close()

    pk = peaks()
    dec = "decode" in legs
    value = world * args.steps / (total_ms / 1e3) if dec else 0.0
    avg_kv = kv_pos_sum / args.steps
    step_bytes = WEIGHT_BYTES + KV_BYTES_PER_POS * avg_kv
    per_gpu_tps = args.steps / (total_ms / 1e3) if dec else 0.0
    if not dec:
        achieved, kernel, launches = 0.0, None, 0
    elif fused:
        # The whole decode step is one kernel: algorithmic bytes per step (weights + the KV rows
        # read at the step's kv_len) over its event-timed duration.
        achieved = step_bytes * per_gpu_tps / 1e9
        kernel = "decode_fused_kernel (whole decode step)"
        launches = sum(1 for _ in range(0, args.steps, RUN_STEPS))
    else:
        lm_s = time_lm_head_gemv(torch, q3b200)
        lm_bytes = LM_HEAD_BYTES + 1024 * 4 + VOCAB * 4
        achieved = lm_bytes / lm_s / 1e9
        kernel = "gemv lm_head (151936x1024 bf16)"
        launches = args.steps * (7 * 28 + 3)

    cpu = None
    cpu_prefill = None
    cpu_legs = {}
    if rank == 0 and world == 1 and q3_ref_available():
        threads = os.cpu_count() or 1
        native, build = ref_build()
        if dec:
            tps, _ = reference_decode(str(path), RUN_STEPS, 0, threads, native=native)
            cpu = {"value": round(tps, 3), "unit": UNIT, "cores": threads, "kind": "reference",
                   "build": build,
                   "sample": f"{RUN_STEPS} greedy decode steps after a {PROMPT_LEN}-token "
                             f"prefill, ctx {CTX}, OMP_NUM_THREADS={threads}"}
        if legs & {"prefill", "dp", "tp"}:
            cpu_legs = cpu_baselines(str(path), threads)
        cpu_prefill = cpu_legs.get("prefill")
    p_tps = world * PREFILL_LEN / (p_ms / 1e3) if p_ms else 0.0
    p_tflops = prefill_flops(PREFILL_LEN) / (p_ms / 1e3) / 1e12 if p_ms else 0.0

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights and prompt IDs)",
            "config": {"workload": "Qwen3-0.6B B=1 greedy decode, ctx 512, 16-token prompt, "
                                   "runs of 64 decode steps (one step = one token)",
                       "model": "Qwen3-0.6B", "global_batch": world, "seq_len": CTX,
                       "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2 (1.19 GB of weights streamed per step)"},
            "gpu_launches": launches,
            "decode_path": "fused" if fused else "layerwise",
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1),
                         "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / pk["hbm_gbs"], 4),
                         "traffic": FUSED_TRAFFIC_PER_STEP if fused else None,
                         "traffic_unit": "bytes per decode step (ncu)" if fused else None,
                         "kernel": kernel, "peak_source": pk["source"]},
            "decode_step_roofline": {
                "bytes_per_step": int(step_bytes),
                "achieved_gbs": round(step_bytes * per_gpu_tps / 1e9, 1),
                "frac": round(step_bytes * per_gpu_tps / 1e9 / pk["hbm_gbs"], 4)},
            "e2e": {"value": round(e2e_tps, 2), "unit": UNIT, "h2d_bytes_per_step": 32,
                    "d2h_bytes_per_step": VOCAB * 4 + 8,
                    "api": "q3_forward_token_greedy per step: ForwardToken + Sampler::Greedy "
                           "(logits into the model's pinned buffer, the reference's "
                           "const-reference return, and their greedy token)"},
            "cpu_baseline": cpu,
            "clocks": clk,
            "dp_decode": {
                "metric": "batched greedy decode tok/s (64 sequences, ctx U[128,4096], "
                          "Qwen3-0.6B bf16)",
                "value": round(args.dp_seqs * DP_STEPS / max(dp_ms / 1e3, 1e-12), 1), "unit": "tok/s",
                "sequences": args.dp_seqs,
                "steps": DP_STEPS, "ms_per_step": round(dp_ms / DP_STEPS, 4),
                "seqs_per_gpu": len(mine), "scaling": "strong",
                "cpu_baseline": cpu_legs.get("dp_decode"),
                "prefill": {"value": round(dp_prefill_tokens / max(dp_prefill_ms / 1e3, 1e-12), 1),
                            "unit": "tok/s", "ms": round(dp_prefill_ms, 3),
                            "tokens": dp_prefill_tokens,
                            "api": "q3_batch_add_many (each rank's prompts prefilled together)"},
                "roofline": {"bound": "hbm", "achieved": round(dp_gbs, 1),
                             "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": round(dp_gbs / pk["hbm_gbs"], 4),
                             "bytes_per_step_per_gpu": int(dp_bytes_step)},
            },
            "tp_decode": {
                "metric": "tensor-parallel greedy decode tok/s (B=1, ctx 32768, 32000-token "
                          "prompt, Qwen3-0.6B bf16)",
                "value": round(TP_STEPS / max(tp_ms / 1e3, 1e-12), 1), "unit": "tok/s",
                "steps": TP_STEPS, "ms_per_step": round(tp_ms / TP_STEPS, 4),
                "parallelism": f"tp{world}", "scaling": "strong",
                "cpu_baseline": cpu_legs.get("tp_decode"),
                "path": tp_default,
                "collective": ("in-kernel exchange of tagged words over NVLink peer memory (CUDA "
                               "IPC handles) from the fused decode kernel's phases, not NCCL"
                               if tp_default == "fused" else
                               "this library's own one-shot all-reduce kernel over NVLink peer "
                               "memory (CUDA IPC handles), not NCCL"),
                "failed_arms": tp_failed or None,
                "arms": {name: {"ms_per_step": round(ms / TP_STEPS, 4),
                                "value": round(TP_STEPS / (ms / 1e3), 1),
                                "collective": TP_ARM_COLLECTIVE[name]}
                         for name, ms in tp_arms.items()},
                "roofline": {"bound": "hbm", "achieved": round(tp_gbs, 1),
                             "peak": pk["hbm_gbs"], "unit": "GB/s per GPU",
                             "frac": round(tp_gbs / pk["hbm_gbs"], 4),
                             "bytes_per_step_per_gpu": int(tp_bytes_gpu)},
            },
            "prefill": {
                "metric": "prefill tok/s (2048-token prompt, ctx 4096, Qwen3-0.6B bf16)",
                "value": round(p_tps, 1), "unit": "tok/s", "ms_per_prefill": round(p_ms, 4),
                "runs": PREFILL_RUNS, "path": "batched tcgen05" if batched else "token by token",
                "api": "q3_prefill (ids in from host, next token out)",
                "roofline": {"bound": "tensor", "achieved": round(p_tflops, 1),
                             "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": round(p_tflops / pk["bf16_tflops"], 4),
                             "flops_per_prefill": prefill_flops(PREFILL_LEN),
                             "peak_source": pk["source"] + " (burst bf16 GEMM)"},
                "cpu_baseline": cpu_prefill,
            },
        }
        for key, leg in (("dp_decode", "dp"), ("tp_decode", "tp"), ("prefill", "prefill")):
            if leg not in legs:
                del line[key]
        if not dec:
            line["value"] = None
            line["note"] = f"decode leg not run (--legs {args.legs})"
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def q3_ref_available() -> bool:
    return (ROOT / "oracle" / "_ref" / "libq3ref.so").exists()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--path", choices=["auto", "fused", "layerwise"], default="auto",
                    help="decode path of the b200 arm (auto: fused when the shape allows)")
    ap.add_argument("--dp-seqs", type=int, default=DP_SEQS,
                    help="sequences of the batched-decode leg (the first n of the 64; a smaller "
                         "case for a profiler run)")
    ap.add_argument("--legs", default="decode,prefill,dp,tp",
                    help="comma-separated legs of the b200 arm to run (decode: the headline "
                         "B=1 decode; prefill; dp: batched decode; tp: tensor-parallel decode); "
                         "a profiler run can select one")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
        if not q3_ref_available():
            print(json.dumps({"impl": "reference",
                              "unavailable": "oracle/_ref/libq3ref.so was not built"}))
            return
        run_reference_arm(args)
    else:
        run_b200_arm(args)


if __name__ == "__main__":
    main()
