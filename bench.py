"""Decode throughput of the B200 MoE decode path (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Workload (configs[3] of BASELINE.json): Mixtral-8x7B-shape model, random
N(0, 0.02) weights from the seeded generator (seed 4) quantized Q4_K (experts)
and Q6_K (attention, embedding, output), F32 router and norms, f16 paged KV.
A 512-token random prompt is fed one position per step, then W untimed and K
timed greedy decode steps at batch B (default 1).  One step = one decode token
for each of the B sequences.  Every step streams ~7.6 GB of weights, far more
than the 126 MB L2, so no flush is needed between steps.

value : decode tok/s with everything resident in HBM, CUDA events on the
        engine's stream around K device-side greedy steps (max over ranks).
e2e   : the same metric through the C-ABI call a host uses (sfk_forward with
        a host token in and host logits + argmax out every step, synchronized;
        W untimed warm-up steps, then up to 128 timed ones).
roofline : the dominant kernel (routed gate/up over the Q4_K experts), its
        algorithmic bytes per launch over its CUDA-event launch duration.
cpu_baseline : the CPU oracle (a C restatement of the reference's ggml CPU
        decode, all host threads) on a bounded sample of the same workload.

--impl reference times that CPU implementation alone (the reference engine
itself needs the un-vendored ggml submodule and cannot be built here).
With --gpus N > 1 (torchrun, one rank per GPU) every rank decodes its own
replica of the model (the Mixtral shape fits one GPU): weak scaling.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "decode tok/s, Mixtral-8x7B-shape Q4_K b=1; mul_mat_id achieved HBM GB/s"
PROMPT = 512
SEED = 4


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed loop runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.15)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_sample(threads: int, n_tokens: int = 4, warm: int = 1, ctx: int = PROMPT):
    """Time the CPU oracle (the ggml CPU decode restated in C) on 2 of the 32
    Mixtral-shape layers plus embedding and lm_head, decoding at a context of
    `ctx` positions (the KV cache is filled as if the bench's prompt had been
    fed); per-token time = head + 16 x (2-layer time)."""
    from oracle import oracle as O
    O.set_threads(threads)
    cfg = O.ModelConfig(n_embd=4096, n_head=32, n_head_kv=8, n_layer=2, n_ff=14336, n_expert=8, n_expert_used=2,
                        n_vocab=32000, n_ctx=ctx + warm + n_tokens + 1, freq_base=1e6, type_embd=O.Q6_K,
                        type_attn=O.Q6_K, type_ffn_gu=O.Q4_K, type_ffn_down=O.Q4_K, type_output=O.Q6_K, kv_f16=True)
    m = O.Model(cfg, seed=SEED)
    s = m.new_seq()
    s.fill_kv(ctx, seed=SEED)
    rng = np.random.default_rng(SEED)
    tok = int(rng.integers(0, cfg.n_vocab))
    for p in range(ctx, ctx + warm):
        tok, _ = s.forward(tok, p)
    l0, h0 = s.timing()
    for p in range(ctx + warm, ctx + warm + n_tokens):
        tok, _ = s.forward(tok, p)
    l1, h1 = s.timing()
    per_tok = (h1 - h0) / n_tokens + 16.0 * (l1 - l0) / n_tokens
    return {"value": 1.0 / per_tok, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"CPU oracle (C restatement of the ggml CPU decode, {threads} thread(s)): {n_tokens} decode "
                      f"tokens at context {ctx} through 2 of 32 Mixtral-shape layers plus embedding and lm_head; "
                      f"per-token time = head + 16 x two-layer time = {per_tok:.3f} s"}


def cpu_baseline_both(n_tokens: int = 3):
    """The reference engine's own setting (one compute thread,
    src/model/engine/engine.cpp:1018) as the value, all host threads beside it."""
    one = cpu_sample(1, n_tokens=n_tokens, warm=1)
    nproc = os.cpu_count() or 1
    alln = cpu_sample(nproc, n_tokens=n_tokens, warm=1)
    out = dict(one)
    out["value_all_threads"] = alln["value"]
    out["cores_all_threads"] = nproc
    out["sample"] = one["sample"] + f"; at {nproc} threads: {alln['value']:.3f} tok/s"
    return out


def run_reference(args, rank: int):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    # each step: one decode token of the bounded CPU sample at the bench's
    # prompt context; at most 8 steps (the GPU arm times K steps of the whole
    # 32-layer model; here each step runs 2 layers and is scaled to 32, so a
    # K of hundreds would not end within minutes)
    steps_done = max(1, min(args.steps, 8))
    res = cpu_sample(threads, n_tokens=steps_done, warm=min(args.warmup, 2))
    value = float(res["value"])
    res["sample"] += (f"; {steps_done} of the requested {args.steps} steps (CPU time bound)"
                      if steps_done != args.steps else "")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": steps_done, "warmup": min(args.warmup, 2), "ms_per_step": 1000.0 / value,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q4_k/q6_k x q8_k int8 dot",
            "data": "synthetic",
            "config": {"workload": "Mixtral-8x7B-shape decode b=1 (bounded CPU sample)", "model": "mixtral-8x7b-shape",
                       "global_batch": 1, "seq_len": PROMPT, "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": res["sample"]},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t0}
    print(json.dumps(line), flush=True)


def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))

    B = args.batch
    PROMPT = args.prompt
    e2e_steps = 0 if args.no_e2e else min(args.steps, 128)
    e2e_warm = 0 if args.no_e2e else args.warmup
    n_ctx = PROMPT + args.warmup + args.steps + e2e_warm + e2e_steps + 16
    cfg = E.mixtral_config(n_ctx=n_ctx, max_batch=B, n_layer=args.layers)
    t_load = time.perf_counter()
    eng = E.Engine.load(cfg, seed=SEED, device=local_rank)
    t_load = time.perf_counter() - t_load
    stream = torch.cuda.ExternalStream(eng.stream, device=torch.device("cuda", local_rank))

    rng = np.random.default_rng(SEED + rank)
    prompt = rng.integers(0, cfg.n_vocab, (B, PROMPT)).astype(np.int32)
    # batched prefill (sfk_prefill), one call per sequence; one untimed call
    # first (it allocates the prefill buffers), then the KV is cleared
    eng.prefill(prompt[0], seq=0, want_logits=False)
    eng.reset_kv()
    torch.cuda.synchronize()
    t_pf = time.perf_counter()
    for s_ in range(B):
        eng.prefill(prompt[s_], seq=s_, want_logits=False)
    t_pf = time.perf_counter() - t_pf
    eng.decode_greedy(args.warmup, B, want_tokens=False)

    # --- device-timed greedy decode ---------------------------------------
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        ev0.record(stream)
        eng.decode_greedy(args.steps, B, want_tokens=False)
        ev1.record(stream)
        ev1.synchronize()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    value = world * B * args.steps / (ms / 1000.0)

    # --- end to end through the C ABI with host buffers ----------------------
    pos0 = PROMPT + args.warmup + args.steps
    tok = prompt[:, 0].copy()
    for i in range(e2e_warm):   # untimed warm-up of the host-buffer path
        tok, _ = eng.forward_batch(tok, np.full(B, pos0 + i, np.int32), want_logits=True)
    pos0 += e2e_warm
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        am, logits = eng.forward_batch(tok, np.full(B, pos0 + i, np.int32), want_logits=True)
        tok = am
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * B * e2e_steps / e2e_s if e2e_steps else None

    # --- dominant kernel: routed gate/up (CUDA events per launch class) -------
    st = eng.stats()
    if args.no_kernel_times:
        if rank == 0:
            print(json.dumps({"value": value, "ms_per_step": ms / args.steps, "steps": args.steps}), flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        eng.close()
        return
    kt = eng.time_kernels(B, iters=64)
    peak, peak_kind = _peaks()
    gu_row = 4096 // 256 * 144
    # distinct experts a step streams per layer: 2 at b=1; for b tokens the
    # expectation of a uniform top-2 draw over 8 experts, 8 (1 - 0.75^b)
    uniq = 2.0 if B == 1 else 8.0 * (1.0 - 0.75 ** B)
    # routed expert rows of gate and up; the routing prologue (F32 router
    # weights + the token's hidden state) rides along in the same kernel
    gu_bytes = uniq * 2 * 14336 * gu_row + (8 * 4096 * 4 + B * 4096 * 4 if kt["router"] == 0.0 else 0)
    gu_ms = kt["gate_up"]
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9
    kv_bytes_tok = 32 * 2 * 8 * 128 * 2 * (PROMPT + args.warmup + args.steps // 2)
    # one step streams the trunk once and each distinct expert once
    expert_bytes_tok = 32 * 2 * 3 * 14336 * gu_row   # two experts per layer, gate + up + down (Q4_K)
    trunk_bytes = st["active_bytes_per_token"] - expert_bytes_tok
    step_bytes = trunk_bytes + expert_bytes_tok * uniq / 2.0 + kv_bytes_tok * B
    step_gbs = step_bytes * args.steps / (ms / 1000.0) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        eng.close()
        cpu = cpu_baseline_both()
    # at 4 or more GPUs the same job also runs configs[4] (the ~1T model,
    # expert-parallel over these ranks) and nests its line
    ep_line = None
    if world >= 4 and not args.no_ep:
        eng.close()
        ep_line = ep_measure(1, 256, 61, 64, 3, rank, world, local_rank, dist)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_k/q6_k weights x q8_k int8 dot (dp4a), fp32 accum", "data": "synthetic",
            "config": {"workload": f"Mixtral-8x7B-shape decode b={B}: {PROMPT}-token random prompt, then greedy decode",
                       "model": "mixtral-8x7b-shape (32L d4096 32q/8kv E8 top2 F14336 V32000)",
                       "global_batch": B * world, "seq_len": PROMPT, "parallelism": f"replicas x{world}",
                       "kv": "f16 paged (16-token pages, permuted pool)",
                       "l2": "no flush: 7.6 GB of weights streamed per step >> 126 MB L2"},
            "clocks": clk.summary(),
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8 * B,
                    "d2h_bytes_per_step": 4 * B * cfg.n_vocab + 8 * B + 4},
            "gpu_launches": st["kernels_per_step"] * args.steps,
            "roofline": {"bound": "hbm", "kernel": "stream2_kernel<Q4_K,2>: routing + routed gate/up (mul_mat_id) + SwiGLU",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": GU_TRAFFIC_BYTES,
                         "bytes_per_launch": gu_bytes, "launch_ms": gu_ms},
            "step_roofline": {"achieved": step_gbs, "peak": peak, "unit": "GB/s", "frac": step_gbs / peak,
                              "bytes_per_token": step_bytes / B},
            "kernel_ms": kt,
            "cpu_baseline": cpu,
            "load_s": t_load, "prefill_s": t_pf, "prefill_tok_s": B * PROMPT / t_pf,
            "prefill": "batched (sfk_prefill: tensor-core GEMMs, one call per sequence)",
        }
        if ep_line is not None:
            line["ep_1t"] = ep_line
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if cpu is None:
        eng.close()


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# the routed gate/up kernel at this shape, from an `ncu --set full` capture of
# the same kernel (2-layer model, identical launch shape): 132.40 MB read +
# 4.69 MB written.
GU_TRAFFIC_BYTES = 137.09e6


def ep_rank_bytes(cfg, world: int, B: int) -> tuple[float, bool]:
    """Bytes one rank streams per step of the expert-parallel decode (Q8_0
    trunk, Q4_K experts, the config's head width) and whether the attention heads are
    split over the ranks.  The heads split, as the engine decides at
    creation, when both head counts divide by the ranks and a rank's query
    columns are whole 256-column blocks (SFK_HEAD_PARALLEL=0 keeps them
    replicated); the router (F32) and the norms stay replicated, the device
    greedy loop scores each rank's slice of the vocabulary (SFK_VOCAB_SHARD=0
    keeps the lm_head whole), and each rank streams its share of the expected
    routed experts."""
    d, F, k = cfg.n_embd, cfg.n_ff, cfg.n_expert_used
    hd = cfg.head_dim if cfg.head_dim > 0 else cfg.n_embd // cfg.n_head   # as sfk_engine_create decides it
    q8 = lambda K: K // 32 * 34   # noqa: E731
    q4 = lambda K: K // 256 * 144   # noqa: E731
    split = (world > 1 and cfg.n_head % world == 0 and cfg.n_head_kv % world == 0 and
             (cfg.n_head // world * hd) % 256 == 0 and os.environ.get("SFK_HEAD_PARALLEL", "1") != "0")
    share = world if split else 1
    attn = ((cfg.n_head + 2 * cfg.n_head_kv) * hd * q8(d) + d * q8(cfg.n_head * hd)) / share
    vshare = world if world > 1 and os.environ.get("SFK_VOCAB_SHARD", "1") != "0" else 1
    trunk = cfg.n_layer * (attn + 4 * d * cfg.n_expert) + -(-cfg.n_vocab // vshare) * q8(d)
    experts_rank = cfg.n_layer * B * k / world * (2 * F * q4(d) + d * q4(F))   # expected routed bytes per rank
    return trunk + experts_rank, split


EP_METRIC = "decode tok/s, ~1T-parameter MoE (61L d7168 E384 top-8) Q4_K experts, expert-parallel"


def run_ep(args, rank: int, world: int, local_rank: int):
    """the ~1T-parameter MoE, experts sharded over the torchrun
    ranks (expert parallelism), trunk replicated; one sequence decoded by the
    whole job."""
    import datetime
    import torch

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    line = ep_measure(args.batch, args.prompt, args.layers, args.steps, args.warmup, rank, world, local_rank, dist)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def ep_measure(B: int, prompt_n: int, n_layer: int, steps: int, warmup: int, rank: int, world: int,
               local_rank: int, dist) -> dict | None:
    """Load the ~1T model sharded over the job's ranks, feed a random prompt,
    time `steps` greedy decode steps (max over ranks) and return rank 0's
    JSON line (other ranks: None).  Every rank takes the same collective
    steps, also when the model does not fit."""
    import torch
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L

    metric = EP_METRIC
    cfg = E.trillion_config(n_ctx=prompt_n + warmup + steps + 16, max_batch=B, n_layer=n_layer,
                            ep_size=world, ep_rank=rank)
    t_load = time.perf_counter()
    try:
        eng = E.Engine.load(cfg, seed=5, device=local_rank)
        ok = 1
    except L.SfkError as ex:
        eng, ok, why = None, 0, str(ex)
    if dist:
        t = torch.tensor([ok], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok = int(t.item())
    if not ok:
        if eng is not None:
            eng.close()
        return {"metric": metric, "n_gpus": world, "unavailable":
                f"the model does not fit: {world} GPU(s) -> {why if eng is None else 'another rank'}"} \
            if rank == 0 else None
    t_load = time.perf_counter() - t_load
    if world > 1:
        eng.ep_connect_group()
    stream = torch.cuda.ExternalStream(eng.stream, device=torch.device("cuda", local_rank))
    rng = np.random.default_rng(5)   # the same prompt on every rank
    prompt = rng.integers(0, cfg.n_vocab, (B, prompt_n)).astype(np.int32)
    t_pf = time.perf_counter()
    for p in range(prompt_n):
        eng.forward_batch(prompt[:, p], np.full(B, p, np.int32), want_logits=False)
    t_pf = time.perf_counter() - t_pf
    eng.decode_greedy(warmup, B, want_tokens=False)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        ev0.record(stream)
        toks = eng.decode_greedy(steps, B, want_tokens=True)
        ev1.record(stream)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    same = 1
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        # every rank must have decoded the same tokens
        tt = torch.from_numpy(toks.astype(np.int64)).cuda()
        t0 = tt.clone()
        dist.broadcast(t0, 0)
        s_ = torch.tensor([int(torch.equal(tt, t0))], device="cuda")
        dist.all_reduce(s_, op=dist.ReduceOp.MIN)
        same = int(s_.item())
    value = B * steps / (ms / 1000.0)
    # the collective the step's peer-memory exchanges stand in for: an NCCL
    # all-reduce (sum) of the same [b, d] f32 partial, timed alone on this
    # job's process group (max over ranks), against the step's
    # 2 x n_layer exchanges
    nccl_us = None
    if dist:
        buf = torch.zeros((B, cfg.n_embd), dtype=torch.float32, device="cuda")
        for _ in range(20):
            dist.all_reduce(buf)
        torch.cuda.synchronize()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        n_ar = 200
        a0.record()
        for _ in range(n_ar):
            dist.all_reduce(buf)
        a1.record()
        a1.synchronize()
        t = torch.tensor([a0.elapsed_time(a1) * 1000.0 / n_ar], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        nccl_us = float(t.item())
    st = eng.stats()
    peak, peak_kind = _peaks()
    rank_bytes, heads_split = ep_rank_bytes(cfg, world, B)
    line = None
    if rank == 0:
        line = {
            "metric": metric, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "q4_k experts / q8_0 trunk x int8 dot (dp4a), fp32 accum",
            "data": "synthetic",
            "config": {"workload": f"~1T-param MoE decode b={B}: {prompt_n}-token random prompt, then greedy decode",
                       "model": "61L d7168 64q/8kv E384 top8 F2048 V160000", "global_batch": B,
                       "seq_len": prompt_n,
                       "parallelism": f"ep{world} (experts sharded, "
                                      f"{'attention heads split' if heads_split else 'trunk replicated'})"},
            "clocks": clk.summary(), "ranks_agree": bool(same),
            "gpu_launches": st["kernels_per_step"] * steps,
            "step_roofline": {"achieved": rank_bytes * steps / (ms / 1000.0) / 1e9, "peak": peak,
                              "unit": "GB/s per GPU", "frac": rank_bytes * steps / (ms / 1000.0) / 1e9 / peak,
                              "bytes_per_token_per_gpu": rank_bytes, "peak_kind": peak_kind},
            "weight_bytes_per_gpu": st["weight_bytes_hbm"], "load_s": t_load, "prefill_s": t_pf,
            "exchanges": {"per_step": 2 * n_layer, "kind": "peer-memory combine kernel (flags + peer loads)",
                          "nccl_allreduce_us": nccl_us,
                          "nccl_allreduce_ms_per_step": None if nccl_us is None else nccl_us * 2 * n_layer / 1e3,
                          "step_ms": ms / steps},
        }
    if dist:
        dist.barrier()
    eng.close()
    return line


def run_sweep(args):
    """configs[1] and configs[2] of BASELINE.json, through the engine's own
    kernels (sfk_time_kernels: CUDA events around 64 back-to-back launches of
    one kernel class, launch gaps included).  Prints one JSON line per case.

    mul_mat_id: Mixtral-shape experts (E=8, gate/up 14336x4096, down
    4096x14336) in Q4_K / Q6_K / Q8_0 at b in {1, 4, 16} tokens (16 is the
    engine's largest step), then b in {16, 64} through the expert-grouped
    tensor-core op (run_sweep_id_tc).  Four layers are resident and the
    launches rotate over them, so every launch streams experts that are not
    in L2.  Bytes = unique routed experts x per-expert matrix bytes; the
    router is a seeded random F32 matrix, so the expected unique count of a
    uniform top-2 draw, 8 (1 - 0.75^b), is used (the last launch's measured
    count is printed beside it).  Steps of one or two tokens route inside the
    gate/up kernel (its time includes the routing, router_us is 0); larger
    steps run the router kernel first (router_us, not in gate/up's time).

    attention: 32q/8kv heads, hd 128, f16 KV in 16-token pages handed out in
    a permuted order, contexts {512, 4096, 32768}, b in {1, 8}; one layer, so
    working sets under 126 MB stay in L2 between the back-to-back launches
    (those cases are latency-bound; their GB/s is not an HBM figure)."""
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L
    peak, peak_kind = _peaks()
    names = {L.TYPE_Q4_K: "Q4_K", L.TYPE_Q6_K: "Q6_K", L.TYPE_Q8_0: "Q8_0"}
    row_bytes = {L.TYPE_Q4_K: lambda K: K // 256 * 144, L.TYPE_Q6_K: lambda K: K // 256 * 210,
                 L.TYPE_Q8_0: lambda K: K // 32 * 34}
    d, F = 4096, 14336
    rng = np.random.default_rng(2)
    for t in (L.TYPE_Q4_K, L.TYPE_Q6_K, L.TYPE_Q8_0):
        cfg = E.mixtral_config(n_layer=4, n_ctx=64, max_batch=16, type_ffn_gu=t, type_ffn_down=t)
        eng = E.Engine.load(cfg, seed=2)
        for b in (1, 4, 16):
            for p in range(2):
                eng.forward_batch(rng.integers(0, cfg.n_vocab, b), np.full(b, p, np.int32), want_logits=False)
            kt = eng.time_kernels(b, iters=64)
            ids, _ = eng.route(b)
            uniq = 8.0 * (1.0 - 0.75 ** b)
            for kern, mb in (("gate_up", 2 * F * row_bytes[t](d)), ("down", d * row_bytes[t](F))):
                byts = uniq * mb
                gbs = byts / (kt[kern] * 1e-3) / 1e9
                print(json.dumps({"sweep": "mul_mat_id", "kernel": kern, "wtype": names[t], "b": b,
                                  "us": kt[kern] * 1e3, "bytes": byts, "GBps": gbs, "frac": gbs / peak,
                                  "router_us": kt["router"] * 1e3,
                                  "peak_kind": peak_kind, "unique_experts_expected": uniq,
                                  "unique_experts_last_launch": int(np.unique(ids).size)}), flush=True)
        eng.close()
    run_sweep_id_tc(peak, peak_kind)
    ctxs = (512, 4096, 32768)
    cfg = E.mixtral_config(n_layer=1, n_ctx=max(ctxs) + 16, max_batch=8)
    eng = E.Engine.load(cfg, seed=3)
    pos = 0
    for ctx in ctxs:
        while pos < ctx:   # fill the KV of all 8 sequences up to position ctx - 1
            eng.forward_batch(rng.integers(0, cfg.n_vocab, 8), np.full(8, pos, np.int32), want_logits=False)
            pos += 1
        for b in (1, 8):
            kt = eng.time_kernels(b, iters=64)
            byts = b * ctx * 8 * 128 * 2 * 2
            gbs = byts / (kt["attention"] * 1e-3) / 1e9
            print(json.dumps({"sweep": "attention", "ctx": ctx, "b": b, "us": kt["attention"] * 1e3, "bytes": byts,
                              "GBps": gbs, "frac": gbs / peak, "peak_kind": peak_kind,
                              "l2_resident": byts < 126e6}), flush=True)
    eng.close()
    run_sweep_attn_hbm(peak, peak_kind)


def run_sweep_attn_hbm(peak, peak_kind):
    """configs[2]'s short contexts with the KV read from HBM: the same
    attention kernel timed by sfk_time_kernels, whose 64 launches rotate over
    the layers, on an engine with enough layers that their KV (layers x b x
    ctx x 8 kv heads x 128 x 2 (K, V) x 2 B) exceeds the 126 MB L2 -- 64
    layers at ctx 512 (134 MB at b = 1), 32 layers at ctx 4096 -- so no launch
    finds its layer's pages in L2.  The FFN is shrunk to 256 columns (the
    attention does not read it) to keep the engine small; each sequence's
    context is filled by sfk_prefill and one batched decode step."""
    from strataflow_b200 import engine as E
    rng = np.random.default_rng(5)
    for ctx, n_layer in ((512, 64), (4096, 32)):
        cfg = E.mixtral_config(n_layer=n_layer, n_ff=256, n_ctx=ctx + 16, max_batch=8)
        eng = E.Engine.load(cfg, seed=3)
        for sq in range(8):
            eng.prefill(rng.integers(0, cfg.n_vocab, ctx - 1), pos0=0, seq=sq, want_logits=False)
        eng.forward_batch(rng.integers(0, cfg.n_vocab, 8), np.full(8, ctx - 1, np.int32), want_logits=False)
        for b in (1, 8):
            kt = eng.time_kernels(b, iters=64)
            byts = b * ctx * 8 * 128 * 2 * 2
            gbs = byts / (kt["attention"] * 1e-3) / 1e9
            print(json.dumps({"sweep": "attention_hbm", "ctx": ctx, "b": b, "us": kt["attention"] * 1e3,
                              "bytes": byts, "GBps": gbs, "frac": gbs / peak, "peak_kind": peak_kind,
                              "layers_rotated": n_layer, "working_set_bytes": n_layer * byts,
                              "l2_resident": n_layer * byts < 126e6}), flush=True)
        eng.close()


def run_sweep_id_tc(peak, peak_kind):
    """configs[1]'s mul_mat_id at b in {16, 64} through the expert-grouped
    tensor-core op (sfk_mul_mat_id_tc): the routed pairs grouped by expert
    into 64-row tiles, one tcgen05 kind::i8 GEMM over every tile, the rows put
    back in pair order.  Mixtral expert shapes (E=8, gate 14336x4096 with one
    activation row per token, down 4096x14336 with one row per pair), top-2
    ids drawn uniformly without replacement (seeded), weights random bytes in
    the device layout.  Time = CUDA events around each whole call (grouping,
    activation quantization, GEMM, ungrouping, and the call's status
    read-back), mean of `iters` calls after 2 warm-up calls; the 8 experts'
    matrices (264-499 MB) exceed the 126 MB L2, so every call streams them
    from HBM.  Bytes = the distinct experts of the call x matrix bytes."""
    import torch
    from strataflow_b200 import lib as L
    from strataflow_b200 import ops
    names = {L.TYPE_Q4_K: "Q4_K", L.TYPE_Q6_K: "Q6_K", L.TYPE_Q8_0: "Q8_0"}
    d, F, E, k, iters = 4096, 14336, 8, 2, 10
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    rng = np.random.default_rng(4)
    for t in (L.TYPE_Q4_K, L.TYPE_Q6_K, L.TYPE_Q8_0):
        for (kern, rows, K) in (("gate", F, d), ("down", d, F)):
            rb = L.load().sfk_dev_row_bytes(t, K)
            w = torch.randint(0, 255, (E * rows * rb,), dtype=torch.uint8, device="cuda", generator=g)
            for b in (16, 64):
                ids_np = np.stack([rng.choice(E, k, replace=False) for _ in range(b)]).astype(np.int32)
                ids = torch.from_numpy(ids_np).cuda()
                x = torch.randn((b, K) if kern == "gate" else (b, k, K), device="cuda", generator=g)
                for _ in range(2):
                    ops.mul_mat_id_tc(t, w, E, rows, K, x, ids)
                torch.cuda.synchronize()
                tot = 0.0
                for _ in range(iters):
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    ops.mul_mat_id_tc(t, w, E, rows, K, x, ids)
                    e1.record()
                    e1.synchronize()
                    tot += e0.elapsed_time(e1)
                ms = tot / iters
                uniq = int(np.unique(ids_np).size)
                byts = uniq * rows * rb
                gbs = byts / (ms * 1e-3) / 1e9
                print(json.dumps({"sweep": "mul_mat_id_tc", "kernel": kern, "wtype": names[t], "b": b, "k": k,
                                  "us": ms * 1e3, "bytes": byts, "GBps": gbs, "frac": gbs / peak,
                                  "peak_kind": peak_kind, "unique_experts": uniq,
                                  "int8_TOPS": 2.0 * b * k * rows * K / (ms * 1e-3) / 1e12,
                                  "note": "whole call: group + quantize + GEMM + ungroup + status read-back"}),
                      flush=True)
            del w


def run_sweep_tc(args):
    """The tensor-core GEMM (sfk_mul_mat_tc, tcgen05 kind::i8) at the Mixtral
    expert shapes for n activation rows -- a batch of n tokens' routed pairs
    of one expert, or n prompt tokens -- and the batched prompt prefill of the
    full 32-layer Mixtral shape.  GEMM: CUDA events around `iters` calls on the
    current stream (activation quantization included, its status read-back
    excluded by timing a whole loop); weights are random bytes in the device
    layout (the timing does not depend on their values).  One JSON line per
    case."""
    import torch
    from strataflow_b200 import engine as E
    from strataflow_b200 import lib as L
    from strataflow_b200 import ops
    names = {L.TYPE_Q4_K: "Q4_K", L.TYPE_Q6_K: "Q6_K", L.TYPE_Q8_0: "Q8_0"}
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    iters = 10
    for t in (L.TYPE_Q4_K, L.TYPE_Q6_K, L.TYPE_Q8_0):
        for (kern, rows, K) in (("gate", 14336, 4096), ("down", 4096, 14336)):
            rb = L.load().sfk_dev_row_bytes(t, K)
            w = torch.randint(0, 255, (rows * rb,), dtype=torch.uint8, device="cuda", generator=g)
            for n in (16, 64, 128, 512):
                x = torch.randn(n, K, device="cuda", generator=g)
                for _ in range(2):
                    ops.mul_mat_tc(t, w, rows, K, x)
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(iters):
                    ops.mul_mat_tc(t, w, rows, K, x)
                e1.record()
                e1.synchronize()
                ms = e0.elapsed_time(e1) / iters
                print(json.dumps({"sweep": "mul_mat_tc", "kernel": kern, "wtype": names[t], "n": n, "rows": rows,
                                  "K": K, "us": ms * 1e3, "int8_TOPS": 2.0 * rows * K * n / (ms * 1e-3) / 1e12,
                                  "weight_GBps": rows * rb / (ms * 1e-3) / 1e9,
                                  "note": "one matrix per call; includes activation quantization"}), flush=True)
            del w
    # the batched prefill of the benchmark's model
    cfg = E.mixtral_config(n_ctx=PROMPT + 16, n_layer=args.layers)
    eng = E.Engine.load(cfg, seed=SEED)
    prompt = np.random.default_rng(SEED).integers(0, cfg.n_vocab, PROMPT).astype(np.int32)
    eng.prefill(prompt, want_logits=False)
    times = []
    for _ in range(3):
        eng.reset_kv()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        eng.prefill(prompt, want_logits=False)
        times.append(time.perf_counter() - t0)
    best = min(times)
    print(json.dumps({"sweep": "prefill", "model": f"Mixtral-8x7B shape, {cfg.n_layer} layers", "tokens": PROMPT,
                      "s": best, "tok_s": PROMPT / best, "runs_s": times,
                      "timing": "host wall clock around sfk_prefill (synchronous), best of 3"}), flush=True)
    eng.close()


def run_tier(args):
    """Decode at the Mixtral shape with a bounded expert tier: `expert_slots`
    of the 256 expert bundles in HBM, the rest streamed from pinned host
    memory (one host-to-device copy per missing bundle).  One JSON line: the
    device-timed decode rate and, over the timed steps, the pool's hits,
    misses and host-to-device traffic against the measured pinned copy rate."""
    import torch
    from strataflow_b200 import engine as E

    torch.cuda.set_device(0)
    B = args.batch
    n_ctx = args.prompt + args.warmup + args.steps + 16
    cfg = E.mixtral_config(n_ctx=n_ctx, max_batch=B, n_layer=args.layers, expert_slots=args.expert_slots,
                           kv_window=args.kv_window)
    t_load = time.perf_counter()
    eng = E.Engine.load(cfg, seed=SEED)
    t_load = time.perf_counter() - t_load
    stream = torch.cuda.ExternalStream(eng.stream, device=torch.device("cuda", 0))
    prompt = np.random.default_rng(SEED).integers(0, cfg.n_vocab, (B, args.prompt)).astype(np.int32)
    torch.cuda.synchronize()
    t_pf = time.perf_counter()
    for s_ in range(B):
        eng.prefill(prompt[s_], seq=s_, want_logits=False)
    t_pf = time.perf_counter() - t_pf
    eng.decode_greedy(args.warmup, B, want_tokens=False)
    s0 = eng.stats()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        ev0.record(stream)
        eng.decode_greedy(args.steps, B, want_tokens=False)
        ev1.record(stream)
        ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    s1 = eng.stats()
    d = {k: s1[k] - s0[k] for k in ("pool_hits", "pool_misses", "pool_evictions", "h2d_expert_bytes",
                                    "prefetch_warmed", "prefetch_used", "kv_pages_evicted", "kv_staged_bytes")}
    h2d_gbs = (d["h2d_expert_bytes"] + d["kv_staged_bytes"]) / (ms / 1e3) / 1e9
    eng.close()
    # the pinned host-to-device copy rate of this box (1 GiB, 5 copies)
    host = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dev = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    dev.copy_(host, non_blocking=True)
    torch.cuda.synchronize()
    c0 = torch.cuda.Event(enable_timing=True)
    c1 = torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(5):
        dev.copy_(host, non_blocking=True)
    c1.record()
    c1.synchronize()
    pin_gbs = 5 * (1 << 30) / (c0.elapsed_time(c1) / 1e3) / 1e9
    bundle = 3 * 14336 * (4096 // 256 * 144)
    line = {
        "metric": METRIC, "value": B * args.steps / (ms / 1e3), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_k/q6_k weights x q8_k int8 dot (dp4a), fp32 accum", "data": "synthetic",
        "config": {"workload": f"Mixtral-8x7B-shape decode b={B}, {args.prompt}-token prompt"
                               + (f", bounded expert tier: {args.expert_slots} of {cfg.n_layer * 8} expert bundles "
                                  "in HBM" if args.expert_slots else "")
                               + (f", KV window of {args.kv_window} tokens" if args.kv_window else ""),
                   "model": "mixtral-8x7b-shape (32L d4096 32q/8kv E8 top2 F14336 V32000)",
                   "global_batch": B, "seq_len": args.prompt, "expert_slots": args.expert_slots,
                   "pool": "global LRU" if os.environ.get("SFK_POOL_GLOBAL_LRU") == "1" else "layer-stratified LRU",
                   "prefetch": {"0": "off", "2": "evicting warm"}.get(os.environ.get("SFK_PREFETCH", "1"),
                                                                       "into free slots")},
        "clocks": clk.summary(),
        "tier": None if not args.expert_slots else {"bundle_bytes": bundle, "hits": d["pool_hits"], "misses": d["pool_misses"],
                 "evictions": d["pool_evictions"], "hit_rate": d["pool_hits"] / max(1, d["pool_hits"] + d["pool_misses"]),
                 "misses_per_token": d["pool_misses"] / (B * args.steps), "prefetch_warmed": d["prefetch_warmed"],
                 "prefetch_used": d["prefetch_used"], "h2d_gbs": h2d_gbs, "pinned_h2d_peak_gbs": pin_gbs,
                 "h2d_frac": h2d_gbs / pin_gbs},
        "kv_window": {"tokens": args.kv_window, "pages_evicted": d["kv_pages_evicted"],
                      "staged_bytes_per_token": d["kv_staged_bytes"] / (B * args.steps)} if args.kv_window else None,
        "load_s": t_load, "prefill_s": t_pf,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt tokens fed before decoding")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end loop")
    ap.add_argument("--layers", type=int, default=32, help="model depth (32 = the benchmark; fewer for profiling)")
    ap.add_argument("--no-kernel-times", action="store_true",
                    help="print only the device-timed decode rate (short profiling runs)")
    ap.add_argument("--model", choices=["mixtral", "1t"], default="mixtral",
                    help="1t: configs[4], experts sharded over the torchrun ranks")
    ap.add_argument("--sweep", action="store_true",
                    help="operator sweeps (configs[1] mul_mat_id, configs[2] attention), one JSON line per case")
    ap.add_argument("--sweep-tc", action="store_true",
                    help="tensor-core GEMM sweep (n = 16..512 rows) and the batched 512-token prefill")
    ap.add_argument("--expert-slots", type=int, default=0,
                    help="decode with a bounded expert tier of this many HBM bundle slots (one GPU)")
    ap.add_argument("--no-ep", action="store_true",
                    help="at 4+ GPUs, skip the nested expert-parallel ~1T measurement")
    ap.add_argument("--kv-window", type=int, default=0,
                    help="decode with a KV window of this many resident tokens per sequence (one GPU)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.sweep:
        run_sweep(args)
        return
    if args.sweep_tc:
        run_sweep_tc(args)
        return
    if args.expert_slots > 0 or args.kv_window > 0:
        run_tier(args)
        return
    if args.model == "1t":
        if args.layers == 32:
            args.layers = 61
        if args.prompt == PROMPT:
            args.prompt = 1024
        run_ep(args, rank, world, local_rank)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
