#!/usr/bin/env python3
"""Benchmark of the B200 attention core (one JSON line on rank 0).

Default workload: batched serving decode of a Qwen3.5-4B
shaped 32-layer stack (24 Gated DeltaNet + 8 gated full-attention layers, 3:1),
256 concurrent sequences per GPU with ragged KV lengths ~ U[512, 32768] (fp16
N(0,1)) and per-sequence fp32 DeltaNet state N(0, 0.1).  One step = one decode
token for every sequence through all 32 layers' attention cores, each layer one
call of the C ABI (anelm_full_attn_decode / anelm_deltanet_decode) on the
layer's synthetic projection rows.  Sequences are independent: under torchrun
each rank owns its own 256 sequences (weak scaling, no data-path collective).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python bench.py --workload fa_b1|gdn_b1      # BASELINE configs 1 / 2 (single sequence)
    python bench.py --workload fa_prefill [--prefill-batch 8]
    python bench.py --workload gdn_prefill
    python bench.py --workload proj|lm_head [--seqs 256]       # the steps next to the core
    python bench.py --workload gdn_layer [--seqs 256]          # one DeltaNet decode layer (ncu size)

The reference arm (--impl reference) times the reference's own CPU attention
core (core/cpu_ops.cpp compiled unmodified + the qwen3_5.cpp glue, oracle/_ref)
on the host cores over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "ane-lm_b200"))

PEAKS = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK_HBM = 6650.0

# Qwen3.5-4B attention-core shape (serve_hybrid.py:32-47)
HQ, HKV, HD, ROT = 16, 4, 256, 64
HK, HV, DK, DV = 16, 32, 128, 128
N_LAYERS = 32
LAYER_TYPES = [1 if (l + 1) % 4 == 0 else 0 for l in range(N_LAYERS)]  # every 4th layer full attention
C_CONV = 2 * HK * DK + HV * DV
FA_PROJ = HQ * 2 * HD + 2 * HKV * HD
GDN_PROJ = C_CONV + HV * DV + 2 * HV
FA_OUT = HQ * HD
GDN_OUT = HV * DV


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    try:
        d = json.load(open(PEAKS))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


def kv_lengths(n, seed=0):
    return np.random.default_rng(seed).integers(512, 32768, size=n, endpoint=True).astype(np.int64)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampling during the timed region (median SM clock + throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        # nvidia-smi takes a while to start: wait (up to 5 s) for its first sample so that the
        # samples cover the timed region that follows
        t_end = time.time() + 5.0
        while time.time() < t_end and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.02)

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = [l.split(",") for l in open(self.path).read().strip().splitlines() if l.count(",") >= 8]
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if "Active" in val and "Not" not in val:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].strip().replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------------ GPU arm

def setup_serving(torch, n_seqs, lengths, slack, seed, device):
    import anelm_b200 as ab
    from anelm_b200.core import Context

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    caps = [int(L) + slack for L in lengths]
    ctx = Context(device=device.index or 0, layer_types=LAYER_TYPES, num_q_heads=HQ, num_kv_heads=HKV, head_dim=HD,
                  rot_dim=ROT, rope_theta=1e7, lin_num_key_heads=HK, lin_num_val_heads=HV,
                  seq_kv_capacity=caps, rope_table_len=4096)
    rng = np.random.default_rng(seed)
    # weights: QK-norm N(1, 0.02); conv fp16 N(0, 0.5); A = 1, dt_bias = 0; norm 1 + N(0, 0.1)
    for l, t in enumerate(LAYER_TYPES):
        if t == ab.LAYER_FULL_ATTN:
            ctx.set_full_attn_weights(l, (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32),
                                      (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32))
        else:
            cw = (0.5 * rng.standard_normal((C_CONV, 4))).astype(np.float16).astype(np.float32)
            ctx.set_deltanet_weights(l, cw, np.ones(HV, np.float32), np.zeros(HV, np.float32),
                                     (1 + 0.1 * rng.standard_normal(DV)).astype(np.float32))
    # KV: fp16 N(0,1) rows drawn from one random pool at rotating offsets (values are
    # N(0,1) everywhere; only their position in the pool repeats).
    row = HKV * HD
    pool_rows = 1 << 18
    src = torch.randn(pool_rows + 32768, row, generator=g, device=device, dtype=torch.float16)
    off = 0
    for l, t in enumerate(LAYER_TYPES):
        if t != ab.LAYER_FULL_ATTN:
            continue
        for s, L in enumerate(lengths):
            L = int(L)
            o1 = off % pool_rows
            o2 = (off * 7 + 12345) % pool_rows
            ctx.kv_write(l, s, 0, src[o1:o1 + L], src[o2:o2 + L])
            ctx.kv_set_meta(l, s, L, 0)
            off += 104729
    del src
    st = (0.1 * torch.randn(16, HV, DK, DV, generator=g, device=device, dtype=torch.float32)).contiguous()
    for l, t in enumerate(LAYER_TYPES):
        if t != ab.LAYER_LINEAR_ATTN:
            continue
        for s in range(n_seqs):
            ctx.deltanet_state_write(l, s, st[(s + l) % 16])
    torch.cuda.synchronize(device)
    del st
    plan = ctx.plan(list(range(n_seqs)))
    projs = []
    for t in LAYER_TYPES:
        w = FA_PROJ if t == ab.LAYER_FULL_ATTN else GDN_PROJ
        projs.append(torch.randn(n_seqs, w, generator=g, device=device, dtype=torch.float16))
    outs = [torch.empty(n_seqs, FA_OUT if t == ab.LAYER_FULL_ATTN else GDN_OUT, device=device,
                        dtype=torch.float16) for t in LAYER_TYPES]
    return ctx, plan, projs, outs


def step_bytes(lengths, step_offset):
    """Algorithmic HBM bytes of ONE full-attention layer launch and ONE DeltaNet layer
    launch over all sequences at `step_offset` tokens past the initial lengths."""
    n = len(lengths)
    Lcur = lengths + step_offset
    fa = 0
    fa += int((2 * Lcur * HKV * HD * 2).sum())          # K and V rows read (old tokens)
    fa += n * (FA_PROJ * 2 + FA_OUT * 2 + 2 * HKV * HD * 2)  # projection in, output, appended k/v
    gdn = n * (2 * HV * DK * DV * 4                      # state read + write
               + C_CONV * 16                             # conv ring: 3 old inputs read + 1 written
               + GDN_PROJ * 2 + GDN_OUT * 2) + C_CONV * 16  # projection in, output; conv weights
    return fa, gdn


def run_gpu(args):
    import torch
    import torch.distributed as dist

    rank, world, local = env_rank()
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    hbm_peak, peak_kind = peaks()

    if args.workload == "fa_prefill":
        return run_prefill(args, torch, device)
    if args.workload == "gdn_prefill":
        return run_gdn_prefill(args, torch, device, hbm_peak, peak_kind)
    if args.workload in ("proj", "lm_head"):
        return run_proj(args, torch, device, hbm_peak, peak_kind)
    if args.workload == "gdn_layer":
        return run_gdn_layer(args, torch, device, hbm_peak, peak_kind)
    if args.workload != "serve":
        return run_gpu_single(args, torch, device, hbm_peak, peak_kind)

    n = args.seqs
    lengths = kv_lengths(n, 0)
    slack = args.warmup + args.steps + 16
    ctx, plan, projs, outs = setup_serving(torch, n, lengths, slack, 1000 + rank, device)
    import anelm_b200 as ab

    pos = [torch.tensor(lengths + k, dtype=torch.int32, device=device) for k in range(args.warmup + args.steps + 1)]
    fa_layers = [l for l, t in enumerate(LAYER_TYPES) if t == ab.LAYER_FULL_ATTN]
    stream = torch.cuda.current_stream(device)

    def step(k, ev=None):
        for l, t in enumerate(LAYER_TYPES):
            if t == ab.LAYER_FULL_ATTN:
                if ev is not None:
                    ev[l][0].record(stream)
                ctx.full_attn_decode(plan, l, projs[l], pos[k], outs[l])
                if ev is not None:
                    ev[l][1].record(stream)
            else:
                if ev is not None:
                    ev[l][0].record(stream)
                ctx.deltanet_decode(plan, l, projs[l], outs[l])
                if ev is not None:
                    ev[l][1].record(stream)

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    ev_steps = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in LAYER_TYPES]
                for _ in range(args.steps)]
    clocks = ClockSampler(local)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    t0.record(stream)
    for k in range(args.steps):
        step(args.warmup + k, ev_steps[k])
    t1.record(stream)
    torch.cuda.synchronize(device)
    ck = clocks.stop()
    ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
        dist.barrier()
    err = ctx.device_error()
    assert err == 0, f"device reported status {err}"

    # per-kernel times (events on the launching stream)
    fa_ms = [ev_steps[k][l][0].elapsed_time(ev_steps[k][l][1]) for k in range(args.steps) for l in fa_layers]
    gdn_ms = [ev_steps[k][l][0].elapsed_time(ev_steps[k][l][1]) for k in range(args.steps)
              for l, t in enumerate(LAYER_TYPES) if t == 0]
    n_fa = len(fa_layers)
    n_gdn = N_LAYERS - n_fa
    fa_b = gdn_b = 0  # per-launch bytes summed over the timed steps
    for k in range(args.steps):
        a, b = step_bytes(lengths, args.warmup + k)
        fa_b += a
        gdn_b += b
    fa_per_launch = fa_b / args.steps
    gdn_per_launch = gdn_b / args.steps
    fa_gbs = fa_per_launch / (statistics.mean(fa_ms) * 1e-3) / 1e9
    gdn_gbs = gdn_per_launch / (statistics.mean(gdn_ms) * 1e-3) / 1e9
    ms_step = ms / args.steps
    tok_s = n * world / (ms_step * 1e-3)
    step_gb = (n_fa * fa_per_launch + n_gdn * gdn_per_launch) / 1e9

    # e2e: same step through the C ABI with host (pinned) buffers, copies inside the timed region
    e2e = run_e2e(args, torch, ctx, plan, projs, outs, pos, device, world)

    result = {
        "metric": "decode attn-core tok/s (batched serving decode, 32-layer 3:1 DeltaNet:attention stack)",
        "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "BASELINE cfg5: batched serving decode, Qwen3.5-4B-shaped 32 layers (24 GDN + 8 FA)",
                   "seqs_per_gpu": n, "global_batch": n * world, "kv_len": "U[512,32768] seed 0",
                   "kv_storage": "fp16 ring [slots][4][256]", "state": "fp32 [32][128][128] per seq per GDN layer",
                   "proj_io": "fp16", "Hq": HQ, "Hkv": HKV, "head_dim": HD, "rot_dim": ROT, "Hv": HV, "Hk": HK,
                   "parallelism": f"sequence-sharded x{world}, no collective",
                   "l2": f"inputs {step_gb:.1f} GB/step > 126 MB L2 (no flush needed)"},
        "hbm_gbs_step": round(step_gb / (ms_step * 1e-3), 1),
        "roofline": {"bound": "hbm", "kernel": "fa_decode_kernel<256>", "achieved": round(fa_gbs, 1),
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(fa_gbs / hbm_peak, 4),
                     "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_bytes_per_launch": int(fa_per_launch)},
        "roofline_gdn": {"bound": "hbm", "kernel": "gdn_decode_kernel", "achieved": round(gdn_gbs, 1),
                         "peak": hbm_peak, "unit": "GB/s", "frac": round(gdn_gbs / hbm_peak, 4),
                         "algorithmic_bytes_per_launch": int(gdn_per_launch)},
        "e2e": e2e,
        "kernel_ms_per_step": {"fa_decode": round(n_fa * statistics.mean(fa_ms), 3),
                               "gdn_decode": round(n_gdn * statistics.mean(gdn_ms), 3)},
        "gpu_launches": args.steps * N_LAYERS,
        "clocks": ck,
    }
    if args.traffic_json and os.path.exists(args.traffic_json):
        tr = json.load(open(args.traffic_json))
        result["roofline"]["traffic"] = tr.get("fa_decode_bytes_per_launch")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_reference_serving(args.cpu_seconds, threads=None, kind="reference")
    if rank == 0:
        print(json.dumps(result), flush=True)
    plan.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, torch, ctx, plan, projs, outs, pos, device, world):
    """The step with projections coming from pinned HOST memory and outputs going back
    to the host every step (copies on a side stream, overlapped with earlier layers)."""
    import anelm_b200 as ab
    import torch.distributed as dist

    host_in = [p.cpu().pin_memory() for p in projs]
    host_out = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
    comp = torch.cuda.current_stream(device)
    copy = torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in LAYER_TYPES]
    ev_out = [torch.cuda.Event() for _ in LAYER_TYPES]
    h2d = sum(h.numel() * h.element_size() for h in host_in)
    d2h = sum(h.numel() * h.element_size() for h in host_out)
    base = args.warmup + args.steps  # positions continue after the device-resident run
    # each e2e step appends one more token; capacity slack covers warmup + steps + 16

    def step(k):
        with torch.cuda.stream(copy):
            for l in range(N_LAYERS):
                projs[l].copy_(host_in[l], non_blocking=True)
                ev_in[l].record(copy)
        for l, t in enumerate(LAYER_TYPES):
            comp.wait_event(ev_in[l])
            if t == ab.LAYER_FULL_ATTN:
                ctx.full_attn_decode(plan, l, projs[l], pos[min(k, len(pos) - 1)], outs[l])
            else:
                ctx.deltanet_decode(plan, l, projs[l], outs[l])
            ev_out[l].record(comp)
            with torch.cuda.stream(copy):
                copy.wait_event(ev_out[l])
                host_out[l].copy_(outs[l], non_blocking=True)
        copy.synchronize()

    n_steps = max(1, min(args.steps, 8))
    step(base)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    t = time.perf_counter()
    for k in range(n_steps):
        step(base)
    torch.cuda.synchronize(device)
    dt = (time.perf_counter() - t) / n_steps
    if world > 1:
        tt = torch.tensor([dt], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dt = float(tt.item())
    n = plan.n
    return {"value": round(n * world / dt, 1), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": n_steps,
            "note": "host pinned projections in / outputs out each step, timed on the host clock"}


def run_prefill(args, torch, device):
    """causal full-attention prefill, Qwen3.5-4B shape, 4096 tokens, bf16 inputs."""
    import anelm_b200 as ab
    from anelm_b200.core import Context

    try:
        peak = float(json.load(open(PEAKS))["bf16_tflops"])
        peak_kind = "measured"
    except Exception:
        peak, peak_kind = 1590.0, "fallback"
    rng = np.random.default_rng(0)
    g = torch.Generator(device=device)
    g.manual_seed(0)
    B, n = args.prefill_batch, args.prefill_len
    ctx = Context(device=device.index or 0, layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=HQ, num_kv_heads=HKV,
                  head_dim=HD, rot_dim=ROT, rope_theta=1e7, max_seqs=B, kv_capacity=n)
    ctx.set_full_attn_weights(0, (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32),
                              (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32))
    plan = ctx.plan(list(range(B)))
    proj = torch.randn(B, n, FA_PROJ, generator=g, device=device).to(torch.bfloat16)
    out = torch.empty(B, n, FA_OUT, device=device, dtype=torch.bfloat16)

    def call():
        ctx.reset(-1)
        ctx.full_attn_prefill(plan, 0, proj, 0, out)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(device)
    times = []
    clocks = ClockSampler(device.index or 0)
    clocks.start()
    for _ in range(args.steps):
        ctx.reset(-1)  # synchronous; outside the timed region
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        ctx.full_attn_prefill(plan, 0, proj, 0, out)
        t1.record()
        torch.cuda.synchronize(device)
        times.append(t0.elapsed_time(t1))
    ck = clocks.stop()
    ms = statistics.median(times)
    flops = 4.0 * n * n * HD * HQ / 2 * B  # causal: half of the S x S score / PV work
    tf = flops / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": "causal prefill attention TFLOP/s (cfg3, Qwen3.5-4B shape)", "value": round(tf, 1),
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 operands, f32 accumulate",
        "data": "synthetic",
        "config": {"workload": f"BASELINE cfg3 prefill B={B} S={n}", "Hq": HQ, "Hkv": HKV, "head_dim": HD,
                   "proj": "bf16 N(0,1)", "timed": "whole call: prep (norm, RoPE, ring append) + V^T + attention"},
        "roofline": {"bound": "tensor", "kernel": "fa_prefill_kernel", "achieved": round(tf, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(tf / peak, 4), "peak_kind": peak_kind, "traffic": None,
                     "algorithmic_flops_per_launch": flops},
        "clocks": ck,
        "gpu_launches": 3 * args.steps}), flush=True)
    plan.close()
    ctx.close()


def gdn_chunk_flops(T, Hv, B=1, C=64, dk=128, dv=128):
    """Algorithmic FLOPs of the chunked delta rule: per chunk and value head 2C^2(3dk + 2dv)
    (K K^T, Q K^T, W, U, M D) + 6 C dk dv (W S, Q S, K^T D)."""
    n_chunks = (T + C - 1) // C
    return float(2 * C * C * (3 * dk + 2 * dv) + 6 * C * dk * dv) * n_chunks * Hv * B


def cpu_reference_gdn_chunk(T_sample, Hk, Hv):
    """The reference delta-rule step (core/cpu_ops.cpp ssm_step via oracle/_ref/libref_core_fast.so)
    over a token sample of the config-4 workload, one host thread; returns seconds per token."""
    from oracle import pyoracle as po

    kind = "ref_fast" if po.available("ref_fast") else "oracle"
    rng = np.random.default_rng(1)
    q = rng.standard_normal((T_sample, Hk, 128)).astype(np.float32)
    k = q / np.linalg.norm(q, axis=-1, keepdims=True)
    v = rng.standard_normal((T_sample, Hv, 128)).astype(np.float32)
    lg = (-0.1 * rng.random((T_sample, Hv))).astype(np.float32)
    beta = rng.random((T_sample, Hv)).astype(np.float32)
    st = np.zeros((Hv, 128, 128), np.float32)
    t0 = time.perf_counter()
    po.gated_delta_tokens(kind, q, k, v, lg, beta, st, 0)
    return (time.perf_counter() - t0) / T_sample, kind


def run_gdn_prefill(args, torch, device, hbm_peak, peak_kind):
    """the chunked gated delta rule, Hv 32 / Hk 16, dk = dv = 128, seq 8192,
    batch 1; bf16 q / k / v N(0, 1) with L2-normalised k, log g ~ U(-0.1, 0), beta ~ U(0, 1)."""
    from anelm_b200.core import gated_delta_chunked
    import anelm_b200 as ab

    try:
        tpeak = float(json.load(open(PEAKS))["bf16_tflops"])
        tpeak_kind = "measured"
    except Exception:
        tpeak, tpeak_kind = 1590.0, "fallback"
    B, T, Hk, Hv = args.prefill_batch, args.gdn_len, 16, 32
    g = torch.Generator(device=device)
    g.manual_seed(4)
    q = torch.randn(B, T, Hk, 128, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(B, T, Hk, 128, generator=g, device=device)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn(B, T, Hv, 128, generator=g, device=device).to(torch.bfloat16)
    lg = -0.1 * torch.rand(B, T, Hv, generator=g, device=device)
    beta = torch.rand(B, T, Hv, generator=g, device=device)
    state = torch.zeros(B, Hv, 128, 128, device=device)
    y = torch.empty(B, T, Hv, 128, device=device, dtype=torch.bfloat16)
    ws = torch.empty(ab.lib().anelm_gated_delta_chunked_workspace_bytes(B, T, Hk, Hv), dtype=torch.uint8,
                     device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)  # > 126 MB L2

    def call():
        gated_delta_chunked(q, k, v, lg, beta, state, ab.DELTA_CPUOPS, y=y, workspace=ws)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index or 0)
    clocks.start()
    times = []
    for _ in range(args.steps):
        flush.zero_()  # inputs (24 MB) would otherwise stay in L2 between iterations
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        call()
        t1.record()
        torch.cuda.synchronize(device)
        times.append(t0.elapsed_time(t1))
    ck = clocks.stop()
    ms = statistics.median(times)
    flops = gdn_chunk_flops(T, Hv, B)
    tf = flops / (ms * 1e-3) / 1e12
    nbytes = B * (2 * T * Hk * 128 * 2 + T * Hv * 128 * 2 + 2 * T * Hv * 4 + T * Hv * 128 * 2 + 2 * Hv * 128 * 128 * 4)
    sec_tok, kind = cpu_reference_gdn_chunk(64, Hk, Hv)
    cpu_tf = flops / (sec_tok * T * B) / 1e12
    print(json.dumps({
        "metric": "chunked Gated DeltaNet prefill TFLOP/s (cfg4, Hv 32 / Hk 16, d 128)", "value": round(tf, 2),
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 in, fp32 (hi/lo fp16 split) tensor-core products and state", "data": "synthetic",
        "config": {"workload": f"BASELINE cfg4 chunked delta rule B={B} S={T} chunk 64", "Hk": Hk, "Hv": Hv,
                   "dk": 128, "dv": 128, "l2": "256 MB buffer written between timed iterations"},
        "roofline": {"bound": "tensor", "kernel": "gdn_pf_chain_kernel + gdn_pf_chunk_kernel", "achieved": round(tf, 2),
                     "peak": tpeak, "unit": "TFLOP/s", "frac": round(tf / tpeak, 4), "peak_kind": tpeak_kind,
                     "traffic": None, "algorithmic_flops_per_launch": flops,
                     "hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 4), "algorithmic_bytes": nbytes},
        "cpu_baseline": {"value": round(cpu_tf, 6), "unit": "TFLOP/s", "cores": 1,
                         "kind": "reference" if kind == "ref_fast" else "port",
                         "sample": "64 tokens x 32 value heads of the token recurrence (ssm_step), scaled to "
                                   "the workload's algorithmic FLOPs"},
        "clocks": ck,
        "gpu_launches": 3 * args.steps}), flush=True)


def run_proj(args, torch, device, hbm_peak, peak_kind):
    """The steps next to the core (widening beyond the core): "proj" = the in- and out-projection
    GEMMs of one attention and one DeltaNet decode layer of the Qwen3.5-4B shape for `--seqs` rows
    (anelm_gemm_bf16); "lm_head" = the in-model top-32 LM head over the 248,320-token vocabulary
    for `--seqs` rows (anelm_lm_head_topk).  bf16 N(0,1) activations, N(0, 1/hidden) weights."""
    from anelm_b200.core import gemm_bf16, lm_head_topk

    try:
        tpeak = float(json.load(open(PEAKS))["bf16_tflops"])
        tpeak_kind = "measured"
    except Exception:
        tpeak, tpeak_kind = 1590.0, "fallback"
    n, H = args.seqs, 2560
    g = torch.Generator(device=device)
    g.manual_seed(0)

    def w(rows, cols):
        return (torch.randn(rows, cols, generator=g, device=device) / cols ** 0.5).to(torch.bfloat16)

    if args.workload == "proj":
        # attention: q|gate|k|v rows 16*512 + 2*4*256 = 10240, o_proj 2560 x 4096; DeltaNet:
        # qkv|z|a|b rows 2*16*128 + 2*32*128 + 2*32 = 12352, o_proj 2560 x 4096
        shapes = [(10240, H), (H, 4096), (12352, H), (H, 4096)]
        ws = [w(N, K) for N, K in shapes]
        xs = [torch.randn(n, K, generator=g, device=device).to(torch.bfloat16) for _, K in shapes]
        ys = [torch.empty(n, N, device=device, dtype=torch.bfloat16) for N, _ in shapes]

        def call():
            for x, wt, y in zip(xs, ws, ys):
                gemm_bf16(x, wt, out=y)

        flops = sum(2 * n * N * K for N, K in shapes)
        nbytes = sum((N * K + n * K + n * N) * 2 for N, K in shapes)
        metric = "decode-layer projection GEMMs TFLOP/s (Qwen3.5-4B attention + DeltaNet layer, bf16)"
        kernel, launches = "gemm_bf16_tn_kernel", len(shapes)
        cfg = {"workload": f"in/out projections of one attention and one DeltaNet layer, {n} rows",
               "gemms": [f"{n}x{N}x{K}" for N, K in shapes]}
    else:
        V = 248320
        wt = w(V, H)
        x = torch.randn(n, H, generator=g, device=device).to(torch.bfloat16)
        wsp = torch.empty(n * V, dtype=torch.uint8, device=device)  # >= the candidate buffer

        def call():
            lm_head_topk(x, wt, 32, wsp)

        flops, nbytes = 2 * n * V * H, (V * H + n * H) * 2 + n * 32 * 8
        metric = "LM head with in-model top-32 TFLOP/s (248,320-token vocabulary, hidden 2560, bf16)"
        kernel, launches = "lm_head_topk_kernel + lm_topk_merge_kernel", 2
        cfg = {"workload": f"top-32 LM head, {n} rows x 248320 x 2560"}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index or 0)
    clocks.start()
    times = []
    for _ in range(args.steps):
        flush.zero_()  # weights would otherwise stay in L2 between iterations
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        call()
        t1.record()
        torch.cuda.synchronize(device)
        times.append(t0.elapsed_time(t1))
    ck = clocks.stop()
    ms = statistics.median(times)
    tf = flops / (ms * 1e-3) / 1e12
    gbs = nbytes / (ms * 1e-3) / 1e9
    bound = "tensor" if flops / nbytes > tpeak * 1e12 / (hbm_peak * 1e9) else "hbm"
    roof = ({"bound": "tensor", "achieved": round(tf, 2), "peak": tpeak, "unit": "TFLOP/s",
             "frac": round(tf / tpeak, 4), "peak_kind": tpeak_kind} if bound == "tensor" else
            {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s",
             "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind})
    roof.update({"kernel": kernel, "traffic": None, "algorithmic_flops_per_launch": flops,
                 "algorithmic_bytes": nbytes})
    # CPU baseline: numpy (BLAS) on an 8-row sample of the same products (the reference runs them
    # on the ANE, so there is no reference CPU code for this step)
    rows = min(8, n)
    cpu_t = 0.0
    if not args.no_cpu_baseline:
        import time
        xs_c = np.random.default_rng(0).standard_normal((rows, H)).astype(np.float32)
        if args.workload == "proj":
            mats = [np.random.default_rng(i).standard_normal((N, K)).astype(np.float32) for i, (N, K) in
                    enumerate(shapes)]
            xin = [np.random.default_rng(9).standard_normal((rows, K)).astype(np.float32) for _, K in shapes]
            t0 = time.perf_counter()
            for xi, m in zip(xin, mats):
                xi @ m.T
            cpu_t = time.perf_counter() - t0
        else:
            m = np.random.default_rng(1).standard_normal((V // 8, H)).astype(np.float32)  # 1/8 of the vocabulary
            t0 = time.perf_counter()
            lg = xs_c @ m.T
            np.argpartition(lg, -32, axis=1)[:, -32:]
            cpu_t = (time.perf_counter() - t0) * 8
    cpu_tf = (flops * rows / n) / cpu_t / 1e12 if cpu_t > 0 else None
    print(json.dumps({
        "metric": metric, "value": round(tf, 2), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 in, fp32 accumulate", "data": "synthetic",
        "config": dict(cfg, l2="256 MB buffer written between timed iterations"),
        "hbm_gbs_step": round(gbs, 1), "roofline": roof,
        "cpu_baseline": {"value": round(cpu_tf, 6) if cpu_tf else None, "unit": "TFLOP/s",
                         "cores": os.cpu_count(), "kind": "port",
                         "sample": f"numpy fp32 matmul on {rows} rows" +
                                   (" of 1/8 of the vocabulary, scaled" if args.workload == "lm_head" else "")},
        "clocks": ck, "gpu_launches": launches * args.steps}), flush=True)


def run_gdn_layer(args, torch, device, hbm_peak, peak_kind):
    """One DeltaNet decode layer of the config-5 shape over `--seqs` sequences (the kernel of the
    serving step on its own, a few hundred MB of state: the size for an ncu capture)."""
    import anelm_b200 as ab
    from anelm_b200.core import Context

    n = args.seqs
    ctx = Context(device=device.index or 0, layer_types=[ab.LAYER_LINEAR_ATTN], lin_num_key_heads=HK,
                  lin_num_val_heads=HV, max_seqs=n, kv_capacity=16)
    rng = np.random.default_rng(0)
    cw = (0.5 * rng.standard_normal((C_CONV, 4))).astype(np.float16).astype(np.float32)
    ctx.set_deltanet_weights(0, cw, np.ones(HV, np.float32), np.zeros(HV, np.float32),
                             (1 + 0.1 * rng.standard_normal(DV)).astype(np.float32))
    g = torch.Generator(device=device)
    g.manual_seed(0)
    st = (0.1 * torch.randn(HV, DK, DV, generator=g, device=device)).contiguous()
    for s in range(n):
        ctx.deltanet_state_write(0, s, st)
    plan = ctx.plan(list(range(n)))
    proj = torch.randn(n, GDN_PROJ, generator=g, device=device, dtype=torch.float16)
    out = torch.empty(n, GDN_OUT, device=device, dtype=torch.float16)
    for _ in range(args.warmup):
        ctx.deltanet_decode(plan, 0, proj, out=out)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ctx.deltanet_decode(plan, 0, proj, out=out)
    e1.record()
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / args.steps
    nbytes = step_bytes(np.full(n, 1), 0)[1]              # same accounting as the serving step
    gbs = nbytes / (ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "DeltaNet decode layer GB/s (config-5 shape, one layer)", "value": round(gbs, 1), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"one DeltaNet layer, {n} sequences", "l2": f"state {n * HV * DK * DV * 4 >> 20} MB"},
        "roofline": {"bound": "hbm", "kernel": "gdn_decode_kernel", "achieved": round(gbs, 1), "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": nbytes},
        "gpu_launches": args.steps}), flush=True)
    plan.close()
    ctx.close()


def run_gpu_single(args, torch, device, hbm_peak, peak_kind):
    """BASELINE configs 1 and 2: one sequence, one layer call per step, replayed from a CUDA graph."""
    import anelm_b200 as ab
    from anelm_b200.core import Context

    rng = np.random.default_rng(0)
    g = torch.Generator(device=device)
    g.manual_seed(0)
    if args.workload == "fa_b1":
        ctx = Context(device=device.index or 0, layer_types=[ab.LAYER_FULL_ATTN], max_seqs=1, kv_capacity=2048)
        ctx.set_full_attn_weights(0, (1 + 0.02 * rng.standard_normal(256)).astype(np.float32),
                                  (1 + 0.02 * rng.standard_normal(256)).astype(np.float32))
        kv = torch.randn(2048, 2, 256, generator=g, device=device, dtype=torch.float16)
        ctx.kv_write(0, 0, 0, kv, kv.flip(0).contiguous())
        ctx.kv_set_meta(0, 0, 2048, 0)
        proj = torch.randn(ctx.fa_proj_dim, generator=g, device=device, dtype=torch.float16)
        out = torch.empty(ctx.fa_out_dim, device=device, dtype=torch.float16)
        call = lambda: ctx.full_attn_from_proj(0, 0, proj, 5000, out)  # noqa: E731
        nbytes = 2 * 2048 * 2 * 256 * 2 + ctx.fa_proj_dim * 2 + ctx.fa_out_dim * 2 + 2 * 2 * 256 * 2
        metric, kname = "FA decode step tok/s (cfg1, 0.8B shape, KV 2048 fp16)", "fa_decode_kernel<256>"
    else:
        ctx = Context(device=device.index or 0, layer_types=[ab.LAYER_LINEAR_ATTN], max_seqs=1)
        C = ctx.conv_channels
        ctx.set_deltanet_weights(0, (0.5 * rng.standard_normal((C, 4))).astype(np.float16).astype(np.float32),
                                 np.ones(16, np.float32), np.zeros(16, np.float32), np.ones(128, np.float32))
        st = (0.1 * torch.randn(16, 128, 128, generator=g, device=device)).contiguous()
        ctx.deltanet_state_write(0, 0, st)
        proj = torch.randn(ctx.gdn_proj_dim, generator=g, device=device, dtype=torch.float16)
        out = torch.empty(ctx.gdn_out_dim, device=device, dtype=torch.float16)
        call = lambda: ctx.deltanet_from_proj(0, 0, proj, out)  # noqa: E731
        nbytes = 2 * 16 * 128 * 128 * 4 + C * 16 + C * 16 + ctx.gdn_proj_dim * 2 + ctx.gdn_out_dim * 2
        metric, kname = "GDN decode step tok/s (cfg2, 16 heads, fp32 state)", "gdn_decode_kernel<8>"
    for _ in range(max(3, args.warmup)):
        call()
    torch.cuda.synchronize(device)
    reps = 64
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for _ in range(reps):
                call()
    torch.cuda.synchronize(device)
    graph.replay()
    torch.cuda.synchronize(device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        graph.replay()
    t1.record()
    torch.cuda.synchronize(device)
    us = t0.elapsed_time(t1) * 1e3 / (args.steps * reps)
    gbs = nbytes / (us * 1e-6) / 1e9
    print(json.dumps({"metric": metric, "value": round(1e6 / us, 1), "unit": "tok/s", "n_gpus": 1,
                      "steps": args.steps * reps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 6),
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                      "data": "synthetic", "config": {"workload": args.workload, "graph_replay": reps},
                      "roofline": {"bound": "hbm", "kernel": kname, "achieved": round(gbs, 1), "peak": hbm_peak,
                                   "unit": "GB/s", "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind,
                                   "traffic": None, "algorithmic_bytes_per_launch": nbytes},
                      "gpu_launches": args.steps * reps}), flush=True)
    ctx.close()


# ------------------------------------------------------------------ CPU reference arm

def cpu_reference_serving(seconds: float, threads=None, kind="reference"):
    """The reference CPU attention core (oracle/_ref/libref_core_fast.so: core/cpu_ops.cpp,
    unmodified, + the qwen3_5.cpp glue restated) on a bounded sample of the serving
    workload: `threads` sequences, each decoded token by token through all 32 layers
    (fp32 KV ring of its length, fp32 DeltaNet state), one host thread per sequence.
    Returns tokens/s over the sample."""
    from oracle import pyoracle as po

    lib_kind = "ref_fast" if po.available("ref_fast") else "oracle"
    threads = threads or max(1, min(os.cpu_count() or 1, 32))
    shape = po.make_shape(num_q_heads=HQ, num_kv_heads=HKV, head_dim=HD, rot_dim=ROT, rope_theta=1e7,
                          lin_num_key_heads=HK, lin_num_val_heads=HV)
    var = po.make_variant()
    lengths = kv_lengths(256, 0)[:threads]
    rng = np.random.default_rng(0)
    qn = (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32)
    cw = (0.5 * rng.standard_normal((C_CONV, 4))).astype(np.float16).astype(np.float32)
    A, dtb = np.ones(HV, np.float32), np.zeros(HV, np.float32)
    nw = np.ones(DV, np.float32)
    rope = po.rope_table(4096, ROT, 1e7)
    block = rng.standard_normal((4096, HKV, HD)).astype(np.float32)
    fa_proj = rng.standard_normal(FA_PROJ).astype(np.float32)
    gdn_proj = rng.standard_normal(GDN_PROJ).astype(np.float32)
    fa = po.fn(lib_kind, "full_attn_from_proj")
    gdn = po.fn(lib_kind, "deltanet_from_proj")
    P = po.P

    def worker(i):
        L = int(lengths[i])
        cap = L + 64
        rings = []
        for _ in range(8):
            k = np.empty((cap, HKV, HD), np.float32)
            v = np.empty((cap, HKV, HD), np.float32)
            for o in range(0, cap, 4096):
                m = min(4096, cap - o)
                k[o:o + m] = block[:m]
                v[o:o + m] = block[::-1][:m]
            rings.append([k, v, ctypes.c_int(L), ctypes.c_int(0)])
        states = [po.DeltaState.zeros(shape) for _ in range(24)]
        for s in states:
            s.ssm[:] = 0.01
        out_fa = np.zeros(FA_OUT, np.float32)
        out_g = np.zeros(GDN_OUT, np.float32)
        tmp = np.zeros(HD, np.float32)
        scratch = np.zeros(2 * C_CONV + GDN_OUT, np.float32)
        pbuf = np.empty(FA_PROJ, np.float32)
        tokens = 0
        t_end = time.perf_counter() + seconds
        t0 = time.perf_counter()
        while True:
            fi = gi = 0
            for t in LAYER_TYPES:
                if t == 1:
                    k, v, ln, st = rings[fi]
                    pbuf[:] = fa_proj
                    fa(ctypes.byref(shape), ctypes.byref(var), P(qn), P(qn), P(k), P(v), ctypes.byref(ln),
                       ctypes.byref(st), cap, P(rope[0]), P(rope[1]), 4096, P(pbuf), L + tokens, P(out_fa), P(tmp))
                    fi += 1
                else:
                    s = states[gi]
                    cp = ctypes.c_int(s.conv_pos)
                    gdn(ctypes.byref(shape), ctypes.byref(var), P(cw), P(A), P(dtb), P(nw), P(s.ssm), P(s.conv),
                        ctypes.byref(cp), P(gdn_proj), P(out_g), P(scratch))
                    s.conv_pos = cp.value
                    gi += 1
            tokens += 1
            if time.perf_counter() >= t_end or tokens >= 60:
                break
        return tokens, time.perf_counter() - t0

    with ThreadPoolExecutor(max_workers=threads) as ex:
        res = list(ex.map(worker, range(threads)))
    toks = sum(r[0] for r in res)
    wall = max(r[1] for r in res)
    cpu_model = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                cpu_model = line.split(":", 1)[1].strip()
                break
    except Exception:
        pass
    return {"value": round(toks / wall, 3), "unit": "tok/s", "cores": threads, "kind": kind,
            "sample": (f"{threads} sequences (KV lengths = the first {threads} of the workload's U[512,32768] draw), "
                       f"{toks} tokens through all 32 layers, fp32 KV/state, {wall:.1f} s wall; "
                       f"lib={os.path.basename(po.LIBS[lib_kind])}; cpu={cpu_model}; nproc={os.cpu_count()}")}


def run_reference(args):
    rank, world, local = env_rank()
    if rank != 0:
        return
    cb = cpu_reference_serving(args.cpu_seconds, threads=None, kind="reference")
    print(json.dumps({
        "impl": "reference",
        "metric": "decode attn-core tok/s (batched serving decode, 32-layer 3:1 DeltaNet:attention stack)",
        "value": cb["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "BASELINE cfg5: batched serving decode, Qwen3.5-4B-shaped 32 layers (24 GDN + 8 FA)",
                   "seqs_per_gpu": args.seqs, "kv_len": "U[512,32768] seed 0"},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="anelm", choices=["anelm", "reference"])
    ap.add_argument("--workload", default="serve",
                    choices=["serve", "fa_b1", "gdn_b1", "fa_prefill", "gdn_prefill", "proj", "lm_head",
                             "gdn_layer"])
    ap.add_argument("--gdn-len", type=int, default=8192)
    ap.add_argument("--prefill-batch", type=int, default=1)
    ap.add_argument("--prefill-len", type=int, default=4096)
    ap.add_argument("--seqs", type=int, default=256)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--traffic-json", default=os.path.join(REPO, "profiles", "traffic.json"))
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
