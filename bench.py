#!/usr/bin/env python3
"""Benchmark of the B200 attention core (one JSON line on rank 0).

Default workload: batched serving decode of a Qwen3.5-4B shaped 32-layer
stack (24 Gated DeltaNet + 8 gated full-attention layers, 3:1), 256 concurrent sequences with
ragged KV lengths ~ U[512, 32768] (fp16 N(0,1)) and per-sequence fp32 DeltaNet state
N(0, 0.1).  One step = one decode token for every sequence through all 32 layers' attention
cores, each layer one call of the C ABI (anelm_full_attn_decode / anelm_deltanet_decode) on the
layer's synthetic projection rows.

Multi-GPU (torchrun, one process per GPU): the 256 sequences are split over the ranks by
greedy longest-first bin packing of their per-step bytes (strong scaling, the headline at
N > 1; no data-path collective).  The line also carries a weak-scaling measurement (256
sequences on every rank) under "weak".

At N = 1 the line carries BASELINE configs 1-4 under "workloads" (single-sequence decode of
each block, causal prefill at B = 1 and 8, chunked DeltaNet prefill), each with its roofline
fraction, clocks and the reference CPU core timed on the same inputs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--no-workloads]
    python bench.py --workload fa_b1|gdn_b1      # BASELINE configs 1 / 2 alone
    python bench.py --workload fa_prefill [--prefill-batch 8]   # BASELINE config 3 alone
    python bench.py --workload gdn_prefill                      # BASELINE config 4 alone
    torchrun ... bench.py --workload fa_prefill|gdn_prefill     # configs 3 (B=1) / 4 head-sharded over N GPUs
    python bench.py --workload proj|lm_head [--seqs 256]       # the steps next to the core
    python bench.py --workload gdn_layer [--seqs 256]          # one DeltaNet decode layer (ncu size)

The reference arm (--impl reference) times the reference's own CPU attention core
(core/cpu_ops.cpp compiled unmodified + the qwen3_5.cpp glue, oracle/_ref) on the host cores
over a bounded sample of the same workload.
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
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "ane-lm_b200"))

PEAKS = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK_HBM, FALLBACK_BF16 = 6650.0, 1590.0

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
GLOBAL_SEQS = 256
METRIC = "decode attn-core tok/s (batched serving decode, 32-layer 3:1 DeltaNet:attention stack)"
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2
# A fixed-length spin kernel (torch.cuda._sleep, ~0.1 ms at 2 GHz) queued right before a timed call's
# start event keeps the GPU busy while the host enqueues the call, so the events time the device work
# of the call, not the host's launch latency.
ENQUEUE_COVER_CYCLES = 200_000


def flush_and_cover(torch, flush, cycles=ENQUEUE_COVER_CYCLES):
    flush.zero_()
    torch.cuda._sleep(cycles)


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    """(HBM GB/s, bf16 TFLOP/s, kind) from MEASURED_PEAKS.json, else the pool's fallback."""
    try:
        d = json.load(open(PEAKS))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM, FALLBACK_BF16, "fallback"


def kv_lengths(n, seed=0):
    return np.random.default_rng(seed).integers(512, 32768, size=n, endpoint=True).astype(np.int64)


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return ""


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
            return self
        # nvidia-smi takes a while to start: wait (up to 5 s) for its first sample so that the
        # samples cover the timed region that follows
        t_end = time.time() + 5.0
        while time.time() < t_end and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.02)
        return self

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


def hbm_roof(gbs, peak, kind, kernel, nbytes):
    return {"bound": "hbm", "kernel": kernel, "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
            "frac": round(gbs / peak, 4), "peak_kind": kind, "traffic": None, "algorithmic_bytes_per_launch": nbytes}


def tensor_roof(tf, peak, kind, kernel, flops):
    return {"bound": "tensor", "kernel": kernel, "achieved": round(tf, 2), "peak": peak, "unit": "TFLOP/s",
            "frac": round(tf / peak, 4), "peak_kind": kind, "traffic": None, "algorithmic_flops_per_launch": flops}


# ------------------------------------------------------------------ serving decode (config 5)

def setup_serving(torch, lengths, slack, seed, device):
    """A context holding every sequence of `lengths` (KV rings filled to their length, random
    DeltaNet states) and one projection / output buffer per layer for up to len(lengths) rows."""
    import anelm_b200 as ab
    from anelm_b200.core import Context

    n_seqs = len(lengths)
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
    projs = []
    for t in LAYER_TYPES:
        w = FA_PROJ if t == ab.LAYER_FULL_ATTN else GDN_PROJ
        projs.append(torch.randn(n_seqs, w, generator=g, device=device, dtype=torch.float16))
    outs = [torch.empty(n_seqs, FA_OUT if t == ab.LAYER_FULL_ATTN else GDN_OUT, device=device,
                        dtype=torch.float16) for t in LAYER_TYPES]
    return ctx, projs, outs


def layer_bytes(kv_lens):
    """Algorithmic HBM bytes of ONE full-attention layer launch and ONE DeltaNet layer launch
    over sequences whose rings hold kv_lens tokens before the step."""
    n = len(kv_lens)
    fa = int((2 * np.asarray(kv_lens) * HKV * HD * 2).sum())   # K and V rows read (old tokens)
    fa += n * (FA_PROJ * 2 + FA_OUT * 2 + 2 * HKV * HD * 2)   # projection in, output, appended k/v
    gdn = n * (2 * HV * DK * DV * 4                           # state read + write
               + C_CONV * 16                                  # conv ring: 3 old inputs read + 1 written
               + GDN_PROJ * 2 + GDN_OUT * 2) + C_CONV * 16    # projection in, output; conv weights
    return fa, gdn


class ServeRun:
    """One rank's serving decode: a context over all sequences it may run and host-side ring
    lengths, so each timed loop knows its positions and bytes."""

    def __init__(self, torch, device, lengths, slack, seed):
        self.torch, self.device = torch, device
        self.ctx, self.projs, self.outs = setup_serving(torch, lengths, slack, seed, device)
        self.cur = np.asarray(lengths, np.int64).copy()  # tokens in each ring
        self.stream = torch.cuda.current_stream(device)
        self.fa_layers = [l for l, t in enumerate(LAYER_TYPES) if t == 1]

    def positions(self, ids, n_steps, pinned=False):
        """Absolute positions [n_steps][len(ids)] int32 of the next n_steps tokens of `ids`: on
        the device, or in pinned host memory for the end-to-end loop to copy in step by step."""
        pos = self.torch.from_numpy(np.stack([self.cur[ids] + k for k in range(n_steps)]).astype(np.int32))
        return pos.pin_memory() if pinned else pos.to(self.device)

    def loop(self, ids, n_steps, pos, events=False, host_io=None):
        """n_steps decode steps of the sequences `ids` at positions pos (from `positions`); returns
        per-step per-layer event pairs if `events`.  host_io = (host_in, host_out, copy_stream):
        every step first copies its positions and each layer's projection rows from pinned host
        memory and copies each layer's outputs back (the copies run on copy_stream, overlapped
        with earlier layers)."""
        torch = self.torch
        import anelm_b200 as ab

        plan = self._plan(ids)
        n = len(ids)
        comp = self.stream
        evs = []
        if host_io:
            host_in, host_out, copy = host_io
            ev_in = [torch.cuda.Event() for _ in LAYER_TYPES]
            ev_out = [torch.cuda.Event() for _ in LAYER_TYPES]
            pos_dev = torch.empty((n_steps, n), dtype=torch.int32, device=self.device)
        for k in range(n_steps):
            ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in LAYER_TYPES] \
                if events else None
            if host_io:
                copy.wait_stream(comp)
                with torch.cuda.stream(copy):
                    pos_dev[k].copy_(pos[k], non_blocking=True)
                    for l in range(N_LAYERS):
                        self.projs[l][:n].copy_(host_in[l][:n], non_blocking=True)
                        ev_in[l].record(copy)
                pk = pos_dev[k]
            else:
                pk = pos[k]
            for l, t in enumerate(LAYER_TYPES):
                if host_io:
                    comp.wait_event(ev_in[l])
                if ev:
                    ev[l][0].record(comp)
                if t == ab.LAYER_FULL_ATTN:
                    self.ctx.full_attn_decode(plan, l, self.projs[l][:n], pk, self.outs[l][:n])
                else:
                    self.ctx.deltanet_decode(plan, l, self.projs[l][:n], self.outs[l][:n])
                if ev:
                    ev[l][1].record(comp)
                if host_io:
                    ev_out[l].record(comp)
                    with torch.cuda.stream(copy):
                        copy.wait_event(ev_out[l])
                        host_out[l][:n].copy_(self.outs[l][:n], non_blocking=True)
            if host_io:
                comp.wait_stream(copy)
            if ev:
                evs.append((self.cur[ids].copy(), ev))
            self.cur[ids] += 1
        return evs

    def _plan(self, ids):
        key = tuple(int(i) for i in ids)
        if getattr(self, "_plans", None) is None:
            self._plans = {}
        if key not in self._plans:
            self._plans[key] = self.ctx.plan(list(key))
        return self._plans[key]

    def close(self):
        for p in (getattr(self, "_plans", None) or {}).values():
            p.close()
        self.ctx.close()


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def timed_serving(sr, ids, args, world, local, hbm_peak, peak_kind):
    """Warm-up, then exactly args.steps timed steps of the sequences `ids` (barrier +
    synchronize on both sides, device events, max over ranks).  Returns the measurement dict."""
    torch = sr.torch
    from anelm_b200.shard import max_over_ranks

    sr.loop(ids, args.warmup, sr.positions(ids, args.warmup))
    pos = sr.positions(ids, args.steps)
    torch.cuda.synchronize(sr.device)
    barrier(world)
    clocks = ClockSampler(local).start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(sr.device)
    t0.record(sr.stream)
    evs = sr.loop(ids, args.steps, pos, events=True)
    t1.record(sr.stream)
    torch.cuda.synchronize(sr.device)
    ck = clocks.stop()
    ms = max_over_ranks(t0.elapsed_time(t1), sr.device)
    barrier(world)
    fa_ms, gdn_ms, fa_b, gdn_b = [], [], 0, 0
    for lens, ev in evs:
        a, b = layer_bytes(lens)
        fa_b += a
        gdn_b += b
        for l, t in enumerate(LAYER_TYPES):
            (fa_ms if t == 1 else gdn_ms).append(ev[l][0].elapsed_time(ev[l][1]))
    fa_per_launch, gdn_per_launch = fa_b / args.steps, gdn_b / args.steps
    fa_gbs = fa_per_launch / (statistics.mean(fa_ms) * 1e-3) / 1e9
    gdn_gbs = gdn_per_launch / (statistics.mean(gdn_ms) * 1e-3) / 1e9
    n_fa = len(sr.fa_layers)
    return {"ms": ms, "ms_step": ms / args.steps, "clocks": ck,
            "step_gb": (n_fa * fa_per_launch + (N_LAYERS - n_fa) * gdn_per_launch) / 1e9,
            "roofline": hbm_roof(fa_gbs, hbm_peak, peak_kind, "fa_decode_kernel<256>", int(fa_per_launch)),
            "roofline_gdn": hbm_roof(gdn_gbs, hbm_peak, peak_kind, "gdn_decode_kernel", int(gdn_per_launch)),
            "kernel_ms_per_step": {"fa_decode": round(n_fa * statistics.mean(fa_ms), 3),
                                   "gdn_decode": round((N_LAYERS - n_fa) * statistics.mean(gdn_ms), 3)}}


def e2e_serving(sr, ids, args, world):
    """The same loop as the device-timed one (same calls, same per-layer events, positions
    advancing the same way) with every step's projection rows copied in from pinned host memory
    and its outputs copied back; host clock around synchronised ends, max over ranks."""
    torch = sr.torch
    from anelm_b200.shard import max_over_ranks

    n = len(ids)
    host_in = [p[:n].cpu().pin_memory() for p in sr.projs]
    host_out = [torch.empty(o[:n].shape, dtype=o.dtype).pin_memory() for o in sr.outs]
    copy = torch.cuda.Stream(sr.device)
    io = (host_in, host_out, copy)
    sr.loop(ids, 1, sr.positions(ids, 1, pinned=True), events=True, host_io=io)
    pos = sr.positions(ids, args.steps, pinned=True)
    torch.cuda.synchronize(sr.device)
    barrier(world)
    t = time.perf_counter()
    sr.loop(ids, args.steps, pos, events=True, host_io=io)
    torch.cuda.synchronize(sr.device)
    dt = max_over_ranks(time.perf_counter() - t, sr.device) / args.steps
    barrier(world)
    h2d = sum(h.numel() * h.element_size() for h in host_in) + pos[0].numel() * 4
    return dt, h2d, sum(h.numel() * h.element_size() for h in host_out)


def run_serve(args, torch, device, world, rank, local):
    import anelm_b200 as ab  # noqa: F401  (fail loudly here if the library is missing)
    from anelm_b200.shard import assign_sequences, seq_step_bytes

    hbm_peak, _, peak_kind = peaks()
    lengths = kv_lengths(GLOBAL_SEQS, 0)
    n_runs = 2 if world > 1 else 1
    slack = n_runs * (args.warmup + 2 * args.steps + 1) + 16
    sr = ServeRun(torch, device, lengths, slack, 1000 + rank)
    costs = [seq_step_bytes(int(L), 8, HKV, HD, 24, HV) for L in lengths]
    mine = assign_sequences(costs, world, rank, mode="strong")
    mine_np = np.asarray(mine, np.int64)
    m = timed_serving(sr, mine_np, args, world, local, hbm_peak, peak_kind)
    dt, h2d, d2h = e2e_serving(sr, mine_np, args, world)
    err = sr.ctx.device_error()
    assert err == 0, f"device reported status {err}"
    tok_s = GLOBAL_SEQS / (m["ms_step"] * 1e-3)
    rank_bytes = np.zeros(world)
    for r in range(world):
        rank_bytes[r] = sum(costs[i] for i in assign_sequences(costs, world, r, mode="strong"))
    result = {
        "metric": METRIC, "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(m["ms_step"], 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "BASELINE cfg5: batched serving decode, Qwen3.5-4B-shaped 32 layers (24 GDN + 8 FA)",
                   "global_batch": GLOBAL_SEQS, "seqs_on_rank0": len(mine), "kv_len": "U[512,32768] seed 0",
                   "kv_storage": "fp16 ring [slots][4][256]", "state": "fp32 [32][128][128] per seq per GDN layer",
                   "proj_io": "fp16", "Hq": HQ, "Hkv": HKV, "head_dim": HD, "rot_dim": ROT, "Hv": HV, "Hk": HK,
                   "parallelism": (f"{GLOBAL_SEQS} sequences split over {world} GPUs by greedy longest-first bin "
                                   f"packing of per-step bytes, no collective" if world > 1 else "1 GPU"),
                   "rank_bytes_imbalance": round(float(rank_bytes.max() / rank_bytes.mean()), 4),
                   "l2": f"inputs {m['step_gb']:.1f} GB/step on rank 0 > 126 MB L2 (no flush needed)"},
        "hbm_gbs_step": round(m["step_gb"] / (m["ms_step"] * 1e-3), 1),
        "roofline": m["roofline"], "roofline_gdn": m["roofline_gdn"],
        "e2e": {"value": round(GLOBAL_SEQS / dt, 1), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "steps": args.steps,
                "note": "the device-timed loop plus, every step, fp16 projection rows in from pinned host memory "
                        "and outputs back (side-stream copies); host clock, synchronised ends, max over ranks"},
        "kernel_ms_per_step": m["kernel_ms_per_step"],
        "gpu_launches": args.steps * N_LAYERS,
        "clocks": m["clocks"],
    }
    if args.traffic_json and os.path.exists(args.traffic_json):
        tr = json.load(open(args.traffic_json))
        ratio = tr.get("fa_decode_traffic_over_algorithmic")
        if ratio:
            result["roofline"]["traffic"] = int(ratio * m["roofline"]["algorithmic_bytes_per_launch"])
            result["roofline"]["traffic_kind"] = ("scaled: ncu DRAM read+write / algorithmic bytes of a "
                                                  "32-sequence capture, times this launch's algorithmic bytes")
    if world > 1:
        # weak scaling beside it: every rank decodes all 256 sequences of its own context
        w = timed_serving(sr, np.arange(GLOBAL_SEQS), args, world, local, hbm_peak, peak_kind)
        result["weak"] = {"value": round(GLOBAL_SEQS * world / (w["ms_step"] * 1e-3), 1), "unit": "tok/s",
                          "seqs_per_gpu": GLOBAL_SEQS, "ms_per_step": round(w["ms_step"], 4),
                          "roofline_frac": w["roofline"]["frac"], "roofline_gdn_frac": w["roofline_gdn"]["frac"],
                          "clocks": w["clocks"]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_reference_serving(args.cpu_seconds, threads=None, kind="reference")
    sr.close()
    return result


# ------------------------------------------------------------------ BASELINE configs 1-4

def graph_replay_us(torch, device, calls, reps_per_graph, replays):
    """Captures `calls` (a list of closures, one launch each) into one CUDA graph and returns the
    device time per call over `replays` replays (after a warm-up replay)."""
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for c in calls:
                c()
    torch.cuda.synchronize(device)
    graph.replay()
    torch.cuda.synchronize(device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(replays):
        graph.replay()
    t1.record()
    torch.cuda.synchronize(device)
    us = t0.elapsed_time(t1) * 1e3 / (replays * len(calls))
    del graph
    return us


def wl_decode_b1(args, torch, device, which):
    """BASELINE config 1 (attention decode, 0.8B shape, ring of 2048 fp16) or config 2 (DeltaNet
    decode, 16 heads, fp32 state): the single-sequence entry point, one call per token.  The
    timed calls rotate over `n_copies` independent sequences whose data together exceed the 126 MB
    L2, so every call streams its KV / state from HBM; calls replay from a CUDA graph."""
    import anelm_b200 as ab
    from anelm_b200.core import Context

    hbm_peak, _, peak_kind = peaks()
    rng = np.random.default_rng(0)
    g = torch.Generator(device=device)
    g.manual_seed(0)
    if which == "fa":
        n_copies = 64                                        # 64 x 4.2 MB = 268 MB
        ctx = Context(device=device.index or 0, layer_types=[ab.LAYER_FULL_ATTN], max_seqs=n_copies,
                      kv_capacity=2048)
        ctx.set_full_attn_weights(0, (1 + 0.02 * rng.standard_normal(256)).astype(np.float32),
                                  (1 + 0.02 * rng.standard_normal(256)).astype(np.float32))
        for s in range(n_copies):
            kv = torch.randn(2048, 2, 256, generator=g, device=device, dtype=torch.float16)
            ctx.kv_write(0, s, 0, kv, kv.flip(0).contiguous())
            ctx.kv_set_meta(0, s, 2048, 0)
        projs = torch.randn(n_copies, ctx.fa_proj_dim, generator=g, device=device, dtype=torch.float16)
        outs = torch.empty(n_copies, ctx.fa_out_dim, device=device, dtype=torch.float16)
        calls = [(lambda s=s: ctx.full_attn_from_proj(0, s, projs[s], 3000, outs[s])) for s in range(n_copies)]
        nbytes = 2 * 2048 * 2 * 256 * 2 + ctx.fa_proj_dim * 2 + ctx.fa_out_dim * 2 + 2 * 2 * 256 * 2
        metric, kname = "attention decode tok/s (cfg1, 0.8B shape, KV 2048 fp16, batch 1)", "fa_decode_kernel<256,1>"
    else:
        n_copies = 128                                       # 128 x 2.3 MB = 295 MB
        ctx = Context(device=device.index or 0, layer_types=[ab.LAYER_LINEAR_ATTN], max_seqs=n_copies)
        C = ctx.conv_channels
        ctx.set_deltanet_weights(0, (0.5 * rng.standard_normal((C, 4))).astype(np.float16).astype(np.float32),
                                 np.ones(16, np.float32), np.zeros(16, np.float32), np.ones(128, np.float32))
        for s in range(n_copies):
            ctx.deltanet_state_write(0, s, (0.1 * torch.randn(16, 128, 128, generator=g, device=device)).contiguous())
        projs = torch.randn(n_copies, ctx.gdn_proj_dim, generator=g, device=device, dtype=torch.float16)
        outs = torch.empty(n_copies, ctx.gdn_out_dim, device=device, dtype=torch.float16)
        calls = [(lambda s=s: ctx.deltanet_from_proj(0, s, projs[s], outs[s])) for s in range(n_copies)]
        nbytes = 2 * 16 * 128 * 128 * 4 + C * 16 + C * 16 + ctx.gdn_proj_dim * 2 + ctx.gdn_out_dim * 2
        metric, kname = "DeltaNet decode tok/s (cfg2, 16 heads, fp32 state, batch 1)", "gdn_decode_kernel<1,8,128>"
    for c in calls:  # the first call per sequence builds its batch-1 plan (allocations: not inside a capture)
        c()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index or 0).start()
    replays = 20
    us = graph_replay_us(torch, device, calls, len(calls), replays)
    ck = clocks.stop()
    err = ctx.device_error()
    ctx.close()
    assert err == 0, f"device reported status {err}"
    gbs = nbytes / (us * 1e-6) / 1e9
    cpu = None if args.no_cpu_baseline else cpu_reference_decode_b1(which, args.cpu_seconds_wl)
    return {"metric": metric, "value": round(1e6 / us, 1), "unit": "tok/s", "us_per_call": round(us, 3),
            "calls_timed": replays * len(calls), "roofline": hbm_roof(gbs, hbm_peak, peak_kind, kname, nbytes),
            "l2": f"calls rotate over {n_copies} sequences ({n_copies * nbytes >> 20} MB > 126 MB L2); CUDA graph",
            "clocks": ck, "cpu_baseline": cpu, "gpu_launches": replays * len(calls)}


def wl_fa_prefill(args, torch, device, B, n=4096, steps=10):
    """causal full-attention prefill, Qwen3.5-4B shape, n tokens per sequence,
    B sequences, bf16 inputs; the whole call (prep: QK-norm, RoPE, ring append; attention)."""
    import anelm_b200 as ab
    from anelm_b200.core import Context

    _, tpeak, tkind = peaks()
    rng = np.random.default_rng(0)
    g = torch.Generator(device=device)
    g.manual_seed(0)
    ctx = Context(device=device.index or 0, layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=HQ, num_kv_heads=HKV,
                  head_dim=HD, rot_dim=ROT, rope_theta=1e7, max_seqs=B, kv_capacity=n)
    ctx.set_full_attn_weights(0, (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32),
                              (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32))
    plan = ctx.plan(list(range(B)))
    proj = torch.randn(B, n, FA_PROJ, generator=g, device=device).to(torch.bfloat16)
    out = torch.empty(B, n, FA_OUT, device=device, dtype=torch.bfloat16)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    for _ in range(max(3, args.warmup)):
        ctx.reset(-1)
        ctx.full_attn_prefill(plan, 0, proj, 0, out)
    torch.cuda.synchronize(device)
    times = []
    clocks = ClockSampler(device.index or 0).start()
    for _ in range(steps):
        ctx.reset(-1)      # synchronous; outside the timed region
        flush_and_cover(torch, flush)  # the B = 1 inputs (84 MB) would otherwise sit in L2
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        ctx.full_attn_prefill(plan, 0, proj, 0, out)
        t1.record()
        torch.cuda.synchronize(device)
        times.append(t0.elapsed_time(t1))
    ck = clocks.stop()
    err = ctx.device_error()
    plan.close()
    ctx.close()
    assert err == 0, f"device reported status {err}"
    ms = statistics.median(times)
    flops = 4.0 * n * n * HD * HQ / 2 * B  # causal: half of the S x S score / PV work
    tf = flops / (ms * 1e-3) / 1e12
    return {"metric": f"causal prefill attention TFLOP/s (cfg3, Qwen3.5-4B shape, B={B}, S={n})",
            "value": round(tf, 1), "unit": "TFLOP/s", "ms": round(ms, 4), "steps": steps,
            "roofline": tensor_roof(tf, tpeak, tkind, "fa_prefill_prep_bulk_kernel + fa_prefill_kernel (whole call)",
                                    flops),
            "timed": "whole call: prep (QK-norm, RoPE, fp16 Q/K/V, sigmoid gate, ring append) + attention",
            "l2": "256 MB buffer written before each timed call (then a fixed spin kernel covers the host's enqueue)",
            "clocks": ck,
            "cpu_baseline": None if args.no_cpu_baseline else cpu_reference_prefill(B, n, args.cpu_seconds_wl, flops),
            "gpu_launches": 3 * steps}


def wl_gdn_prefill(args, torch, device, B=1, T=8192, steps=10):
    """the chunked gated delta rule, Hv 32 / Hk 16, dk = dv = 128, seq 8192,
    batch 1; bf16 q / k / v N(0, 1) with L2-normalised k, log g ~ U(-0.1, 0), beta ~ U(0, 1)."""
    from anelm_b200.core import gated_delta_chunked
    import anelm_b200 as ab

    hbm_peak, tpeak, tkind = peaks()
    Hk, Hv = 16, 32
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
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)

    def call():
        gated_delta_chunked(q, k, v, lg, beta, state, ab.DELTA_CPUOPS, y=y, workspace=ws)

    for _ in range(max(3, args.warmup)):
        call()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index or 0).start()
    times = []
    for _ in range(steps):
        flush_and_cover(torch, flush)  # inputs (24 MB) would otherwise stay in L2 between iterations
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
    roof = tensor_roof(tf, tpeak, tkind, "gdn_pf_chunk + gdn_pf_chain (whole call; q / k / v read in place)",
                       flops)
    roof.update({"hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 4), "algorithmic_bytes": nbytes})
    return {"metric": f"chunked Gated DeltaNet prefill TFLOP/s (cfg4, Hv 32 / Hk 16, d 128, S={T}, B={B})",
            "value": round(tf, 2), "unit": "TFLOP/s", "ms": round(ms, 4), "steps": steps, "roofline": roof,
            "l2": "256 MB buffer written before each timed call (then a fixed spin kernel covers the host's enqueue)",
            "clocks": ck,
            "cpu_baseline": (None if args.no_cpu_baseline else
                             cpu_reference_gdn_chunk(T, B, Hk, Hv, flops, args.cpu_seconds_wl)),
            "gpu_launches": 2 * steps}  # bf16 inputs on 16-byte boundaries: no pack launch


def gdn_chunk_flops(T, Hv, B=1, C=64, dk=128, dv=128):
    """Algorithmic FLOPs of the chunked delta rule: per chunk and value head 2C^2(3dk + 2dv)
    (K K^T, Q K^T, W, U, M D) + 6 C dk dv (W S, Q S, K^T D)."""
    n_chunks = (T + C - 1) // C
    return float(2 * C * C * (3 * dk + 2 * dv) + 6 * C * dk * dv) * n_chunks * Hv * B


def wl_prefill_sharded(args, torch, device, world, rank, which):
    """Configs 3 (B = 1) and 4 split over the ranks for a single long sequence: causal prefill by
    KV-head group (shard.head_shard, parallel.sharded_full_attn_prefill) or the chunked delta rule by
    value head (shard.value_head_shard); each rank computes its heads, then one all-gather gives every
    rank the full output.  Each rank's input columns are selected before the timed region (in a model
    they come from that rank's share of the in-projection).  Time = max over ranks of the whole step;
    the all-gather's share is timed with events around it."""
    import torch.distributed as dist

    import anelm_b200 as ab
    from anelm_b200.core import Context, gated_delta_chunked
    from anelm_b200.parallel import PeerOutputs, fused_sharded_full_attn_prefill, local_proj_columns
    from anelm_b200.shard import gather_heads, head_shard, max_over_ranks, value_head_shard

    _, tpeak, tkind = peaks()
    g = torch.Generator(device=device)
    g.manual_seed(0)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    if which == "fa":
        n = args.prefill_len
        rng = np.random.default_rng(0)
        qh, kvh = head_shard(HQ, HKV, world, rank)
        ctx = Context(device=device.index or 0, layer_types=[ab.LAYER_FULL_ATTN], num_q_heads=len(qh),
                      num_kv_heads=len(kvh), head_dim=HD, rot_dim=ROT, rope_theta=1e7, max_seqs=1, kv_capacity=n)
        ctx.set_full_attn_weights(0, (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32),
                                  (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32))
        plan = ctx.plan([0])
        proj = torch.randn(n, FA_PROJ, generator=g, device=device).to(torch.bfloat16)
        cols = local_proj_columns(HQ, HKV, HD, qh, kvh).to(device)
        local = proj.index_select(1, cols).unsqueeze(0).contiguous()
        out_local = torch.empty(1, n, len(qh) * HD, device=device, dtype=torch.bfloat16)

        peers = PeerOutputs((1, n, HQ * HD), torch.bfloat16, device)

        def compute():
            if args.nccl_gather:
                ctx.full_attn_prefill(plan, 0, local, 0, out_local)
            else:  # the gather is inside: every rank's epilogue stores into every rank's buffer
                fused_sharded_full_attn_prefill(ctx, plan, 0, local, peers, HQ, HKV, HD)

        def collect():
            return gather_heads(out_local[0], HQ, HKV, HD) if args.nccl_gather else peers.local

        def before():
            ctx.reset(-1)

        flops = 4.0 * n * n * HD * HQ / 2
        metric = (f"head-sharded causal prefill TFLOP/s (cfg3 B=1, S={n}, {world} GPUs, "
                  f"{'NCCL all-gather' if args.nccl_gather else 'all-gather fused into the attention epilogue'})")
        shard = f"q heads {qh[0]}-{qh[-1]}, kv heads {kvh}"
        gathered = n * HQ * HD * 2
    else:
        T, Hk, Hv = args.gdn_len, 16, 32
        keys, vals = value_head_shard(Hk, Hv, world, rank)
        k0, k1, v0, v1 = keys[0], keys[-1] + 1, vals[0], vals[-1] + 1
        q = torch.randn(1, T, Hk, 128, generator=g, device=device).to(torch.bfloat16)
        k = torch.randn(1, T, Hk, 128, generator=g, device=device)
        k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
        v = torch.randn(1, T, Hv, 128, generator=g, device=device).to(torch.bfloat16)
        lg = -0.1 * torch.rand(1, T, Hv, generator=g, device=device)
        beta = torch.rand(1, T, Hv, generator=g, device=device)
        ql, kl = q[:, :, k0:k1].contiguous(), k[:, :, k0:k1].contiguous()
        vl, lgl, bl = v[:, :, v0:v1].contiguous(), lg[:, :, v0:v1].contiguous(), beta[:, :, v0:v1].contiguous()
        state = torch.zeros(1, v1 - v0, 128, 128, device=device)
        y = torch.empty(1, T, v1 - v0, 128, device=device, dtype=torch.bfloat16)
        ws = torch.empty(ab.lib().anelm_gated_delta_chunked_workspace_bytes(1, T, k1 - k0, v1 - v0),
                         dtype=torch.uint8, device=device)
        parts = torch.empty(world * T, (v1 - v0) * 128, device=device, dtype=torch.bfloat16)

        def compute():
            gated_delta_chunked(ql, kl, vl, lgl, bl, state, ab.DELTA_CPUOPS, y=y, workspace=ws)

        def collect():
            dist.all_gather_into_tensor(parts, y.view(T, -1))
            return parts.view(world, T, -1).transpose(0, 1).reshape(T, -1)

        def before():
            pass

        flops = gdn_chunk_flops(T, Hv, 1)
        metric = f"value-head-sharded chunked DeltaNet prefill TFLOP/s (cfg4, S={T}, {world} GPUs)"
        shard = f"value heads {v0}-{v1 - 1}, key heads {k0}-{k1 - 1}"
        gathered = T * Hv * 128 * 2
    for _ in range(max(3, args.warmup)):
        before()
        compute()
        collect()
    torch.cuda.synchronize(device)
    steps = max(args.steps, 5)
    tot, gat = [], []
    clocks = ClockSampler(device.index or 0).start()
    for _ in range(steps):
        before()
        torch.cuda.synchronize(device)
        dist.barrier()
        flush_and_cover(torch, flush)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        compute()
        e1.record()
        collect()
        e2.record()
        torch.cuda.synchronize(device)
        tot.append(max_over_ranks(e0.elapsed_time(e2), device))
        gat.append(max_over_ranks(e1.elapsed_time(e2), device))
    ck = clocks.stop()
    ms = statistics.median(tot)
    if which == "fa":
        peers.close()
        plan.close()
        ctx.close()
    tf = flops / (ms * 1e-3) / 1e12
    return {"metric": metric, "value": round(tf, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 in, fp32 accumulate", "data": "synthetic",
            "config": {"workload": metric, "rank0_shard": shard,
                       "l2": "256 MB buffer written before each step (then a fixed spin kernel covers the host's enqueue)",
                       "parallelism": f"heads over {world} GPUs, one all-gather of the output"},
            "roofline": tensor_roof(tf / world, tpeak, tkind, "per GPU, whole step", flops / world),
            "allgather": {"ms": round(statistics.median(gat), 4), "share": round(statistics.median(gat) / ms, 4),
                          "form": ("NCCL all_gather_into_tensor after the prefill" if which != "fa" or args.nccl_gather
                                   else "inside the prefill kernel (peer TMA stores); timed here: nothing left"),
                          "bytes_gathered": gathered,
                          "gbs_per_gpu_in": round(gathered * (world - 1) / world / (statistics.median(gat) * 1e-3) / 1e9,
                                                  1)},
            "clocks": ck, "gpu_launches": steps * (3 if which == "fa" else 2)}


def run_workloads(args, torch, device):
    out = {}
    for name, fn in (("cfg1", lambda: wl_decode_b1(args, torch, device, "fa")),
                     ("cfg2", lambda: wl_decode_b1(args, torch, device, "gdn")),
                     ("cfg3_b1", lambda: wl_fa_prefill(args, torch, device, 1)),
                     ("cfg3_b8", lambda: wl_fa_prefill(args, torch, device, 8)),
                     ("cfg4", lambda: wl_gdn_prefill(args, torch, device))):
        out[name] = fn()
        torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ the steps next to the core

def run_proj(args, torch, device):
    """The steps next to the core (widening beyond the core): "proj" = the in- and out-projection
    GEMMs of one attention and one DeltaNet decode layer of the Qwen3.5-4B shape for `--seqs` rows
    (anelm_gemm_bf16); "lm_head" = the in-model top-32 LM head over the 248,320-token vocabulary
    for `--seqs` rows (anelm_lm_head_topk).  bf16 N(0,1) activations, N(0, 1/hidden) weights."""
    from anelm_b200.core import gemm_bf16, lm_head_topk

    hbm_peak, tpeak, tpeak_kind = peaks()
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
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index or 0).start()
    times = []
    for _ in range(args.steps):
        # weights would otherwise stay in L2 between iterations; the longer spin covers the calls'
        # host work (tensor maps, workspace set-up, several launches)
        flush_and_cover(torch, flush, 3 * ENQUEUE_COVER_CYCLES)
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
    roof = (tensor_roof(tf, tpeak, tpeak_kind, kernel, flops) if bound == "tensor" else
            hbm_roof(gbs, hbm_peak, tpeak_kind, kernel, nbytes))
    # CPU baseline: numpy (BLAS) on an 8-row sample of the same products (the reference runs them
    # on the ANE, so there is no reference CPU code for this step)
    rows = min(8, n)
    cpu_t = 0.0
    if not args.no_cpu_baseline:
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
    return {
        "metric": metric, "value": round(tf, 2), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 in, fp32 accumulate", "data": "synthetic",
        "config": dict(cfg, l2="256 MB buffer written between timed iterations"),
        "hbm_gbs_step": round(gbs, 1), "roofline": roof,
        "cpu_baseline": {"value": round(cpu_tf, 6) if cpu_tf else None, "unit": "TFLOP/s",
                         "cores": os.cpu_count(), "kind": "port",
                         "sample": f"numpy fp32 matmul on {rows} rows" +
                                   (" of 1/8 of the vocabulary, scaled" if args.workload == "lm_head" else "")},
        "clocks": ck, "gpu_launches": launches * args.steps}


def run_gdn_layer(args, torch, device):
    """One DeltaNet decode layer of the config-5 shape over `--seqs` sequences (the kernel of the
    serving step on its own, a few hundred MB of state: the size for an ncu capture)."""
    import anelm_b200 as ab
    from anelm_b200.core import Context

    hbm_peak, _, peak_kind = peaks()
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
    nbytes = layer_bytes(np.full(n, 1))[1]              # same accounting as the serving step
    gbs = nbytes / (ms * 1e-3) / 1e9
    plan.close()
    ctx.close()
    return {"metric": "DeltaNet decode layer GB/s (config-5 shape, one layer)", "value": round(gbs, 1),
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"one DeltaNet layer, {n} sequences", "l2": f"state {n * HV * DK * DV * 4 >> 20} MB"},
            "roofline": hbm_roof(gbs, hbm_peak, peak_kind, "gdn_decode_kernel", nbytes),
            "gpu_launches": args.steps}


def single_line(args, wl):
    """The one-workload form of a configs 1-4 entry, as a full bench line."""
    line = {"metric": wl["metric"], "value": wl["value"], "unit": wl["unit"], "n_gpus": 1, "steps": wl.get("steps"),
            "warmup": args.warmup, "ms_per_step": wl.get("ms", wl.get("us_per_call", 0) / 1e3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "see metric",
            "data": "synthetic", "config": {"workload": args.workload, "l2": wl["l2"]}}
    line.update({k: v for k, v in wl.items() if k not in line and k not in ("metric", "value", "unit")})
    return line


def run_gpu(args):
    import torch
    import torch.distributed as dist

    rank, world, local = env_rank()
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    try:
        if args.workload == "serve":
            result = run_serve(args, torch, device, world, rank, local)
            if world == 1 and not args.no_workloads:
                result["workloads"] = run_workloads(args, torch, device)
                result["gpu_launches"] += sum(w["gpu_launches"] for w in result["workloads"].values())
        elif args.workload in ("fa_b1", "gdn_b1"):
            result = single_line(args, wl_decode_b1(args, torch, device, args.workload[:-3]))
        elif args.workload in ("fa_prefill", "gdn_prefill") and world > 1:
            result = wl_prefill_sharded(args, torch, device, world, rank, args.workload[:-8])
        elif args.workload == "fa_prefill":
            result = single_line(args, wl_fa_prefill(args, torch, device, args.prefill_batch, args.prefill_len,
                                                     args.steps))
        elif args.workload == "gdn_prefill":
            result = single_line(args, wl_gdn_prefill(args, torch, device, args.prefill_batch, args.gdn_len,
                                                      args.steps))
        elif args.workload in ("proj", "lm_head"):
            result = run_proj(args, torch, device)
        else:
            result = run_gdn_layer(args, torch, device)
        if rank == 0:
            print(json.dumps(result), flush=True)
    except BaseException:
        if world > 1:
            dist.destroy_process_group()  # no barrier: the other ranks learn of it by their own timeout
        raise
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------ CPU reference (oracle/_ref)

def _ref_kind():
    from oracle import pyoracle as po
    return "ref_fast" if po.available("ref_fast") else "oracle"


def cpu_reference_serving(seconds: float, threads=None, kind="reference"):
    """The reference CPU attention core (oracle/_ref/libref_core_fast.so: core/cpu_ops.cpp,
    unmodified, + the qwen3_5.cpp glue restated) on a bounded sample of the serving workload:
    one host thread per sampled sequence, each decoding token by token through all 32 layers
    (fp32 KV ring of its length, fp32 DeltaNet state).  The sample takes the sequences at evenly
    spaced quantiles of the 256-sequence length draw, so its mean KV length matches the
    workload's.  Returns tokens/s over the sample (all threads together)."""
    from oracle import pyoracle as po

    lib_kind = _ref_kind()
    threads = threads or max(1, os.cpu_count() or 1)
    shape = po.make_shape(num_q_heads=HQ, num_kv_heads=HKV, head_dim=HD, rot_dim=ROT, rope_theta=1e7,
                          lin_num_key_heads=HK, lin_num_val_heads=HV)
    var = po.make_variant()
    population = np.sort(kv_lengths(GLOBAL_SEQS, 0))
    pick = ((np.arange(threads) + 0.5) * GLOBAL_SEQS / threads).astype(int).clip(0, GLOBAL_SEQS - 1)
    lengths = population[pick]
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
    return {"value": round(toks / wall, 3), "unit": "tok/s", "cores": threads, "kind": kind,
            "sample_mean_kv": round(float(lengths.mean()), 1), "workload_mean_kv": round(float(population.mean()), 1),
            "sample": (f"{threads} sequences at evenly spaced quantiles of the workload's 256-sequence U[512,32768] "
                       f"draw (mean KV {lengths.mean():.0f} vs {population.mean():.0f}), {toks} tokens through all "
                       f"32 layers, fp32 KV/state, one thread per sequence, {wall:.1f} s wall; "
                       f"lib={os.path.basename(po.LIBS[lib_kind])}; cpu={cpu_model()}; nproc={os.cpu_count()}")}


def cpu_reference_decode_b1(which, seconds):
    """The reference core (oracle/_ref/libref_core_fast.so) on configs 1 / 2: one sequence, one
    thread (the reference's core is single-threaded and batch 1 has nothing else to spread),
    token by token for up to `seconds`."""
    from oracle import pyoracle as po

    kind = _ref_kind()
    P = po.P
    rng = np.random.default_rng(0)
    if which == "fa":
        shape = po.make_shape()
        qn = (1 + 0.02 * rng.standard_normal(256)).astype(np.float32)
        k = rng.standard_normal((2048, 2, 256)).astype(np.float32)
        v = rng.standard_normal((2048, 2, 256)).astype(np.float32)
        ln, st = ctypes.c_int(2048), ctypes.c_int(0)
        rope = po.rope_table(4096, 64, 1e7)
        proj = rng.standard_normal(8 * 512 + 2 * 2 * 256).astype(np.float32)
        pbuf, out, tmp = np.empty_like(proj), np.zeros(8 * 256, np.float32), np.zeros(256, np.float32)
        f = po.fn(kind, "full_attn_from_proj")

        def step(i):
            pbuf[:] = proj
            f(ctypes.byref(shape), ctypes.byref(po.make_variant()), P(qn), P(qn), P(k), P(v), ctypes.byref(ln),
              ctypes.byref(st), 2048, P(rope[0]), P(rope[1]), 4096, P(pbuf), 3000 + i, P(out), P(tmp))
        what = "ring of 2048 (full, sliding), 8/2 heads"
    else:
        shape = po.make_shape(lin_num_key_heads=16, lin_num_val_heads=16)
        C = 6144
        cw = (0.5 * rng.standard_normal((C, 4))).astype(np.float16).astype(np.float32)
        A, dtb, nw = np.ones(16, np.float32), np.zeros(16, np.float32), np.ones(128, np.float32)
        s = po.DeltaState.zeros(shape)
        s.ssm[:] = (0.1 * rng.standard_normal(s.ssm.shape)).astype(np.float32)
        proj = rng.standard_normal(C + 16 * 128 + 32).astype(np.float32)
        out, scratch = np.zeros(16 * 128, np.float32), np.zeros(2 * C + 16 * 128, np.float32)
        cp = ctypes.c_int(0)
        f = po.fn(kind, "deltanet_from_proj")

        def step(i):
            f(ctypes.byref(shape), ctypes.byref(po.make_variant()), P(cw), P(A), P(dtb), P(nw), P(s.ssm), P(s.conv),
              ctypes.byref(cp), P(proj), P(out), P(scratch))
        what = "16/16 heads, fp32 state 128x128 per head"
    step(0)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds and n < 100000:
        step(n)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 2), "unit": "tok/s", "cores": 1, "kind": "reference" if kind == "ref_fast" else "port",
            "sample": f"{n} successive tokens, {what}, {dt:.1f} s; lib={os.path.basename(po.LIBS[kind])}; "
                      f"cpu={cpu_model()}"}


def cpu_reference_prefill(B, n, seconds, flops):
    """The reference's prefill of config 3 is its per-token loop (qwen3_5.cpp:1205-1217): token t
    runs forward_full_attn_from_proj over a ring holding t keys.  Sample: tokens at evenly spaced
    positions of the prompt, each timed over a ring filled to that position; the prompt's time is
    the sample mean times n.  One thread per sequence, B sequences at once."""
    from oracle import pyoracle as po

    kind = _ref_kind()
    P = po.P
    shape = po.make_shape(num_q_heads=HQ, num_kv_heads=HKV, head_dim=HD, rot_dim=ROT, rope_theta=1e7)
    rope = po.rope_table(4096, ROT, 1e7)
    f = po.fn(kind, "full_attn_from_proj")
    K = 16

    def worker(b):
        rng = np.random.default_rng(b)
        qn = (1 + 0.02 * rng.standard_normal(HD)).astype(np.float32)
        k = rng.standard_normal((n, HKV, HD)).astype(np.float32)
        v = rng.standard_normal((n, HKV, HD)).astype(np.float32)
        proj = rng.standard_normal(FA_PROJ).astype(np.float32)
        pbuf, out, tmp = np.empty_like(proj), np.zeros(FA_OUT, np.float32), np.zeros(HD, np.float32)
        total, done, t_end = 0.0, 0, time.perf_counter() + seconds
        for i in range(K):
            p = int((i + 0.5) * n / K)
            ln, st = ctypes.c_int(p), ctypes.c_int(0)
            pbuf[:] = proj
            t0 = time.perf_counter()
            f(ctypes.byref(shape), ctypes.byref(po.make_variant()), P(qn), P(qn), P(k), P(v), ctypes.byref(ln),
              ctypes.byref(st), n, P(rope[0]), P(rope[1]), 4096, P(pbuf), p, P(out), P(tmp))
            total += time.perf_counter() - t0
            done += 1
            if time.perf_counter() > t_end:
                break
        return total / done * n, done

    with ThreadPoolExecutor(max_workers=B) as ex:
        res = list(ex.map(worker, range(B)))
    wall = max(r[0] for r in res)   # B sequences on B threads: the slowest one's prompt time
    return {"value": round(flops / wall / 1e12, 6), "unit": "TFLOP/s", "cores": B,
            "kind": "reference" if kind == "ref_fast" else "port", "est_prompt_s": round(wall, 2),
            "sample": (f"{res[0][1]} tokens per sequence at evenly spaced positions of the {n}-token prompt "
                       f"(forward_full_attn_from_proj over a ring filled to that position), mean x {n} = the "
                       f"per-token prefill loop's time; {B} thread(s); lib={os.path.basename(po.LIBS[kind])}")}


def cpu_reference_gdn_chunk(T, B, Hk, Hv, flops, seconds):
    """The reference delta-rule step (core/cpu_ops.cpp ssm_step via oracle/_ref) over a token sample
    of the config-4 workload, one host thread; scaled to the workload's tokens."""
    from oracle import pyoracle as po

    kind = _ref_kind()
    rng = np.random.default_rng(1)
    T_s = 64
    q = rng.standard_normal((T_s, Hk, 128)).astype(np.float32)
    k = q / np.linalg.norm(q, axis=-1, keepdims=True)
    v = rng.standard_normal((T_s, Hv, 128)).astype(np.float32)
    lg = (-0.1 * rng.random((T_s, Hv))).astype(np.float32)
    beta = rng.random((T_s, Hv)).astype(np.float32)
    st = np.zeros((Hv, 128, 128), np.float32)
    t0 = time.perf_counter()
    po.gated_delta_tokens(kind, q, k, v, lg, beta, st, 0)
    sec_tok = (time.perf_counter() - t0) / T_s
    return {"value": round(flops / (sec_tok * T * B) / 1e12, 6), "unit": "TFLOP/s", "cores": 1,
            "kind": "reference" if kind == "ref_fast" else "port",
            "sample": f"{T_s} tokens x {Hv} value heads of the token recurrence (ssm_step), scaled to the "
                      f"workload's {T * B} tokens and its algorithmic FLOPs"}


def run_reference(args):
    rank, world, local = env_rank()
    if rank != 0:
        return
    cb = cpu_reference_serving(args.cpu_seconds, threads=None, kind="reference")
    print(json.dumps({
        "impl": "reference", "metric": METRIC,
        "value": cb["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": None, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "BASELINE cfg5: batched serving decode, Qwen3.5-4B-shaped 32 layers (24 GDN + 8 FA)",
                   "global_batch": GLOBAL_SEQS, "kv_len": "U[512,32768] seed 0",
                   "note": "the host's cores run the reference CPU core; the GPU count does not change it"},
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
    ap.add_argument("--seqs", type=int, default=256, help="rows for the proj / lm_head / gdn_layer workloads")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--cpu-seconds-wl", type=float, default=3.0, help="CPU sample per configs 1-4 entry")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-workloads", action="store_true", help="skip the configs 1-4 entries of the default line")
    ap.add_argument("--nccl-gather", action="store_true",
                    help="head-sharded prefill: all-gather with NCCL after the kernel instead of inside it")
    ap.add_argument("--traffic-json", default=os.path.join(REPO, "profiles", "traffic.json"))
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
