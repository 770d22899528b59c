#!/usr/bin/env python
"""Benchmark of the LUCID attention hot path on B200.

Metric: LUCID attention fwd+bwd TFLOP/s and fraction of the
dense-BF16 peak at N=32K, with the overhead against plain causal attention
of the same shape.

Workload per GPU (one step): one LUCID attention layer forward + backward,
bf16, B=1, H=32 (MHA), N=32768, D=128, causal; Q ~ N(0,1)/sqrt(128),
K, V, dO ~ N(0,1) (seeded synthetic data, per rank).  Every input tensor is
268 MB, larger than the 126 MB L2, so no flush is needed between steps.

Algorithmic FLOPs per (batch, head): 14 N^2 D
  attention fwd 2 N^2 D + bwd 5 N^2 D, LUCID solve fwd 2 N^2 D + bwd 5 N^2 D.

Multi-GPU (torchrun): the workload is the whole job and is split, not
replicated: rank r of W takes the contiguous (batch, kv head) pairs
[r B Hkv / W, (r + 1) B Hkv / W) (all query heads of those kv heads), with no
data-path collective; the step time is the max over ranks and `value` the whole
job's algorithmic work over it (strong scaling).  Every (batch, head) slice is
drawn from its own seeded generator, so the data do not depend on the GPU count.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--config path measures the LUCID-Path op instead (
parallel_lucid_path_attention fwd+bwd, B=2, H=16, T=16384, K=V=128, bf16,
q = k; k, v ~ N(0,1), w ~ N(0,1) L2-normalised, beta = 2 sigmoid(N(0,1)),
dO ~ N(0,1)), with the algorithmic count 14 T^2 K per (batch, head).
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

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "LUCID attn fwd+bwd TFLOP/s & % BF16 peak at 32K; overhead vs causal attn"
CONFIGS = {
    # name: (B per rank, H, N, D, q_scale)
    "32k": (1, 32, 32768, 128, 128 ** -0.5),
    "cfg2": (4, 32, 4096, 128, 128 ** -0.5),
    "small": (1, 8, 4096, 128, 128 ** -0.5),
    "8k": (1, 32, 8192, 128, 128 ** -0.5),   # profiling case (about 1.5 GB on the device)
    "32k-gqa": (1, 32, 32768, 128, 128 ** -0.5),
    # one rank's share of the 32K job at 8 GPUs (4 of its 32 heads), measured on one GPU:
    # the stages whose per-head dependency chains set the 8-GPU step time
    "32k-r8": (1, 4, 32768, 128, 128 ** -0.5),
}
# kv heads of the grouped-query configurations (the others are MHA)
KV_HEADS = {"32k-gqa": 4}


def flops_per_step(B, H, N, D, Hkv=None):
    """Algorithmic flops of one LUCID fwd+bwd: the attention's 7 N^2 D per query head
    and the solve's 7 N^2 D per kv head (14 N^2 D per head without grouping)."""
    Hkv = H if Hkv is None else Hkv
    return 7.0 * N * N * D * B * (H + Hkv)


def stage_units(H, Hkv):
    """Per stage: its algorithmic GEMM work in units of N^2 D per batch element (a causal
    GEMM over the lower triangle is N^2 D flops per head).  The attention stages run per
    query head, the solve stages per kv head; the row passes' 1 excludes the S and dP
    recomputation of the recomputing schedule, which is executed but not algorithmic."""
    return {"solve_fwd": 2 * Hkv, "attn_fwd": 2 * H, "attn_bwd": 4 * H, "attn_bwd_row": 1 * H,
            "solve_bwd": 4 * Hkv, "solve_bwd_row": 1 * Hkv}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), \
            float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi, during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        # nvidia-smi takes a moment to start: begin the timed region only once
        # it has written its first sample (short regions would see none)
        t0 = time.time()
        while time.time() - t0 < 5.0:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.02)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        loaded = [s for s in sm if s > 0.5 * max(sm)] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's torch path (restated in oracle/torch_ref.py)
# ---------------------------------------------------------------------------
def cpu_reference_sample(N: int, D: int, seed: int = 0):
    """One LUCID layer fwd+bwd for one (batch, head) on the host cores, fp32
    (the reference's solve_triangular path has no bf16 CPU kernel)."""
    import torch

    from oracle import torch_ref

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, 1, N, D, generator=g) * D ** -0.5
    k = torch.randn(1, 1, N, D, generator=g)
    v = torch.randn(1, 1, N, D, generator=g)
    do = torch.randn(1, N, 1, D, generator=g)
    t0 = time.perf_counter()
    torch_ref.lucid_fwd_bwd(q, k, v, do)
    return time.perf_counter() - t0


def cpu_baseline(N_cpu: int, D: int, reps: int = 1):
    cpu_reference_sample(1024, D)  # warm-up (thread pool, allocator)
    times = [cpu_reference_sample(N_cpu, D, seed=i) for i in range(reps)]
    t = statistics.median(times)
    fl = flops_per_step(1, 1, N_cpu, D)
    return {"value": fl / t / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"1 (batch, head) of the workload at N={N_cpu}, D={D}, fp32, fwd+bwd via "
                      f"oracle/torch_ref.py (reference torch path), median of {reps}",
            "seconds_per_sample": t}


def reference_arm(args):
    """--impl reference: the reference's CPU path on the host cores, same
    metric/config; rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.config == "path":
        return path_reference_arm(args)
    if args.config == "cp128k":
        return cp_reference_arm(args)
    if args.config == "prefill":
        return prefill_reference_arm(args)
    if args.config == "decode":
        return decode_reference_arm(args)
    B, H, N, D, _ = CONFIGS[args.config]
    Hkv = KV_HEADS.get(args.config, H)
    heads = f"H{H}" if Hkv == H else f"Hq{H} Hkv{Hkv}"
    n_cpu = args.cpu_n
    cpu_reference_sample(1024, D)
    for _ in range(args.warmup):
        cpu_reference_sample(n_cpu, D)
    times = [cpu_reference_sample(n_cpu, D, seed=i) for i in range(args.steps)]
    t = statistics.median(times)
    val = flops_per_step(1, 1, n_cpu, D) / t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"LUCID attention fwd+bwd B{B} {heads} N{N} D{D} causal (whole job; sampled: "
                               f"1 head at N={n_cpu})",
                   "global_batch": B, "seq_len": N, "parallelism": "cpu"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"1 (batch, head) at N={n_cpu}, D={D}, fp32, oracle/torch_ref.py"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# LUCID-Path
# ---------------------------------------------------------------------------
PATH_METRIC = "LUCID-Path fwd+bwd TFLOP/s (parallel_lucid_path_attention, B2 H16 T16384 K128)"
PATH_CONFIG = (2, 16, 16384, 128)   # B per rank, H, T, K


def path_cpu_sample(T: int, seed: int = 0):
    """Seconds for one (batch, head) of the LUCID-Path fwd+bwd at length T on
    the host: the float64 block restatement of the reference algorithm
    (oracle/path_oracle.py, blocks of 64 like the reference)."""
    from oracle.path_oracle import make_path_inputs, path_bwd_blockwise
    d = make_path_inputs(seed, 1, T, 1, 128)
    t0 = time.perf_counter()
    path_bwd_blockwise(d["k"], d["v"], d["w"], d["beta"], d["do"], bt=64)
    return time.perf_counter() - t0


def path_reference_arm(args):
    B, H, T, K = PATH_CONFIG
    n_cpu = min(args.cpu_n, 4096)
    path_cpu_sample(256)
    for _ in range(args.warmup):
        path_cpu_sample(n_cpu)
    times = [path_cpu_sample(n_cpu, seed=i) for i in range(args.steps)]
    t = statistics.median(times)
    val = 14.0 * n_cpu * n_cpu * K / t / 1e12
    line = {
        "impl": "reference", "metric": PATH_METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"LUCID-Path fwd+bwd B{B} H{H} T{T} K{K} (whole job; sampled: 1 head at T={n_cpu})",
                   "global_batch": B, "seq_len": T, "parallelism": "cpu"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"1 (batch, head) at T={n_cpu}, float64 numpy, oracle/path_oracle.py"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def bench_path(args, torch, dist, dev, world, rank, local, barrier):
    import ctypes as ct
    from lucid_b200 import _lib
    from lucid_b200.path import parallel_lucid_path_attention, path_bwd, path_fwd
    lib = _lib.load()
    Bg, Hg, T, K = PATH_CONFIG
    if args.path_seq:   # a shorter sequence (profiling cases); the metric is quoted at T = 16384
        T = args.path_seq
    b0, B, h0, H = shard(Bg, Hg, world, rank)
    k, v, w, do = (torch.empty(B, T, H, K, dtype=torch.bfloat16, device=dev) for _ in range(4))
    beta = torch.empty(B, T, H, dtype=torch.bfloat16, device=dev)
    for bi in range(B):
        for hi in range(H):
            # every (batch, head) slice from its own generator: independent of the GPU count
            g = torch.Generator(device=dev).manual_seed(3000 + 8 * ((b0 + bi) * 4096 + h0 + hi))
            k[bi, :, hi] = torch.randn(T, K, generator=g, device=dev).bfloat16()
            v[bi, :, hi] = torch.randn(T, K, generator=g, device=dev).bfloat16()
            w[bi, :, hi] = torch.nn.functional.normalize(torch.randn(T, K, generator=g, device=dev), dim=-1).bfloat16()
            beta[bi, :, hi] = (2 * torch.sigmoid(torch.randn(T, generator=g, device=dev))).bfloat16()
            do[bi, :, hi] = torch.randn(T, K, generator=g, device=dev).bfloat16()
    for t in (k, v, w, beta):
        t.requires_grad_(True)

    def step():
        k.grad = v.grad = w.grad = beta.grad = None
        o, _ = parallel_lucid_path_attention(k, v, w, beta)
        o.backward(do)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step()
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    fl = 14.0 * T * T * K * Bg * Hg      # the whole job's work, fixed as the GPU count grows
    tflops = fl / (ms * 1e-3) / 1e12

    # ---- per kernel family (profile hook), dominant kernel -> roofline ----
    pk_burst, pk_sust, hbm, pk_kind = peaks()
    stage_ms, stage_n = {}, {}
    names = ["path_block", "path_scores", "path_solve", "path_solve_t", "path_row", "path_col"]
    with torch.no_grad():
        kd, vd, wd, bd = (t.detach() for t in (k, v, w, beta))
        for name in names:
            lib.lucid_profile_enable(_lib.KERNEL_IDS[name])
            for _ in range(2):
                o, st, _ = path_fwd(kd, vd, wd, bd)
                path_bwd(st, do, kd, wd, bd)
                del o, st
            torch.cuda.synchronize()
            tot, n = ct.c_float(), ct.c_int()
            lib.lucid_profile_read(ct.byref(tot), ct.byref(n))
            stage_ms[name] = tot.value / 2
            stage_n[name] = n.value // 2
        lib.lucid_profile_enable(0)
    # algorithmic bytes / flops of each O(T^2) kernel per (batch, head): one 128x128
    # bf16 tile is 32 KiB, one 128^3 tile GEMM is 2*128^3 flops
    NB = T // 128
    pairs = NB * (NB - 1) // 2 * B * H
    tile_b, tile_f = 128 * 128 * 2, 2.0 * 128 ** 3
    alg = {  # (bytes that must cross HBM, tensor flops)
        "path_scores": (2 * pairs * tile_b, 4 * pairs * tile_f),     # write L and Q~; S hi+lo, S2, update
        "path_solve": (pairs * tile_b, pairs * tile_f),               # read L; L O
        "path_solve_t": (pairs * tile_b, pairs * tile_f),
        "path_row": (3 * pairs * tile_b, 4 * pairs * tile_f),         # read L, write dA and dQ~; 4 GEMMs
        "path_col": (3 * pairs * tile_b, 2 * pairs * tile_f),         # read dA, Q~, dQ~; 2 GEMMs
    }
    stage = {}
    for n_, (by, fl_) in alg.items():
        sec = stage_ms[n_] * 1e-3
        stage[n_] = {"ms": stage_ms[n_], "gbs": by / sec / 1e9, "hbm_frac": by / sec / 1e9 / hbm,
                     "tflops": fl_ / sec / 1e12, "tensor_frac": fl_ / sec / 1e12 / pk_burst}
    dom = max(alg, key=lambda n_: stage_ms[n_])
    bound = "hbm" if stage[dom]["hbm_frac"] >= stage[dom]["tensor_frac"] else "tensor"
    if bound == "hbm":
        roof = {"bound": "hbm", "kernel": dom, "achieved": stage[dom]["gbs"], "peak": hbm, "unit": "GB/s",
                "frac": stage[dom]["hbm_frac"], "peak_kind": f"{pk_kind} HBM copy bandwidth"}
    else:
        roof = {"bound": "tensor", "kernel": dom, "achieved": stage[dom]["tflops"], "peak": pk_burst,
                "unit": "TFLOP/s", "frac": stage[dom]["tensor_frac"], "peak_kind": f"{pk_kind} burst bf16"}
    roof["traffic"] = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                tj = json.load(f)
            roof["traffic"] = tj.get("path", {}).get(dom)
        except Exception:
            pass

    # ---- end to end through the public API with host buffers ----
    e2e = None
    if not args.no_e2e:
        hk, hv, hw, hb, hdo = (t.detach().cpu().pin_memory() for t in (k, v, w, beta, do))
        outs = [torch.empty_like(hk).pin_memory() for _ in range(4)] + [torch.empty_like(hb).pin_memory()]

        def e2e_step():
            kk, vv, ww, bb = (h.to(dev, non_blocking=True).requires_grad_(True) for h in (hk, hv, hw, hb))
            dd = hdo.to(dev, non_blocking=True)
            oo, _ = parallel_lucid_path_attention(kk, vv, ww, bb)
            oo.backward(dd)
            for h, t in zip(outs, (oo, kk.grad, vv.grad, ww.grad, bb.grad)):
                h.copy_(t.detach(), non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ne = max(1, min(args.steps, 3))
        a0.record()
        for _ in range(ne):
            e2e_step()
        a1.record()
        torch.cuda.synchronize()
        barrier()
        ems = a0.elapsed_time(a1) / ne
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        nb4 = B * T * H * K * 2
        e2e = {"value": fl / (ems * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ems,
               "h2d_bytes_per_step": 4 * nb4 + B * T * H * 2, "d2h_bytes_per_step": 4 * nb4 + B * T * H * 2}

    # ---- the reference Triton op on the same inputs, and both deviations from float64 ----
    ref_gpu = None
    if world == 1 and not args.no_ref_gpu:
        lv = [t.detach().requires_grad_(True) for t in (k, v, w, beta)]
        oo, _ = parallel_lucid_path_attention(*lv)
        oo.backward(do)
        ours = (oo.detach(), lv[0].grad, lv[1].grad, lv[2].grad, lv[3].grad)
        torch.cuda.synchronize()
        del lv, oo
        torch.cuda.empty_cache()
        ref_gpu = reference_gpu_bar(lambda rg: rg.triton_path(torch, k, v, w, beta, do, ours=ours,
                                                              steps=max(1, min(args.steps, 3)),
                                                              check=T <= 16384), ms)
        del ours

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        n_cpu = min(args.cpu_n, 4096)
        path_cpu_sample(256)
        tc = min(path_cpu_sample(n_cpu, seed=i) for i in range(2))
        cpu = {"value": 14.0 * n_cpu * n_cpu * K / tc / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count(),
               "kind": "port", "sample": f"1 (batch, head) at T={n_cpu}, float64 numpy block restatement "
                                         f"(oracle/path_oracle.py), best of 2",
               "seconds_per_sample": tc}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    # the hook brackets the dbeta row-dot and the three gradient packs as one scope
    launches = sum(stage_n.values()) - 1 + 4
    line = {
        "metric": PATH_METRIC, "value": tflops, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"LUCID-Path fwd+bwd B{Bg} H{Hg} T{T} K{K} (whole job), q = k",
                   "global_batch": Bg, "seq_len": T, "heads": Hg, "head_dim": K,
                   "parallelism": f"(batch, head) shards: {B * H} of {Bg * Hg} pairs per rank x{world}, "
                                  f"no collective",
                   "l2": "inputs and path tiles larger than L2, no flush"},
        "tokens_per_s": Bg * T / (ms * 1e-3),
        "frac_of_bf16_peak": tflops / (pk_sust * world),
        "stage": stage, "stage_ms": stage_ms, "roofline": roof, "clocks": clk, "reference_gpu": ref_gpu,
        "gpu_launches": launches * args.steps, "e2e": e2e, "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# full-model prefill
# ---------------------------------------------------------------------------
PREFILL_METRIC = ("Full-model prefill tokens/s: Llama-architecture decoder with LUCID attention "
                  "(lucid/config: 22 layers, hidden 2048, 32/4 heads, head_dim 68), 32768 tokens per GPU (config 4)")
PREFILL_N = 32768


def prefill_cpu_sample(N: int, seed: int = 0):
    """Seconds for ONE decoder layer of the reference model on the host at N
    tokens, float32: LlamaRMSNorm, q/k/v/o projections, the reference's LUCID
    attention (oracle/torch_ref.py: get_v_prime + SDPA) and the SiLU MLP."""
    import torch

    from lucid_b200.decoder import LUCID_CONFIG as C
    from oracle import torch_ref
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    hs, hd, hq, hk, im = C["hidden_size"], C["head_dim"], C["num_attention_heads"], C["num_key_value_heads"], \
        C["intermediate_size"]
    w = lambda *sh: torch.randn(*sh, generator=g) * 0.02
    Wq, Wk, Wv, Wo = w(hq * hd, hs), w(hk * hd, hs), w(hk * hd, hs), w(hs, hq * hd)
    Wg, Wu, Wd = w(im, hs), w(im, hs), w(hs, im)
    x = torch.randn(1, N, hs, generator=g)
    norm = lambda t: t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-5)
    t0 = time.perf_counter()
    with torch.no_grad():
        h = norm(x)
        q = (h @ Wq.T).view(1, N, hq, hd).transpose(1, 2)
        k = (h @ Wk.T).view(1, N, hk, hd).transpose(1, 2)
        v = (h @ Wv.T).view(1, N, hk, hd).transpose(1, 2)
        x = x + torch_ref.lucid_layer(q, k, v, hd ** -0.5).reshape(1, N, hq * hd) @ Wo.T
        h = norm(x)
        x = x + (torch.nn.functional.silu(h @ Wg.T) * (h @ Wu.T)) @ Wd.T
    return time.perf_counter() - t0


def prefill_reference_arm(args):
    n_cpu = min(args.cpu_n, 4096)
    layers = 22
    prefill_cpu_sample(512)
    for _ in range(args.warmup):
        prefill_cpu_sample(n_cpu)
    times = [prefill_cpu_sample(n_cpu, seed=i) for i in range(args.steps)]
    t = sum(times) / len(times) * layers
    val = n_cpu / t
    line = {
        "impl": "reference", "metric": PREFILL_METRIC, "value": val, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"decoder prefill, sampled: 1 of {layers} layers at N={n_cpu} (tokens/s = N / "
                               f"({layers} x layer time); embedding and LM head not timed)",
                   "global_batch": 1, "seq_len": PREFILL_N, "parallelism": "cpu"},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"1 decoder layer at N={n_cpu}, fp32, attention by oracle/torch_ref.py"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


DECODE_METRIC = ("LUCID decode step tokens/s (get_new_v_prime + cache append + decode attention), "
                 "B4 H32 D128, 32768-token cache")


def decode_cpu_sample(Nc: int, seed: int = 0):
    """Seconds for one decode step of one (batch, head) on the host: the
    reference's get_new_v_prime (modeling_lucid.py:576-598) and the attention of
    the new query over the cache, float32 (oracle/torch_ref.py's formulas)."""
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    D = 128
    kc, xc = torch.randn(1, 1, Nc, D, generator=g), torch.randn(1, 1, Nc, D, generator=g)
    q, kn, vn = (torch.randn(1, 1, 1, D, generator=g) for _ in range(3))
    s = D ** -0.5
    t0 = time.perf_counter()
    with torch.no_grad():
        nk = torch.nn.functional.rms_norm(kn, (D,), eps=1e-5)
        nc = torch.nn.functional.rms_norm(kc, (D,), eps=1e-5)
        x_new = vn - torch.exp(s * nk @ nc.transpose(-1, -2) - 1 / s) @ xc
        k_all, x_all = torch.cat([kc, kn], 2), torch.cat([xc, x_new], 2)
        torch.nn.functional.scaled_dot_product_attention(q, k_all, x_all, scale=s)
    return time.perf_counter() - t0


def decode_reference_arm(args):
    n_cpu = min(args.cpu_n, 32768)
    decode_cpu_sample(1024)
    for _ in range(args.warmup):
        decode_cpu_sample(n_cpu)
    times = [decode_cpu_sample(n_cpu, seed=i) for i in range(args.steps)]
    t = sum(times) / len(times) * 4 * 32   # B4 x H32 (batch, head) pairs per step
    val = 4 / t
    line = {
        "impl": "reference", "metric": DECODE_METRIC, "value": val, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"decode step B4 H32 D128 cache {n_cpu} (sampled: one (batch, head), x 128)",
                   "global_batch": 4, "seq_len": n_cpu, "parallelism": "cpu"},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"1 (batch, head) decode step, cache {n_cpu}, fp32 torch"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def bench_decode(args, torch, dist, dev, world, rank, local, barrier):
    """One decode step per iteration through decode_step (the path LucidAttention
    takes): x_new = get_new_v_prime(k_new, v_new) over the cache (raw keys, solved
    values) and the new query's attention over the cache plus the new token, in one
    pass over the cache (HBM-bound), then the append of (k_new, x_new).  The
    comparison is PyTorch SDPA decoding one query over a plain KV cache of the same
    size (also one pass)."""
    import torch.nn.functional as F

    from lucid_b200 import decode_step, decode_step_fused
    B, H, Nc, D = 4, 32, 32768, 128
    s = D ** -0.5
    g = torch.Generator(device=dev).manual_seed(6000 + rank)
    bf = dict(dtype=torch.bfloat16, device=dev)
    kc = torch.randn(B, H, Nc + 1, D, generator=g, device=dev).to(torch.bfloat16)
    xc = (0.1 * torch.randn(B, H, Nc + 1, D, generator=g, device=dev)).to(torch.bfloat16)
    q, kn, vn = (torch.randn(B, H, 1, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))

    assert decode_step_fused(H, H, 1)

    def step():
        o, x_new = decode_step(q, kn, vn, kc[:, :, :Nc], xc[:, :, :Nc], s, 1e-5)
        kc[:, :, Nc:] = kn
        xc[:, :, Nc:] = x_new
        return o

    def sdpa_step():
        return F.scaled_dot_product_attention(q, kc, xc, scale=s)

    mkev = lambda: torch.cuda.Event(enable_timing=True)
    reps = args.steps

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = mkev(), mkev()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    clocks = ClockSampler(local)
    clocks.start()
    ms = timed(step)
    clk = clocks.stop()
    sdpa_ms = timed(sdpa_step)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # algorithmic bytes: one read of the cache's K and X
    cache_bytes = 2 * B * H * Nc * D * 2
    gbs = cache_bytes / (ms * 1e-3) / 1e9
    _, _, hbm, pk_kind = peaks()

    # end to end: the new token's q / k / v from pinned host memory, the output back
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, kn, vn))
        out = torch.empty(B, 1, H, D, dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            q_, k_, v_ = (h.to(dev, non_blocking=True) for h in (hq, hk, hv))
            o, x_new = decode_step(q_, k_, v_, kc[:, :, :Nc], xc[:, :, :Nc], s, 1e-5)
            kc[:, :, Nc:] = k_
            xc[:, :, Nc:] = x_new
            out.copy_(o, non_blocking=True)

        ems = timed(e2e_step)
        e2e = {"value": world * B / (ems * 1e-3), "unit": "tokens/s", "ms_per_step": ems,
               "h2d_bytes_per_step": 3 * B * H * D * 2, "d2h_bytes_per_step": B * H * D * 2}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        decode_cpu_sample(1024)
        tc = min(decode_cpu_sample(Nc, seed=i) for i in range(3))
        cpu = {"value": B / (tc * B * H), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"1 (batch, head) decode step at cache {Nc}, fp32 torch, best of 3, x {B * H}"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": DECODE_METRIC, "value": world * B / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": reps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"decode step B{B} H{H} D{D}, cache {Nc} tokens (raw keys, solved values), one new "
                               f"token per sequence", "global_batch": B * world, "seq_len": Nc,
                   "parallelism": f"data parallel replicas x{world}",
                   "l2": "cache (2 GiB of K and X) larger than L2, no flush"},
        "roofline": {"bound": "hbm", "kernel": "fused decode step (update + attention partials)",
                     "timed": "whole step (partial, finish and the cache append)", "achieved": gbs, "peak": hbm,
                     "unit": "GB/s", "frac": gbs / hbm, "peak_kind": f"{pk_kind} HBM copy bandwidth",
                     "traffic": None},
        "sdpa_decode_ms": sdpa_ms, "overhead_vs_sdpa_decode": ms / sdpa_ms,
        "clocks": clk, "gpu_launches": 2 * reps, "e2e": e2e, "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def bench_prefill(args, torch, dist, dev, world, rank, local, barrier):
    import ctypes as ct

    from transformers import DynamicCache

    from lucid_b200 import _lib
    from lucid_b200.decoder import LucidForCausalLM, lucid_config
    lib = _lib.load()
    cfg = lucid_config()
    L, N = cfg.num_hidden_layers, PREFILL_N
    hd, hq, hk = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    with torch.device(dev):
        model = LucidForCausalLM(cfg)
    model = model.to(torch.bfloat16).init_weights(seed=4000 + rank).eval()
    g = torch.Generator().manual_seed(4100 + rank)
    ids_host = torch.randint(0, cfg.vocab_size, (1, N), generator=g).pin_memory()
    ids = ids_host.to(dev)

    def step(inp, events=None):
        with torch.no_grad():
            # the reference's prefill: use_cache=True fills (raw keys, solved values)
            return model(inp, past_key_values=DynamicCache(), logits_to_keep=1, attn_events=events)

    for _ in range(args.warmup):
        step(ids)
    torch.cuda.synchronize()
    mkev = lambda: torch.cuda.Event(enable_timing=True)
    events = [[(mkev(), mkev()) for _ in range(L)] for _ in range(args.steps)]
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = mkev(), mkev()
    ev0.record()
    for i in range(args.steps):
        logits = step(ids, events[i])
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    attn_ms = sum(a.elapsed_time(b) for evs in events for a, b in evs) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tok_s = world * N / (ms * 1e-3)
    finite = bool(torch.isfinite(logits).all().item())

    # ---- the LUCID kernels alone (profile hook) and the dominant one's roofline ----
    pk_burst, pk_sust, hbm, pk_kind = peaks()
    stage_ms, stage_n = {}, {}
    for name in ("prep", "solve_fwd", "attn_fwd"):
        lib.lucid_profile_enable(_lib.KERNEL_IDS[name])
        step(ids)
        torch.cuda.synchronize()
        tot, n = ct.c_float(), ct.c_int()
        lib.lucid_profile_read(ct.byref(tot), ct.byref(n))
        stage_ms[name], stage_n[name] = tot.value, n.value
    lib.lucid_profile_enable(0)
    # algorithmic flops per layer at the model's head_dim: causal attention 2 N^2 D per
    # query head, the solve 2 N^2 D per kv head.  Executed: the attention forward runs
    # its GEMMs over the head_dim rounded up to 16 columns, the solve over all 128
    alg = {"attn_fwd": 2.0 * N * N * hd * hq, "solve_fwd": 2.0 * N * N * hd * hk}
    exec_d = {"attn_fwd": -(-hd // 16) * 16, "solve_fwd": 128}
    dom = max(alg, key=lambda n_: stage_ms[n_])
    per_launch_ms = stage_ms[dom] / max(1, stage_n[dom])
    ach = alg[dom] / (per_launch_ms * 1e-3) / 1e12
    roof = {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": pk_burst, "unit": "TFLOP/s",
            "frac": ach / pk_burst, "peak_kind": f"{pk_kind} burst bf16",
            "executed_tflops": ach * exec_d[dom] / hd,
            "note": f"algorithmic flops at head_dim {hd}; the kernel computes {exec_d[dom]} zero-padded columns"}
    roof["traffic"] = None

    # ---- end to end: token ids from pinned host memory, last logits back to the host ----
    e2e = None
    if not args.no_e2e:
        out_host = torch.empty(1, 1, cfg.vocab_size, dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            lg = step(ids_host.to(dev, non_blocking=True))
            out_host.copy_(lg, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        a0, a1 = mkev(), mkev()
        ne = max(1, min(args.steps, 3))
        a0.record()
        for _ in range(ne):
            e2e_step()
        a1.record()
        torch.cuda.synchronize()
        barrier()
        ems = a0.elapsed_time(a1) / ne
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": world * N / (ems * 1e-3), "unit": "tokens/s", "ms_per_step": ems,
               "h2d_bytes_per_step": N * 8, "d2h_bytes_per_step": cfg.vocab_size * 2}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        n_cpu = min(args.cpu_n, 4096)
        prefill_cpu_sample(512)
        tc = min(prefill_cpu_sample(n_cpu, seed=i) for i in range(2))
        cpu = {"value": n_cpu / (L * tc), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"1 of {L} decoder layers at N={n_cpu}, fp32 (attention by oracle/torch_ref.py), best "
                         f"of 2; tokens/s = N / ({L} x layer time)", "seconds_per_layer": tc}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": PREFILL_METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform token ids, random N(0, 0.02) weights)",
        "config": {"workload": f"prefill forward of the {L}-layer LUCID decoder (lucid/config), batch 1 x {N} "
                               f"tokens per GPU, use_cache=True (cache filled), logits of the last position",
                   "global_batch": world, "seq_len": N, "parallelism": f"data parallel replicas x{world}",
                   "l2": "activations and weights larger than L2, no flush"},
        "attention_ms": attn_ms, "attention_share": attn_ms / ms,
        "stage_ms": stage_ms, "roofline": roof, "clocks": clk, "output_finite": finite,
        "gpu_launches": 3 * L * args.steps, "e2e": e2e, "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# context-parallel forward + backward at 128K
# ---------------------------------------------------------------------------
CP_METRIC = "LUCID attention fwd+bwd TFLOP/s, context-parallel, B1 H32 N131072 D128 (config 5)"
CP_METRIC_FWD = "LUCID attention forward TFLOP/s, context-parallel, B1 H32 N131072 D128 (config 5)"


def cp_cpu_sample(N: int, seed: int = 0, backward: bool = True):
    """Seconds for one (batch, head) of the LUCID attention forward (+ backward)
    at length N on the host (oracle/torch_ref.py, fp32, correlated keys of config 5)."""
    import torch

    from oracle import torch_ref
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    D = 128
    q = torch.randn(1, 1, N, D, generator=g)
    k = 0.6 * torch.randn(1, 1, 1, D, generator=g) + 0.8 * torch.randn(1, 1, N, D, generator=g)
    v = torch.randn(1, 1, N, D, generator=g)
    do = torch.randn(1, N, 1, D, generator=g)
    t0 = time.perf_counter()
    if backward:
        torch_ref.lucid_fwd_bwd(q, k, v, do)
    else:
        with torch.no_grad():
            torch_ref.lucid_layer(q, k, v)
    return time.perf_counter() - t0


def cp_reference_arm(args):
    bwd = not args.cp_forward_only
    n_cpu = min(args.cpu_n, 4096 if bwd else 8192)
    cp_cpu_sample(1024, backward=bwd)
    for _ in range(args.warmup):
        cp_cpu_sample(n_cpu, backward=bwd)
    times = [cp_cpu_sample(n_cpu, seed=i, backward=bwd) for i in range(args.steps)]
    t = sum(times) / len(times)
    val = (14.0 if bwd else 4.0) * n_cpu * n_cpu * 128 / t / 1e12
    what = "forward + backward" if bwd else "forward"
    line = {
        "impl": "reference", "metric": CP_METRIC if bwd else CP_METRIC_FWD, "value": val, "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"LUCID attention {what} B1 H32 N131072 D128 (sampled: 1 head at N={n_cpu})",
                   "global_batch": 1, "seq_len": 131072, "parallelism": "cpu"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"1 (batch, head) at N={n_cpu}, fp32 {what}, oracle/torch_ref.py"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def bench_cp(args, torch, dist, dev, world, rank, local, barrier):
    from lucid_b200.cp import (Layout, balanced_bounds, cp_lucid_attention, cp_lucid_attention_forward,
                               train_bounds, zigzag_layout)
    B, H, N, D = 1, 32, 131072, 128
    bwd = not args.cp_forward_only
    lay = args.cp_layout   # contiguous chunks unless zigzag is asked for by name
    if lay == "zigzag":
        layout = zigzag_layout(N, world)
        layout_desc = f"zigzag: {2 * world} segments, rank r owning r and {2 * world - 1}-r"
    else:
        bounds = train_bounds(N, world) if bwd else balanced_bounds(N, world)
        layout = Layout.contiguous(bounds)
        layout_desc = f"contiguous chunks ({'train_bounds' if bwd else 'balanced_bounds'} {bounds})"
    C = layout.local_rows(rank)
    s = D ** -0.5
    # K = 0.6 s + 0.8 n with s shared per head (the same on every rank) and n per token
    gs = torch.Generator(device=dev).manual_seed(5000)
    shared = torch.randn(B, H, 1, D, generator=gs, device=dev)
    g = torch.Generator(device=dev).manual_seed(5001 + rank)
    q = torch.randn(B, H, C, D, generator=g, device=dev).bfloat16()
    k = (0.6 * shared + 0.8 * torch.randn(B, H, C, D, generator=g, device=dev)).bfloat16()
    v = torch.randn(B, H, C, D, generator=g, device=dev).bfloat16()
    do = torch.randn(B, C, H, D, generator=g, device=dev).bfloat16()
    q.requires_grad_(bwd)
    k.requires_grad_(bwd)
    v.requires_grad_(bwd)

    def step():
        if not bwd:
            return cp_lucid_attention_forward(q, k, v, scale=s, head_groups=args.head_groups, layout=layout)
        q.grad = k.grad = v.grad = None
        o = cp_lucid_attention(q, k, v, scale=s, head_groups=args.head_groups, layout=layout)
        o.backward(do)
        return o.detach()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        o = step()
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    finite = bool(torch.isfinite(o).all().item())
    if bwd:
        finite = finite and all(bool(torch.isfinite(t.grad).all().item()) for t in (q, k, v))
    # per (batch, head): forward (solve 2 N^2 D + attention 2 N^2 D), backward 10 N^2 D
    fl = (14.0 if bwd else 4.0) * N * N * D * B * H
    tflops = fl / (ms * 1e-3) / 1e12
    pk_burst, pk_sust, hbm, pk_kind = peaks()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    G = args.head_groups
    # launches of rank 0 per step: forward prep / solve / attention per group; backward delta,
    # prep of the later rows, flag publishes (one per later rank), attention column pass,
    # transposed solve, solve row pass + finalize and attention row pass per group
    mine = layout.mine(rank)
    first, last = mine[0], mine[-1]
    foreign_before = sum(1 for x in range(last) if layout.owner(x) != rank)
    foreign_after = sum(1 for x in range(first + 1, layout.n) if layout.owner(x) != rank)
    # rank 0 per step: forward prep of every segment up to its last, solve + attention per own
    # segment, one flag publish per received segment (all per head group); backward delta,
    # prep of the later segments, attention column, transposed solve, solve row + finalize and
    # attention row per own segment, one publish per received dV segment
    launches = G * ((last + 1) + 2 * len(mine) + foreign_before)
    if bwd:
        launches += G * (len(mine) + (layout.n - 1 - last) + 5 * len(mine) + foreign_after)
    what = "forward + backward" if bwd else "FORWARD"
    line = {
        "metric": CP_METRIC if bwd else CP_METRIC_FWD, "value": tflops, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"LUCID attention {what} B{B} H{H} N{N} D{D}, keys 0.6 s + 0.8 n, sequence split "
                               f"over {world} ranks, {layout_desc}, {G} head groups pipelined",
                   "global_batch": B, "seq_len": N, "parallelism": f"context parallel x{world} (NCCL send/recv)",
                   "l2": "inputs larger than L2, no flush"},
        "tokens_per_s": B * N / (ms * 1e-3),
        "frac_of_bf16_peak": tflops / (pk_sust * world),
        "output_finite": finite,
        "clocks": clk,
        "gpu_launches": launches * args.steps,
        "e2e": None, "cpu_baseline": None,
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
# ---------------------------------------------------------------------------
# LUCID attention (the metric's configuration and config 2)
# ---------------------------------------------------------------------------
def shard(B, Hkv, world, rank):
    """(batch, kv head) pairs of a B x Hkv workload split into `world` contiguous equal
    shards (GPU g gets pairs [g B Hkv / W, (g + 1) B Hkv / W)).  Returns (b0, nb, kv0, nkv):
    rank `rank` owns batch elements [b0, b0 + nb) x kv heads [kv0, kv0 + nkv) (with all
    query heads of those kv heads).  Raises ValueError when the pairs do not split into
    such rectangles."""
    pairs = B * Hkv
    if world < 1 or pairs % world:
        raise ValueError(f"{pairs} (batch, kv head) pairs do not split over {world} ranks")
    per = pairs // world
    start = rank * per
    if per % Hkv == 0:
        return start // Hkv, per // Hkv, 0, Hkv
    if Hkv % per == 0:
        return start // Hkv, 1, start % Hkv, per
    raise ValueError(f"{per} pairs per rank do not tile batch x {Hkv} kv heads")


def shard_inputs(torch, dev, B0, nb, kv0, nkv, G, N, D, qs, seed=1000):
    """This rank's slice of the global inputs: every (batch, head) slice is drawn from its
    own generator seeded by its global index, so the data do not depend on the GPU count."""
    def head(seed_, sc=1.0):
        g = torch.Generator(device=dev).manual_seed(seed_)
        return (torch.randn(N, D, generator=g, device=dev) * sc).to(torch.bfloat16)
    q = torch.empty(nb, nkv * G, N, D, dtype=torch.bfloat16, device=dev)
    do = torch.empty(nb, N, nkv * G, D, dtype=torch.bfloat16, device=dev)
    k = torch.empty(nb, nkv, N, D, dtype=torch.bfloat16, device=dev)
    v = torch.empty(nb, nkv, N, D, dtype=torch.bfloat16, device=dev)
    for bi in range(nb):
        b = B0 + bi
        for hi in range(nkv):
            kvh = kv0 + hi
            k[bi, hi] = head(seed + 4 * (b * 4096 + kvh))
            v[bi, hi] = head(seed + 4 * (b * 4096 + kvh) + 1)
            for gi in range(G):
                hq = kvh * G + gi
                q[bi, hi * G + gi] = head(seed + 4 * (b * 4096 + hq) + 2, qs)
                do[bi, :, hi * G + gi] = head(seed + 4 * (b * 4096 + hq) + 3)
    return q, k, v, do


def pipelined_e2e(torch, dev, steps, h_in, make_outs, run):
    """End-to-end time per step through the public API with host buffers: every step
    copies its inputs from pinned host memory (h_in) to the device, computes, and copies
    its results back into pinned host memory.  Copies in, compute and copies out run on
    three streams, double-buffered, so step i's compute overlaps the copies of steps
    i - 1 and i + 1.  `run(inputs, wait_in, emit)` does the compute: `wait_in(j)` makes it
    wait for input j's copy only where it first needs it, and `emit(j, t)` queues the copy
    of result j as soon as it is computed (every result of the step must be emitted).
    Returns ms per step (device events from the first copy in to the last copy out)."""
    comp = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    d_in = [[torch.empty_like(t, device=dev) for t in h_in] for _ in range(2)]
    h_out = [make_outs() for _ in range(2)]
    in_ready = [[torch.cuda.Event() for _ in h_in] for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_free = [torch.cuda.Event() for _ in range(2)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def copy_in(i):
        s = i & 1
        with torch.cuda.stream(h2d):
            if i >= 2:
                h2d.wait_event(in_free[s])       # step i - 2 is done with these buffers
            for j, (d, h) in enumerate(zip(d_in[s], h_in)):
                d.copy_(h, non_blocking=True)
                in_ready[s][j].record(h2d)

    torch.cuda.synchronize()
    t0.record(h2d)
    copy_in(0)
    for i in range(steps):
        s = i & 1
        if i + 1 < steps:
            copy_in(i + 1)
        first = [True]

        def wait_in(j, s=s):
            comp.wait_event(in_ready[s][j])

        def emit(j, t, s=s, i=i, first=first):
            ready = torch.cuda.Event()
            ready.record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ready)
                if i >= 2 and first[0]:
                    d2h.wait_event(out_free[s])  # step i - 2's host buffers were read
                first[0] = False
                t.record_stream(d2h)
                h_out[s][j].copy_(t.detach(), non_blocking=True)

        run(d_in[s], wait_in, emit)
        in_free[s].record(comp)
        out_free[s].record(d2h)
    t1.record(d2h)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / steps


def bench_lucid(args, torch, dist, dev, world, rank, local, barrier):
    from lucid_b200 import _lib, attn_bwd, attn_fwd, lucid_attention, solve_bwd, solve_fwd
    lib = _lib.load()
    Bg, Hg, N, D, qs = CONFIGS[args.config]
    Hkvg = KV_HEADS.get(args.config, Hg)
    G = Hg // Hkvg
    b0, B, kv0, Hkv = shard(Bg, Hkvg, world, rank)
    H = Hkv * G
    s = D ** -0.5
    q, k, v, do = shard_inputs(torch, dev, b0, B, kv0, Hkv, G, N, D, qs)
    q.requires_grad_(True)
    k.requires_grad_(True)
    v.requires_grad_(True)

    def step():
        q.grad = k.grad = v.grad = None
        o = lucid_attention(q, k, v, s)
        o.backward(do)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _lib.check_status()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        step()
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    _lib.check_status()
    ms_local = ev0.elapsed_time(ev1) / args.steps
    ms = ms_local
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    fl = flops_per_step(Bg, Hg, N, D, Hkvg)          # the whole job's work, fixed as N grows
    tflops = fl / (ms * 1e-3) / 1e12

    # ---- per-kernel timing on this rank's shard (dominant kernel -> roofline) ----
    pk_burst, pk_sust, hbm, pk_kind = peaks()
    per_stage_flops = stage_units(H, Hkv)
    # the stored-tile schedule (chosen by the ops when its workspace fits) streams the
    # column passes' tiles through the row passes: one GEMM per tile, no recompute
    from lucid_b200.ops import stored_tiles_fit
    stored = stored_tiles_fit(lib.lucid_attn_bwd_fast_workspace_bytes(B, H, Hkv, N, D), dev)
    row_exec = 1 if stored else 3
    executed_flops = dict(per_stage_flops, attn_bwd_row=row_exec * H, solve_bwd_row=row_exec * Hkv)
    stage_ms = {}
    with torch.no_grad():
        x, khat, u, rstd, dinv = solve_fwd(k, v, s, 1e-5)
        o, lse, o_res = attn_fwd(q, k, x, s, residual=True)
        dq, dkf, dxf = attn_bwd(q, k, x, o, do, lse, s, o_res=o_res)
        torch.cuda.synchronize()
        runs = {
            "prep": lambda: solve_fwd(k, v, s, 1e-5),
            "solve_fwd": lambda: solve_fwd(k, v, s, 1e-5),
            "attn_fwd": lambda: attn_fwd(q, k, x, s, residual=True),
            "attn_bwd": lambda: attn_bwd(q, k, x, o, do, lse, s, o_res=o_res),
            "attn_bwd_row": lambda: attn_bwd(q, k, x, o, do, lse, s, o_res=o_res),
            "solve_bwd": lambda: solve_bwd(k, x, khat, u, rstd, dinv, dxf, s, dk_add=dkf),
            "solve_bwd_row": lambda: solve_bwd(k, x, khat, u, rstd, dinv, dxf, s, dk_add=dkf),
        }
        for name, fn in runs.items():
            lib.lucid_profile_enable(_lib.KERNEL_IDS[name])
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            tot, n = ctypes.c_float(), ctypes.c_int()
            lib.lucid_profile_read(ctypes.byref(tot), ctypes.byref(n))
            stage_ms[name] = tot.value / max(n.value, 1)
        lib.lucid_profile_enable(0)
        del x, khat, u, rstd, dinv, o, lse, dq, dkf, dxf
    unit_flops = float(N) * N * D * B
    stage_tflops = {n: {"alg": per_stage_flops[n] * unit_flops / (stage_ms[n] * 1e-3) / 1e12,
                        "executed": executed_flops[n] * unit_flops / (stage_ms[n] * 1e-3) / 1e12}
                    for n in per_stage_flops}
    dom = max(per_stage_flops, key=lambda n: stage_ms[n])
    achieved = stage_tflops[dom]["alg"]
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath) and world == 1:
        try:
            with open(tpath) as f:
                tj = json.load(f)
            traffic = tj.get(args.config, {}).get(dom)
        except Exception:
            traffic = None

    # ---- causal attention of the same shape (overhead reference) ----
    sdpa_ms = sdpa_fwd_bwd_ms(torch, q, k, v, do, s)
    our_attn_ms = stage_ms["attn_fwd"] + stage_ms["attn_bwd"] + stage_ms["attn_bwd_row"]

    # ---- end to end through the public API with host buffers ----
    e2e = None
    if not args.no_e2e:
        h_in = [t.detach().cpu().pin_memory() for t in (q, k, v, do)]

        def make_outs():
            return [torch.empty(B, N, H, D, dtype=torch.bfloat16).pin_memory(),
                    torch.empty(B, H, N, D, dtype=torch.bfloat16).pin_memory()] + \
                   [torch.empty(B, Hkv, N, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]

        def run(d, wait_in, emit):
            # the forward starts once q, k, v are in; dO's copy overlaps it, and O's copy
            # back overlaps the backward
            for j in range(3):
                wait_in(j)
            qq, kk, vv = (t.detach().requires_grad_(True) for t in d[:3])
            oo = lucid_attention(qq, kk, vv, s)
            emit(0, oo)
            wait_in(3)
            oo.backward(d[3])
            emit(1, qq.grad)
            emit(2, kk.grad)
            emit(3, vv.grad)

        pipelined_e2e(torch, dev, 2, h_in, make_outs, run)      # warm-up
        barrier()
        ems = pipelined_e2e(torch, dev, max(2, min(args.steps, 6)), h_in, make_outs, run)
        barrier()
        _lib.check_status()
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        # q, dO (o, dq) per query head; k, v (dk, dv) per kv head: this rank's bytes
        nbytes = 2 * B * N * D * 2 * (H + Hkv)
        e2e = {"value": fl / (ems * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ems,
               "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
               "schedule": "copies in / compute / copies out on three streams, double-buffered; the "
                           "forward waits for q, k, v only and O is copied back during the backward"}
        del h_in

    # ---- the reference's own GPU path on the same inputs (config 2: it fits one GPU) ----
    ref_gpu = None
    if world == 1 and args.config == "cfg2" and not args.no_ref_gpu:
        ref_gpu = reference_gpu_bar(lambda rg: rg.torch_path_cfg2(torch, q, k, v, do, ours_outputs(
            torch, lucid_attention, q, k, v, do, s), steps=max(1, min(args.steps, 3))), ms)

    # ---- the grouped-query layout of the reference model (Hq 32, Hkv 4) beside it ----
    gqa = None
    if world == 1 and args.config == "32k" and not args.no_gqa:
        del q, k, v, do
        torch.cuda.empty_cache()
        gqa = gqa_overhead(torch, dev, lucid_attention, _lib, N, D, qs)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(args.cpu_n, D, reps=10)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    # prep, solve, attn fwd, delta, attn bwd col + row, solve bwd col + row, finalize
    launches_per_step = 9
    heads = f"H{Hg}" if Hkvg == Hg else f"Hq{Hg} Hkv{Hkvg}"
    line = {
        "metric": METRIC,
        "value": tflops,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"LUCID attention fwd+bwd B{Bg} {heads} N{N} D{D} causal "
                               f"{'MHA' if Hkvg == Hg else 'GQA'} (whole job)",
                   "global_batch": Bg, "seq_len": N, "heads": Hg, "kv_heads": Hkvg, "head_dim": D,
                   "parallelism": f"(batch, kv head) shards: {B * Hkv} of {Bg * Hkvg} pairs per rank x{world}, "
                                  f"no collective",
                   "l2": "inputs larger than L2 (268 MB per tensor at one GPU), no flush"},
        "tokens_per_s": Bg * N / (ms * 1e-3),
        "frac_of_bf16_peak": tflops / (pk_sust * world),
        "peak_used": {"bf16_tflops_sustained": pk_sust, "bf16_tflops_burst": pk_burst, "kind": pk_kind,
                      "note": "frac_of_bf16_peak divides by the peak of all GPUs of the run"},
        "rank0_ms_per_step": ms_local,
        "overhead_vs_causal_attn": {"sdpa_fwd_bwd_ms": sdpa_ms, "lucid_fwd_bwd_ms": ms_local,
                                    "ratio_vs_sdpa": ms_local / sdpa_ms, "our_attention_only_ms": our_attn_ms,
                                    "ratio_vs_our_attention": ms_local / our_attn_ms,
                                    "shape": f"rank 0 shard B{B} Hq{H} Hkv{Hkv} N{N}"},
        "gqa_overhead_vs_causal_attn": gqa,
        "reference_gpu": ref_gpu,
        "stage_ms": stage_ms,
        "stage_tflops": stage_tflops,
        "backward_schedule": "stored tiles" if stored else "recompute",
        "roofline": {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": pk_burst,
                     "unit": "TFLOP/s", "frac": achieved / pk_burst, "traffic": traffic,
                     "peak_kind": f"{pk_kind} burst bf16 (kernel timed alone)"},
        "clocks": clk,
        "gpu_launches": launches_per_step * args.steps,
        "e2e": e2e,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def ours_outputs(torch, lucid_attention, q, k, v, do, s):
    """(o, dq, dk, dv) of one fwd+bwd of our op on the benchmark's inputs."""
    qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
    o = lucid_attention(qq, kk, vv, s)
    o.backward(do)
    return o.detach(), qq.grad, kk.grad, vv.grad


def reference_gpu_bar(run, our_ms):
    """Run one reference-GPU comparison (baseline/reference_gpu.py) and add our speed-up
    over it; a missing or failing reference copy is reported, not fatal."""
    import torch
    try:
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        import reference_gpu as rg
        out = run(rg)
        out["our_speedup"] = out["ms_per_step"] / our_ms
        return out
    except Exception as e:   # the comparator is optional: report why it did not run (and where)
        import traceback
        frames = [f"{os.path.basename(fr.filename)}:{fr.lineno} {fr.name}" for fr in traceback.extract_tb(e.__traceback__)
                  if "_ref" in fr.filename]
        return {"unavailable": f"{type(e).__name__}: {str(e)[:300]}", "where": frames[-3:]}
    finally:
        torch.cuda.empty_cache()


def sdpa_fwd_bwd_ms(torch, q, k, v, do, s, reps=3):
    """PyTorch SDPA (cuDNN on B200) causal fwd+bwd of the same shape, ms per step."""
    import torch.nn.functional as F
    G = q.shape[1] // k.shape[1]
    qd, kd, vd = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    dot = do.transpose(1, 2)

    def sdpa_step():
        qd.grad = kd.grad = vd.grad = None
        F.scaled_dot_product_attention(qd, kd, vd, is_causal=True, scale=s, enable_gqa=G > 1).backward(dot)
    for _ in range(2):
        sdpa_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        sdpa_step()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def gqa_overhead(torch, dev, lucid_attention, _lib, N, D, qs, Hq=32, Hkv=4, reps=3):
    """LUCID fwd+bwd against causal SDPA fwd+bwd at the reference model's grouped-query
    layout (Hq 32 query heads over Hkv 4 kv heads, modeling_lucid.py:523-524), B1 N D."""
    q, k, v, do = shard_inputs(torch, dev, 0, 1, 0, Hkv, Hq // Hkv, N, D, qs, seed=5000)
    q.requires_grad_(True)
    k.requires_grad_(True)
    v.requires_grad_(True)
    s = D ** -0.5

    def step():
        q.grad = k.grad = v.grad = None
        lucid_attention(q, k, v, s).backward(do)
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        step()
    e1.record()
    torch.cuda.synchronize()
    _lib.check_status()
    ms = e0.elapsed_time(e1) / reps
    sdpa = sdpa_fwd_bwd_ms(torch, q, k, v, do, s, reps)
    fl = flops_per_step(1, Hq, N, D, Hkv)
    return {"shape": f"B1 Hq{Hq} Hkv{Hkv} N{N} D{D}", "lucid_fwd_bwd_ms": ms, "sdpa_fwd_bwd_ms": sdpa,
            "ratio_vs_sdpa": ms / sdpa, "lucid_tflops": fl / (ms * 1e-3) / 1e12,
            "arithmetic_ratio": (Hq + Hkv) / Hq}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + ["path", "cp128k", "prefill", "decode"], default="32k")
    ap.add_argument("--head-groups", type=int, default=8, help="cp128k: kv-head groups pipelined across ranks")
    ap.add_argument("--cp-forward-only", action="store_true", help="cp128k: time the forward chain alone")
    ap.add_argument("--path-seq", type=int, default=0,
                    help="path: sequence length instead of config 3's 16384 (smaller profiling cases)")
    ap.add_argument("--cp-layout", choices=["zigzag", "contiguous"], default="contiguous",
                    help="cp128k: rows per rank (contiguous: one chunk per rank, solved X chunks flowing "
                         "rank to rank, the default; zigzag: segments r and 2W-1-r, a non-default variant)")
    ap.add_argument("--cpu-n", type=int, default=8192, help="sequence length of the CPU sample")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-gqa", action="store_true", help="skip the grouped-query overhead measurement")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="cfg2 / path: skip timing the reference's own GPU code (baseline/_ref) beside ours")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        return reference_arm(args)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        # a short timeout ends a stuck collective with an error instead of holding all GPUs
        dist.init_process_group("nccl", timeout=timedelta(seconds=60 if args.config == "cp128k" else 300),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    if args.config == "path":
        return bench_path(args, torch, dist, dev, world, rank, local, barrier)
    if args.config == "cp128k":
        return bench_cp(args, torch, dist, dev, world, rank, local, barrier)
    if args.config == "prefill":
        return bench_prefill(args, torch, dist, dev, world, rank, local, barrier)
    if args.config == "decode":
        return bench_decode(args, torch, dist, dev, world, rank, local, barrier)
    return bench_lucid(args, torch, dist, dev, world, rank, local, barrier)

if __name__ == "__main__":
    sys.exit(main())
