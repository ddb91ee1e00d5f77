#!/usr/bin/env python
"""Benchmark: train tokens/s of toy's training step (forward + cross-entropy +
backward + AdamW) on B200s, with the step's roofline fraction.

Default workload (one GPU): SmolLM2-135M shape, full f32 fine-tune with every
weight N(0, 0.02), B=8 sequences of T=512 tokens per GPU, data-parallel over N
GPUs (weak scaling). The same line carries the QLoRA workload (q, v adapters
over a frozen Q8_0 base, B=8 T=512) as `qlora_step`. Synthetic data:
token ids uniform in [0, vocab), labels = ids shifted by one inside each
sequence, weights from the reference's seeded init stream.

The CPU baseline (rank 0, one GPU) and the reference arm (`--impl reference`)
run the oracle's numpy restatement of toy's CPU step in float32 on the host
cores, on the workload's own B and T (one full step, ~0.5-1 min).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload smollm2_full_ft_b8_t512|smollm2_qlora_b8_t512]

One JSON line is printed by rank 0.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from toy_b200.adamw import AdamW  # noqa: E402
from toy_b200.batch import next_token_labels, positions, synthetic_token_ids  # noqa: E402

METRIC = "train tokens/sec (fwd+bwd+AdamW) at 1/2/4/8 B200; % of step roofline"
KIND_NAMES = ["gemm", "rmsnorm_fwd", "rmsnorm_bwd", "colsum", "rope", "softmax", "swiglu", "cross_entropy",
              "loss_reduce", "adamw", "embedding", "split", "allreduce", "flash_fwd", "flash_bwd", "flash_prep",
              "lora"]

WORKLOADS = {
    "smollm2_full_ft_b8_t512": dict(mode=0, B=8, T=512, lora=None, lr=1e-4, wd=0.01, init_std=0.02),
    "smollm2_qlora_b8_t512": dict(mode=1, B=8, T=512, lora=("q", "v"), lr=1e-4, wd=0.01, init_std=0.0),
    # toy's own LoRA recipe: per-head LoRA-Q (one rank-8 pair per query head, scale 1) over the Q8_0 base
    "smollm2_lora_q_b8_t512": dict(mode=1, B=8, T=512, lora=("q",), per_head=True, lr=1e-4, wd=0.01,
                                   init_std=0.0),
    # the other benchmark configurations' shapes (QLoRA over a Q8_0 base), one GPU each
    "llama32_1b_qlora_r16_b16_t1024": dict(model="llama32_1b", mode=1, B=16, T=1024, rank=16,
                                           lora=("q", "k", "v", "o", "gate", "up", "down"), lr=1e-4, wd=0.01,
                                           init_std=0.0),
    "qwen25_7b_qlora_r16_b4_t2048": dict(model="qwen25_7b", mode=1, B=4, T=2048, rank=16,
                                         lora=("q", "k", "v", "o", "gate", "up", "down"), lr=1e-4, wd=0.01,
                                         init_std=0.0),
    "olmoe_1b_7b_qlora_r8_b8_t1024": dict(model="olmoe_1b_7b", mode=1, B=8, T=1024, rank=8,
                                          lora=("q", "k", "v", "o"), lr=1e-4, wd=0.01, init_std=0.0),
}
MODEL_NAMES = {"smollm2": "SmolLM2-135M shape", "llama32_1b": "Llama-3.2-1B shape", "qwen25_7b": "Qwen2.5-7B shape",
               "olmoe_1b_7b": "OLMoE-1B-7B shape"}

# DRAM traffic of the step's GEMM launches, from one ncu capture of the full
# workload (dram__bytes_read.sum + dram__bytes_write.sum summed over the 363
# GEMM launches of one graph-replayed step, one pass per launch; ncu with
# gpu__time_duration, dram__bytes_read and dram__bytes_write, -s 272 -c 2000).
# The algorithmic bytes (gemm_algorithmic_bytes) are each GEMM's operands plus
# its output and residual addend, summed over the step's GEMMs. ncu writes back and
# invalidates L2 between captured kernels, so an output that still sits in L2
# when its kernel ends is not counted as a DRAM write: the traffic is a lower
# bound on writes, exact on reads.
GEMM_TRAFFIC = {
    "smollm2_full_ft_b8_t512": {"bytes_per_step": 11705450240, "launches": 363,
                                "source": "ncu, full workload, -s 272 -c 2000, the second step (a graph replay)"},
}


def gemm_algorithmic_bytes(cfg, N, f16_wgrad):
    """Operand and output bytes of one full fine-tune step's GEMMs (dense Llama, fused
    flash attention): each operand read once (split planes 4 bytes per element, fp16
    weight-gradient operands 2), each f32 output written once, residual addends read."""
    d, H, KV, dh, ff, L, V = cfg.d_model, cfg.n_heads, cfg.n_kv, cfg.d_head, cfg.d_ff, cfg.n_layers, cfg.vocab
    W = (H + 2 * KV) * dh
    pl, f32 = 4, 4
    wg = 2 if f16_wgrad else 4

    def g(m_rows, k_cols, n_rows, out, a_b=pl, res=0):   # A [M][K], B [N][K], output bytes
        return a_b * (m_rows * k_cols + n_rows * k_cols) + out + res
    per_layer = (
        g(N, d, W, N * W * pl)                              # q|k|v (+ RoPE, head-major planes)
        + g(N, H * dh, d, N * d * f32, res=N * d * f32)     # o (+ residual)
        + g(N, d, 2 * ff, N * 2 * ff * f32)                 # gate|up
        + g(N, ff, d, N * d * f32, res=N * d * f32)         # down (+ residual)
        + g(N, d, ff, N * ff * f32)                         # dX down
        + g(N, 2 * ff, d, N * d * f32)                      # dX gate|up
        + g(N, d, H * dh, N * H * dh * f32)                 # dX o
        + g(N, W, d, N * d * f32)                           # dX q|k|v
        + g(d, N, ff, d * ff * f32, a_b=wg)                 # dW down
        + g(2 * ff, N, d, 2 * ff * d * f32, a_b=wg)         # dW gate|up
        + g(d, N, H * dh, d * H * dh * f32, a_b=wg)         # dW o
        + g(W, N, d, W * d * f32, a_b=wg))                  # dW q|k|v
    head = (g(N, d, V, N * V * f32)                         # LM head (logits)
            + g(N, V, d, N * d * f32)                       # dX of the LM head
            + g(V, N, d, V * d * f32, a_b=wg))              # dW of the LM head
    return L * per_layer + head


def f16_wgrad_on():
    """The library's fp16 weight-gradient setting (read by setting it back)."""
    from toy_b200._lib import lib
    prev = lib().tb2_set_f16_wgrad(1)
    lib().tb2_set_f16_wgrad(prev)
    return prev == 1


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0), \
            "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def step_flops_per_token(cfg, T, mode, lora_targets, rank, per_head=False):
    """Algorithmic FLOPs per token: full FT 6*P_mm + 3*A; QLoRA 4*P_mm + 3*A + 6*P_lora,
    P_mm = projection + LM-head parameters touched per token (an expert block: the
    router and the n_experts_used experts a token visits), A = 4*L*H*dh*(T+1)/2
    (per-head LoRA-Q: P_lora = L*H*r*(d + dh))."""
    d, H, KV, dh, ff, L, V = cfg.d_model, cfg.n_heads, cfg.n_kv, cfg.d_head, cfg.d_ff, cfg.n_layers, cfg.vocab
    ffn = 3 * ff * d * (cfg.n_experts_used if cfg.n_experts else 1) + (cfg.n_experts * d if cfg.n_experts else 0)
    per_layer = d * (H + 2 * KV) * dh + H * dh * d + ffn
    p_mm = L * per_layer + V * d
    A = 4 * L * H * dh * (T + 1) / 2
    if mode == 0:
        return 6 * p_mm + 3 * A
    shapes = {"q": (H * dh, d), "k": (KV * dh, d), "v": (KV * dh, d), "o": (d, H * dh), "gate": (ff, d),
              "up": (ff, d), "down": (d, ff)}
    p_lora = L * sum(rank * (shapes[t][0] + shapes[t][1]) for t in lora_targets)
    if per_head:
        p_lora = L * H * rank * (d + dh)
    return 4 * p_mm + 3 * A + 6 * p_lora


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, device_index: int):
        self.dev = device_index
        self.rows = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.dev)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() in ("active", "1", "0x1"):
                        reasons.add(nm)
            except (ValueError, IndexError):
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def cpu_port_step_rate(wl, steps):
    """The oracle (numpy restatement of toy's CPU step, float32 like ggml-cpu) on
    the host cores, on the workload's own B and T: `steps` full steps (forward,
    CE, backward, AdamW), each timed alone. Returns (tokens/s, steps timed)."""
    from oracle import oracle as O
    cfg_o = O.smollm2_135m()
    B, T = wl["B"], wl["T"]
    if wl["mode"] == 0:
        mdl = O.full_ft_model(cfg_o, seed=42, std_all=wl["init_std"])
    elif wl.get("per_head"):
        mdl = O.qlora_model(cfg_o, O.LoraCfg(rank=8, per_head_q=True, targets=("q",), a_std=1.0), seed=42)
    else:
        mdl = O.qlora_model(cfg_o, O.LoraCfg(rank=8, alpha=16.0, targets=wl["lora"]), seed=42)
    mdl.dtype = np.float32
    mdl.zero_moments()
    times = []
    opt = AdamW.for_lora()
    opt.lr, opt.weight_decay = wl["lr"], wl["wd"]
    for s in range(steps):
        ids = synthetic_token_ids(100 + s, T * B, cfg_o.vocab)
        lab = next_token_labels(ids, T, B, cfg_o.vocab)
        t0 = time.perf_counter()
        O.train_step(mdl, ids, positions(T, B), lab, T, B, opt.hp(s + 1), s == 0)
        times.append(time.perf_counter() - t0)
    return T * B * len(times) / sum(times), len(times)


def cores():
    try:
        from threadpoolctl import threadpool_info
        th = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        if th:
            return max(th)
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_sample_text(wl, n):
    return (f"{n} full step(s) (fwd+CE+bwd+AdamW) of the oracle port (numpy float32, BLAS threads = host cores) "
            f"on the workload's own shape, B={wl['B']} T={wl['T']}, same model and init")


def run_reference(args, wl):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    if wl.get("model", "smollm2") != "smollm2":
        print(json.dumps({"impl": "reference", "unavailable": "the CPU port of this shape takes hours per step; "
                          "the reference arm runs the SmolLM2-135M workloads"}), flush=True)
        return
    # one full step of the workload takes ~0.5-1 min on the host: time one, a second when the first was quick
    value, n = cpu_port_step_rate(wl, 1)
    if wl["B"] * wl["T"] / value < 45.0 and args.steps > 1:
        value, n = cpu_port_step_rate(wl, 2)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": n, "warmup": 0, "ms_per_step": 1000.0 * wl["B"] * wl["T"] / value, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (uniform ids, seeded init)",
            "config": {"workload": args.workload, "model": "SmolLM2-135M shape", "global_batch": wl["B"],
                       "seq_len": wl["T"], "parallelism": "none (host CPU, rank 0)"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores(), "kind": "port",
                             "sample": cpu_sample_text(wl, n)},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def realize(wl, cfg, device):
    from toy_b200 import FromScratch, LoRA, LoraOptions, RecipeOptions
    B, T = wl["B"], wl["T"]
    if wl["mode"] == 0:
        rec = FromScratch(device=device)
        rec.realize(cfg, RecipeOptions(t_seq=T, t_batch=B, seed=42, init_std=wl["init_std"]))
        return rec, rec.fs_cache
    rec = LoRA(device=device)
    r = wl.get("rank", 8)
    lo = None if wl.get("per_head") else LoraOptions(rank=r, alpha=2.0 * r, targets=wl["lora"])
    rec.realize(cfg, r, RecipeOptions(t_seq=T, t_batch=B, seed=42), lo)   # None: the recipe's per-head LoRA-Q
    return rec, rec.lora_cache


def measure(wl, cfg, args, dp, rank, world, local, profile=True):
    """One workload on this rank: warm-up through the public API, e2e (host
    buffers, public step API, wall clock), then K graph replays timed by CUDA
    events on the step stream (inputs resident), max over ranks."""
    from toy_b200._lib import lib
    L = lib()
    B, T = wl["B"], wl["T"]
    N = B * T
    rec, eng = realize(wl, cfg, local)
    if dp:
        dp.attach(eng)
    sess = eng.sess
    opt = AdamW.for_lora()
    opt.lr, opt.weight_decay = wl["lr"], wl["wd"]

    def batch(step):
        ids = synthetic_token_ids(1000 * step + rank, N, cfg.vocab)
        return ids, positions(T, B), next_token_labels(ids, T, B, cfg.vocab)

    batches = [batch(s) for s in range(4)]
    # warm-up through the public API (the first step also captures the CUDA graph)
    for s in range(args.warmup):
        ids, pos, lab = batches[s % len(batches)]
        rec.step(ids, pos, lab, opt.hp(s + 1), s == 0)
    L.tb2_sync(sess)
    # e2e: the public step API with host buffers (uploads + step + loss read-back), wall clock
    if dp:
        dp.barrier()
    t0 = time.perf_counter()
    for s in range(args.steps):
        ids, pos, lab = batches[s % len(batches)]
        rec.step(ids, pos, lab, opt.hp(args.warmup + s + 1), False)
    L.tb2_sync(sess)
    e2e_s = time.perf_counter() - t0
    if dp:
        e2e_s = dp.max_scalar(e2e_s)
    # bytes the step's uploads move host->device: ids, their by-id row order, segment
    # ids/starts/count (embedding scatter), positions, labels (i32 each) and 7 hp floats
    nseg = len(np.unique(batches[0][0]))
    h2d = 4 * N * 4 + 4 * nseg + 4 * (nseg + 1) + 4 + 7 * 4
    # value: inputs resident on the device, K graph replays timed by CUDA events, max over ranks
    ms = C.c_float(0.0)
    with ClockSampler(local) as clk:
        if dp:
            dp.barrier()
        rc = L.tb2_run_steps(sess, args.steps, C.byref(ms))
        if rc != 0:
            raise RuntimeError(f"tb2_run_steps failed: {rc}")
        step_ms = ms.value / args.steps
        if dp:
            step_ms = dp.max_scalar(step_ms)
            dp.barrier()
    out = {"step_ms": step_ms, "e2e_s": e2e_s, "h2d": h2d, "clocks": clk.summary(),
           "launches": L.tb2_step_launches(sess)}
    if profile:
        # live per-kernel breakdown from one profiled (eager) step
        cap = 8192
        kinds = (C.c_int * cap)()
        kms = (C.c_float * cap)()
        kfl = (C.c_double * cap)()
        n = L.tb2_profile_step(sess, 0, kinds, kms, kfl, cap)
        per_kind, gemm_flops, gemm_ms, gemm_n = {}, 0.0, 0.0, 0
        for i in range(min(n, cap)):
            k = KIND_NAMES[kinds[i]] if kinds[i] < len(KIND_NAMES) else "other"
            per_kind[k] = per_kind.get(k, 0.0) + kms[i]
            if kinds[i] == 0:
                gemm_flops += kfl[i]
                gemm_ms += kms[i]
                gemm_n += 1
        out.update(per_kind=per_kind, gemm_flops=gemm_flops, gemm_ms=gemm_ms, gemm_n=gemm_n)
    if dp:
        dp.detach()
    eng.close()
    return out


def run_decode(args):
    """Decode throughput of the KV-cache path (not the training metric): SmolLM2-135M
    shape over the Q8_0 base, n_seq sequences in lockstep at a context of ctx
    positions, f32 and Q8_0 caches; tokens/s from CUDA events around graph replays
    of one decode step (each replay attends over the ctx cached positions)."""
    from toy_b200 import LlamaConfig, LoRA, LoraOptions, RecipeOptions
    from toy_b200._lib import lib
    from toy_b200.decode import KVDecoder
    L = lib()
    cfg = LlamaConfig.smollm2_135m()
    rec = LoRA()
    rec.realize(cfg, 8, RecipeOptions(t_seq=64, t_batch=1, seed=42), LoraOptions(rank=8, targets=("q", "v")))
    rows = []
    ctx = 512
    for kv_q8 in (False, True):
        for nseq in (1, 8, 16):
            dec = KVDecoder(rec.lora_cache, max_T=ctx + 1, n_seq=nseq, kv_q8=kv_q8)
            prompt = synthetic_token_ids(7, nseq * 4, cfg.vocab).reshape(nseq, 4)
            dec.decode_batch(prompt)
            dec.decode_step(prompt[:, 0], np.full(nseq, ctx))   # the timed step attends over ctx + 1 positions
            ms = C.c_float(0.0)
            check_rc = L.tb2_kv_run(rec.lora_cache.sess, args.warmup, C.byref(ms))
            check_rc |= L.tb2_kv_run(rec.lora_cache.sess, args.steps, C.byref(ms))
            if check_rc:
                raise RuntimeError("tb2_kv_run failed")
            step_ms = ms.value / args.steps
            rows.append({"n_seq": nseq, "kv_cache": "q8_0" if kv_q8 else "f32", "ctx": ctx + 1,
                         "ms_per_step": step_ms, "tokens_per_s": nseq / (step_ms * 1e-3),
                         "launches_per_step": L.tb2_kv_launches(rec.lora_cache.sess)})
            dec.close()
    burst, sustained, hbm, src = peaks()
    d, V, ff = cfg.d_model, cfg.vocab, cfg.d_ff
    per_layer = d * (cfg.n_heads + 2 * cfg.n_kv) * cfg.d_head + cfg.n_heads * cfg.d_head * d + 3 * ff * d
    weight_bytes = cfg.n_layers * per_layer * 34 / 32 + V * d * 4   # Q8_0 projections + f32 tied head
    for r in rows:
        kv = cfg.n_layers * cfg.n_kv * cfg.d_head * 2 * r["ctx"] * r["n_seq"] * (34 / 32 if r["kv_cache"] == "q8_0" else 4)
        r["hbm_gbs"] = (weight_bytes + kv) / (r["ms_per_step"] * 1e-3) / 1e9
        r["hbm_frac"] = r["hbm_gbs"] / hbm
    print(json.dumps({"metric": "decode tokens/s (KV cache, Q8_0 base)", "model": "SmolLM2-135M shape",
                      "data": "synthetic", "steps": args.steps, "warmup": args.warmup,
                      "algorithmic_bytes_per_step": "Q8_0 weights + f32 tied head once per step, plus the cache read",
                      "peak_hbm_gbs": hbm, "rows": rows}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="smollm2_full_ft_b8_t512", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-qlora", action="store_true", help="skip the QLoRA sub-measurement")
    ap.add_argument("--decode", action="store_true", help="measure KV-cache decode instead of training")
    ap.add_argument("--batch", type=int, default=0, help="override sequences per GPU (small profiling cases)")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the decoder depth (small profiling cases; recorded in config)")
    ap.add_argument("--q8-ring-l2", type=int, default=1, choices=[0, 1],
                    help="QLoRA plane ring kept resident in the L2 (1, the library default) or not")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    wl = dict(WORKLOADS[args.workload])
    if args.decode:
        run_decode(args)
        return
    if args.impl == "reference":
        run_reference(args, wl)
        return

    rank, world, local = dist_env()
    from toy_b200 import LlamaConfig
    from toy_b200._lib import lib
    lib().tb2_set_q8_ring_l2(args.q8_ring_l2)
    cfg = getattr(LlamaConfig, {"smollm2": "smollm2_135m"}.get(wl.get("model", "smollm2"),
                                                               wl.get("model", "smollm2")))()
    if args.layers:
        cfg.n_layers = args.layers
    if args.batch:
        wl["B"] = args.batch
    B, T = wl["B"], wl["T"]
    N = B * T
    dp = None
    if world > 1:
        from toy_b200.parallel import DataParallel
        dp = DataParallel(rank, world, local)
    r = measure(wl, cfg, args, dp, rank, world, local)
    qlora = None
    if not args.no_qlora and wl["mode"] == 0 and wl.get("model", "smollm2") == "smollm2":
        qwl = dict(WORKLOADS["smollm2_qlora_b8_t512"])
        if args.batch:
            qwl["B"] = args.batch
        qlora = measure(qwl, cfg, args, dp, rank, world, local, profile=False)
    burst, sustained, hbm, src = peaks()
    step_ms = r["step_ms"]
    gemm_tflops = r["gemm_flops"] / (r["gemm_ms"] * 1e-3) / 1e12 if r["gemm_ms"] > 0 else 0.0
    f_tok = step_flops_per_token(cfg, T, wl["mode"], wl["lora"] or (), wl.get("rank", 8), wl.get("per_head", False))
    tokens = N * world
    value = tokens / (step_ms * 1e-3)
    step_tflops = f_tok * N / (step_ms * 1e-3) / 1e12
    if rank != 0:
        if dp:
            dp.close()
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline and not args.layers and not args.batch and \
            wl.get("model", "smollm2") == "smollm2":
        v, nsteps = cpu_port_step_rate(wl, 1)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores(), "kind": "port", "sample": cpu_sample_text(wl, nsteps)}
    tot = sum(r["per_kind"].values())
    traffic = GEMM_TRAFFIC.get(args.workload) if not (args.layers or args.batch) else None
    f16w = wl["mode"] == 0 and f16_wgrad_on()
    alg_bytes = gemm_algorithmic_bytes(cfg, tokens // world, f16w) if traffic else None
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (tensor-core products on split-bf16 pairs, f32 accumulate" +
                 ("; weight gradients: one fp16 pass, gradients scaled per tensor by a power of two)" if f16w
                  else ")"),
        "data": "synthetic (uniform ids, seeded init)",
        "config": {"workload": args.workload, "model": MODEL_NAMES[wl.get("model", "smollm2")], "global_batch": B * world,
                   "seq_len": T, "parallelism": f"dp{world}", "tokens_per_step": tokens,
                   "init": "every weight N(0, 0.02) f32" if wl["mode"] == 0 else "Q8_0 base from N(0, 0.02)",
                   "l2": "inputs larger than L2: the step's working set (activations and weights, several GB) "
                         "far exceeds the 126 MB L2",
                   **({"layers_override": cfg.n_layers} if args.layers else {})},
        "step_roofline": {"tflops_algorithmic": step_tflops, "peak_tflops": sustained,
                          "frac": step_tflops / sustained, "peak_source": f"bf16 sustained, {src}",
                          "flops_per_token": f_tok},
        "roofline": {"bound": "tensor", "kernel": "gemm_split_bf16 (all GEMM launches of one step)",
                     "achieved": gemm_tflops, "peak": sustained, "unit": "TFLOP/s",
                     "frac": gemm_tflops / sustained,
                     "traffic": traffic["bytes_per_step"] / r["gemm_n"] if traffic else None,
                     "traffic_note": (f"mean DRAM bytes per GEMM launch (ncu dram__bytes_read+write over "
                                      f"{traffic['launches']} GEMM launches of one step, {traffic['source']}); "
                                      f"algorithmic operand+output bytes per launch "
                                      f"{alg_bytes / r['gemm_n']:.3e}")
                     if traffic else None,
                     "gemm_launches_per_step": r["gemm_n"],
                     "mma_passes": "3 (forward, dX), 1 fp16 (dW)" if f16w else 3,
                     "peak_source": f"bf16 sustained, {src}"},
        "kernel_ms": {k: round(v, 4) for k, v in sorted(r["per_kind"].items(), key=lambda kv: -kv[1])},
        "kernel_share": {k: round(v / tot, 4) for k, v in r["per_kind"].items()} if tot > 0 else {},
        "e2e": {"value": tokens / (r["e2e_s"] / args.steps), "unit": "tokens/s", "h2d_bytes_per_step": r["h2d"],
                "d2h_bytes_per_step": 8},
        "gpu_launches": r["launches"] * args.steps,
        "clocks": r["clocks"],
        "cpu_baseline": cpu,
    }
    if qlora:
        qwl = WORKLOADS["smollm2_qlora_b8_t512"]
        qf = step_flops_per_token(cfg, T, 1, qwl["lora"], 8)
        qv = qwl["B"] * qwl["T"] * world / (qlora["step_ms"] * 1e-3) if not args.batch else \
            N * world / (qlora["step_ms"] * 1e-3)
        line["qlora_step"] = {
            "workload": "smollm2_qlora_b8_t512", "lora": "q,v rank 8 alpha 16 over a frozen Q8_0 base",
            "q8_ring_l2_resident": bool(args.q8_ring_l2),
            "value": qv, "unit": "tokens/s", "ms_per_step": qlora["step_ms"], "steps": args.steps,
            "step_roofline": {"tflops_algorithmic": qf * qv / world / 1e12, "peak_tflops": sustained,
                              "frac": qf * qv / world / 1e12 / sustained, "flops_per_token": qf},
            "e2e": {"value": qv * qlora["step_ms"] * 1e-3 / (qlora["e2e_s"] / args.steps), "unit": "tokens/s",
                    "h2d_bytes_per_step": qlora["h2d"], "d2h_bytes_per_step": 8},
            "gpu_launches": qlora["launches"] * args.steps, "clocks": qlora["clocks"]}
    print(json.dumps(line), flush=True)
    if dp:
        dp.close()


if __name__ == "__main__":
    main()
