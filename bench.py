#!/usr/bin/env python
"""Benchmark of the QVex hot path on B200: 4-bit g64 qmv over one decode step.

Workload (the decode-step case the headline metric is quoted on): every
4-bit group-64 linear of one decode step of a Qwen3.5-9B-shaped model (24 gated-DeltaNet
+ 8 gated-attention layers, hidden 4096, MLP 12288, vocab 248320; 145 projections,
4.464 GB of packed weights), applied to x bf16 [M, K] ~ N(0,1) with M = 1.  Weights are
synthetic (seeded): codes uniform 0..15, scales |N(0,1)|*0.002, biases -8*scale.  One
"step" is the 145 qmv launches of one decode step, replayed from a CUDA graph (the
launches carry programmatic-dependent-launch edges).  The weights total 4.46 GB, far
above the 126 MB L2, so no flush is needed between steps.

With --gpus N (torchrun, one rank per GPU) the step is tensor-parallel: the projections that
feed a local nonlinearity (DeltaNet in_proj, attention q/k/v, MLP gate_up) keep 1/N of their
output rows on each rank and exchange nothing; the projections that close a block (out_proj,
o_proj, down) keep 1/N of their input columns and sum their partial outputs over the ranks;
lm_head keeps 1/N of its rows and is gathered.  By default both exchanges run inside the qmv
kernel (qvx_qmv_fused: partial sums, or output rows, stored into the peers' inboxes over
NVLink as words tagged with the launch; no NCCL call inside the step), 65 per step;
--gather nccl runs the local kernels followed by NCCL all-reduces / all-gathers instead.
Strong scaling: the whole job's work is fixed.  After the timed region each rank checks
lm_head bit for bit and a row-parallel projection against the unsharded kernel, and reads
the device status word; the result goes into the JSON line.

Prints ONE JSON line (rank 0).  `--impl reference` times the reference's arithmetic on
the host CPU cores instead (the oracle port of engine/kernels.py's qmv arithmetic: MLX,
which the reference uses, is not installed here), on a bounded row sample of the same
workload.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qvex-3.5_b200"))

METRIC = "4-bit qmv HBM GB/s (M=1) & %peak; decode tok/s Qwen3.5-9B-shape at 1/2/4/8 GPU"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=1, help="tokens per step (1 = batch-1 decode)")
    ap.add_argument("--layers", type=int, default=32, help="decoder layers (32 = the full 9B shape)")
    ap.add_argument("--gather", choices=("fused", "nccl"), default="fused",
                    help="N>1: all-gather fused into the qmv kernel (peer stores over NVLink) or NCCL")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the M=2/4/8 side measurements")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the model-level decode (random-init 9B-shaped model, batch 1 and batch 64)")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the config-2/3 kernel measurements (prefill qmm, quantize, gated DeltaNet)")
    ap.add_argument("--profile", nargs="?", const="step", default=None,
                    choices=["step", "qmm", "qmm_small", "quantize", "gd_prefill", "gd_decode", "model_decode",
                             "attn_decode"],
                    help="run one case eagerly for a profiler (no graph, clocks or CPU baseline)")
    return ap.parse_args()


# ------------------------------------------------------------------ config 2 / 3 kernels

def _cuda_time(torch, fn, reps, warm=3):
    """Device time per call (ms) of `fn` replayed from a CUDA graph of `reps` calls, so host
    overhead of the Python wrapper is not counted."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) / reps  # ms


def config_cases(torch, device, small=False):
    """Inputs of the quantize + prefill-qmm case (W ~ N(0, 0.02) [12288, 4096], x [2048, 4096])."""
    import qvex
    g = torch.Generator(device=device)
    g.manual_seed(0)
    N, K, M = (4096, 4096, 512) if small else (12288, 4096, 2048)
    W = (torch.randn((N, K), device=device, generator=g) * 0.02).to(torch.bfloat16)
    wq, s, b = qvex.quantize(W)
    x = torch.randn((M, K), device=device, generator=g).to(torch.bfloat16)
    return {"W": W, "wq": wq, "s": s, "b": b, "x": x, "M": M, "N": N, "K": K}


def gd_case(torch, device, B, T):
    """Config 3: Hk=16, Hv=32, D=128; q, k L2-normalised, v ~ N(0,1), a, b ~ N(0,1),
    A_log = dt_bias = 0 (log-decay = -softplus(a), beta = sigmoid(b)), state N(0,1)*0.1."""
    g = torch.Generator(device=device)
    g.manual_seed(3)
    Hk, Hv, D = 16, 32, 128
    q = torch.nn.functional.normalize(torch.randn((B, T, Hk, D), device=device, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn((B, T, Hk, D), device=device, generator=g), dim=-1)
    v = torch.randn((B, T, Hv, D), device=device, generator=g)
    a = torch.randn((B, T, Hv), device=device, generator=g)
    bb = torch.randn((B, T, Hv), device=device, generator=g)
    st = torch.randn((B, Hv, D, D), device=device, generator=g) * 0.1
    z = torch.zeros(Hv, device=device)
    bf = torch.bfloat16
    return (q.to(bf), k.to(bf), v.to(bf), a.to(bf), bb.to(bf), z, z, st.float())


def measure_configs(torch, device, hbm_peak, tc_peak):
    """Device-timed throughput of the config-2 and config-3 kernels with their rooflines."""
    import qvex
    out = {}
    # config 0: one [12288, 4096] projection at M = 1 (28.3 MB of weights, inside L2), so six
    # seeded weight copies (170 MB) rotate to make every launch stream from HBM
    from qvex.model import QLinear
    from qvex.shapes import qmv_bytes
    g0 = torch.Generator(device=device)
    g0.manual_seed(0)
    N0, K0 = 12288, 4096
    x0 = torch.randn((1, K0), device=device, generator=g0).to(torch.bfloat16)
    copies = []
    for _ in range(6):
        w0 = torch.randint(-2 ** 31, 2 ** 31, (N0, K0 // 8), dtype=torch.int64, device=device, generator=g0)
        s0 = (torch.randn((N0, K0 // 64), device=device, generator=g0).abs() * 0.002).to(torch.bfloat16)
        copies.append(QLinear(w0.to(torch.int32), s0, (-8.0 * s0.float()).to(torch.bfloat16), 64, 4))
    y0 = torch.empty((1, N0), dtype=torch.bfloat16, device=device)
    it0 = iter(range(1 << 30))
    ms = _cuda_time(torch, lambda: copies[next(it0) % 6](x0, out=y0), 60)
    b0 = qmv_bytes(1, N0, K0)
    out["qmv_config0"] = {"ms": round(ms, 5), "gbs": round(b0 / ms / 1e6, 1), "frac_hbm": round(b0 / ms / 1e6 / hbm_peak, 3),
                          "bytes": b0, "note": "one launch per call, graph of 60 calls over 6 rotated weight copies"}
    del copies
    c = config_cases(torch, device)
    M, N, K = c["M"], c["N"], c["K"]
    # quantize / pack: reads bf16 W, writes codes + scales + biases; two copies of W
    # alternate so that 200 MB of inputs (> 126 MB L2) are streamed
    qb = N * K * 2 + N * K // 2 + N * (K // 64) * 4
    Ws = [c["W"], c["W"].clone()]
    it = iter(range(1 << 30))
    ms = _cuda_time(torch, lambda: qvex.quantize(Ws[next(it) & 1]), 20)
    del Ws
    out["quantize_config2"] = {"ms": round(ms, 4), "gbs": round(qb / ms / 1e6, 1),
                               "frac_hbm": round(qb / ms / 1e6 / hbm_peak, 3), "bytes": qb}
    # prefill qmm (tcgen05): 2 M N K flops, prepasses included
    ws = torch.empty(qvex.qmm_workspace_size(M, N, K), dtype=torch.uint8, device=device)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=device)
    ms = _cuda_time(torch, lambda: qvex.quantized_matmul(c["x"], c["wq"], c["s"], c["b"], out=y, workspace=ws), 20)
    fl = 2.0 * M * N * K
    out["qmm_config2"] = {"ms": round(ms, 4), "tflops": round(fl / ms / 1e9, 1),
                          "frac_bf16_dense": round(fl / ms / 1e9 / tc_peak, 3), "M": M, "N": N, "K": K}
    # batched decode through qmm (M = 64 tokens; the tiles do not fill the SMs, so K is
    # split across them): five weight copies rotate so that they stream from HBM
    Mb = 64
    xb = c["x"][:Mb].contiguous()
    wqs = [c["wq"]] + [c["wq"].clone() for _ in range(4)]
    ws_b = torch.empty(qvex.qmm_workspace_size(Mb, N, K), dtype=torch.uint8, device=device)
    yb = torch.empty((Mb, N), dtype=torch.bfloat16, device=device)
    it = iter(range(1 << 30))
    # the weight prepass made once, as QLinear does for its constant weights (the copies
    # share scales and biases)
    prep_b = qvex.core.qmm_prepare(c["s"], c["b"])
    ms = _cuda_time(torch, lambda: qvex.quantized_matmul(xb, wqs[next(it) % 5], c["s"], c["b"], out=yb,
                                                         workspace=ws_b, prep=prep_b), 20)
    wbytes = N * K // 2 + N * (K // 64) * 4
    out["qmm_batch64"] = {"ms": round(ms, 4), "weight_gbs": round(wbytes / ms / 1e6, 1),
                          "frac_hbm": round(wbytes / ms / 1e6 / hbm_peak, 3),
                          "tflops": round(2.0 * Mb * N * K / ms / 1e9, 1), "M": Mb, "N": N, "K": K,
                          "prepared_weights": True}
    del wqs, ws_b, yb, xb, prep_b
    del c, ws, y
    # q/k conditioning in front of the recurrence (config-3 shape, T = 2048, B = 8):
    # bf16 in and out, 4 bytes per element, 268 MB per call
    g = torch.Generator(device=device)
    g.manual_seed(4)
    qk = [torch.randn((8, 2048, 16, 128), device=device, generator=g).to(torch.bfloat16) for _ in range(2)]
    ms = _cuda_time(torch, lambda: qvex.qk_condition(qk[0], qk[1]), 10)
    qkb = 2 * qk[0].numel() * 4
    out["qk_condition_B8_T2048"] = {"ms": round(ms, 4), "gbs": round(qkb / ms / 1e6, 1),
                                    "frac_hbm": round(qkb / ms / 1e6 / hbm_peak, 3)}
    del qk
    # sampling after lm_head (engine/sampler.py defaults: T 0.6, top_p 0.95, top_k 20) on a
    # bf16 logits row of the Qwen vocabulary: scores + pick, one token
    logits = (torch.randn((1, 248320), device=device, generator=g) * 3).to(torch.bfloat16)
    ms = _cuda_time(torch, lambda: qvex.sample_pick(qvex.sample_scores(logits), greedy=False, seed=1, offset=1), 20)
    out["sampler_V248320"] = {"ms": round(ms, 4), "tokens_per_s": round(1e3 / ms, 1)}
    del logits
    # gated DeltaNet: decode step (HBM: state in + out) and 2048-step prefill (serial in T)
    for B, T in ((1, 1), (8, 1), (1, 2048), (8, 2048)):
        args = gd_case(torch, device, B, T)
        # decode steps rotate over enough distinct states (>= 256 MB) that they come from HBM
        n_st = max(1, (256 << 20) // (B * 32 * 128 * 128 * 4)) if T == 1 else 1
        states = [args[-1]] + [args[-1].clone() for _ in range(n_st - 1)]
        outs = [torch.empty_like(args[-1]) for _ in range(n_st)]
        it = iter(range(1 << 30))

        def call():
            i = next(it) % n_st
            return qvex.gated_delta(*args[:-1], states[i], out_state=outs[i])
        ms = _cuda_time(torch, call, 10 if T > 1 else 2 * n_st)
        del states, outs
        state_bytes = B * 32 * 128 * 128 * 4 * 2
        io_bytes = B * T * (2 * 16 * 128 + 2 * 32 * 128 + 2 * 32) * 2
        flops = 7.0 * 128 * 128 * 32 * B * T
        out[f"gated_delta_B{B}_T{T}"] = {"ms": round(ms, 4), "steps_per_s": round(T / ms * 1e3, 1),
                                        "gbs": round((state_bytes + io_bytes) / ms / 1e6, 1),
                                        "fp32_tflops": round(flops / ms / 1e9, 3)}
    return out


def measure_model(torch, device, peak_gbs, world=1, rank=0, dist=None, decode_steps=256, prefill=4096, batch=64,
                  batch_prefill=128):
    """Model-level decode of a random-initialised Qwen3.5-9B-shaped 4-bit model (config 4):
    batch 1 after a `prefill`-token prompt (fed in 512-token chunks, as the reference's engine
    does), and `batch` sequences after `batch_prefill`-token prompts; greedy decode replayed
    from one CUDA graph per step (tokens and position stay on the device).  With `world` > 1
    the model is tensor-parallel (qvex.tp: heads and MLP slices per rank, row-parallel block
    outputs summed inside the projection kernels for batch <= 8, by NCCL above).  Device-timed
    with CUDA events, max over ranks; the weights (5 GB with the embedding) exceed L2."""
    from qvex.qwen35 import Config, DecodeGraph, Qwen35, random_params
    from qvex.sampler import sample_pick, sample_scores
    from qvex.shapes import Qwen35Shape, qlinear_bytes
    cfg = Config.qwen35_9b()
    if world > 1:
        from qvex import tp as TPM
        P = random_params(cfg, 0, device)
        lcfg, LP = TPM.shard_params(cfg, P, world, rank)
        del P
        model = Qwen35.from_params(lcfg, LP)
        TPM.attach(model, TPM.TP(None, world, rank, cfg.vocab_size))
    else:
        model = Qwen35.random(cfg, seed=0, device=device)
    weight_bytes = sum(qlinear_bytes(N, K) for _, N, K in Qwen35Shape().decode_linears())
    g = torch.Generator(device=device)
    g.manual_seed(5)

    def max_ms(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    out = {}
    for B, P in ((1, prefill), (batch, batch_prefill)):
        cache = model.make_cache(capacity=P + decode_steps + 8)
        ids = torch.randint(0, cfg.vocab_size, (B, P), device=device, generator=g, dtype=torch.int64).to(torch.int32)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for c0 in range(0, P, 512):
            logits = model(ids[:, c0:c0 + 512].contiguous(), cache, last_only=True)
        e1.record()
        torch.cuda.synchronize()
        prefill_ms = max_ms(e0.elapsed_time(e1))
        first = sample_pick(sample_scores(logits.view(B, -1), temperature=0.0), True).view(B, 1)
        dg = DecodeGraph(model, cache, first, pos=P)
        n_warm = 3
        for _ in range(n_warm):
            dg.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0.record()
        steps = decode_steps - n_warm
        for _ in range(steps):
            dg.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = max_ms(e0.elapsed_time(e1)) / steps
        key = "batch1" if B == 1 else f"batch{B}"
        out[key] = {"tok_per_s": round(B * 1e3 / ms, 1), "ms_per_step": round(ms, 4), "context": P,
                    "decode_steps": steps, "prefill_ms": round(prefill_ms, 1),
                    "prefill_tok_per_s": round(B * P / prefill_ms * 1e3, 1),
                    "weight_gbs": round(weight_bytes / ms / 1e6, 1),
                    "frac_hbm_weights_per_gpu": round(weight_bytes / world / ms / 1e6 / peak_gbs, 3)}
        del dg, cache
    if world > 1:
        from qvex import tp as TPM
        TPM.close(model)
    del model
    torch.cuda.empty_cache()
    return out


def profile_case(torch, device, case, reps):
    """One eagerly-launched case for ncu (small enough for a full-section capture).
    model_decode: prefill 4096 tokens outside the profiler range, then `reps` eager decode
    steps of the 9B-shaped model inside it (ncu --profile-from-start off)."""
    import qvex
    if case == "model_decode":
        from qvex.qwen35 import Config, Qwen35
        cfg = Config.qwen35_9b()
        model = Qwen35.random(cfg, seed=0, device=device)
        cache = model.make_cache(capacity=4096 + reps + 8)
        g = torch.Generator(device=device)
        g.manual_seed(5)
        ids = torch.randint(0, cfg.vocab_size, (1, 4096), device=device, generator=g, dtype=torch.int64).to(torch.int32)
        for c0 in range(0, 4096, 512):
            model(ids[:, c0:c0 + 512].contiguous(), cache, last_only=True)
        model.prepare_decode(cache, 1, device)
        pos = torch.tensor([4096], dtype=torch.int32, device=device)
        tok = ids[:, -1:].contiguous()
        model.decode_step(tok, cache, pos)  # warm (module loads) outside the range
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        for _ in range(reps):
            model.decode_step(tok, cache, pos)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"profile_run": case, "reps": reps}))
        return
    if case == "attn_decode":
        # one layer's decode attention: 1 sequence, 32 query / 8 KV heads of 128, 4096 cached
        # positions (16.8 MB of keys and values), 18 key ranges (the model's split at B = 1)
        from qvex import glue
        H, Hkv, D, pos = 32, 8, 128, 4096
        g = torch.Generator(device=device)
        g.manual_seed(0)
        qkv = torch.randn((1, 1, (2 * H + 2 * Hkv) * D), device=device, generator=g).to(torch.bfloat16)
        kc = torch.randn((1, Hkv, pos + 64, D), device=device, generator=g).to(torch.bfloat16)
        vc = torch.randn_like(kc)
        qn = torch.ones(D, device=device, dtype=torch.bfloat16)
        inv = glue.rope_inv_freq(32, 1e7, device)
        ns = glue.default_splits(1, Hkv, device)
        ws = glue.attention_workspace(1, Hkv, H // Hkv, 1, D, ns, device)
        for _ in range(reps):
            glue.attention(qkv, qn, qn, 1e-6, inv, kc, vc, pos, H, Hkv, D, workspace=ws, nsplit=ns)
        torch.cuda.synchronize()
        print(json.dumps({"profile_run": case, "reps": reps, "nsplit": ns}))
        return
    if case in ("qmm", "qmm_small"):
        c = config_cases(torch, device, small=(case == "qmm_small"))
        for _ in range(reps):
            qvex.quantized_matmul(c["x"], c["wq"], c["s"], c["b"])
    elif case == "quantize":
        c = config_cases(torch, device)
        for _ in range(reps):
            qvex.quantize(c["W"])
    else:
        B, T = (8, 2048) if case == "gd_prefill" else (8, 1)
        args = gd_case(torch, device, B, T)
        for _ in range(reps):
            qvex.gated_delta(*args)
    torch.cuda.synchronize()
    print(json.dumps({"profile_run": case, "reps": reps}))


# ------------------------------------------------------------------ environment

def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def tc_peak() -> float:
    """Dense bf16 tensor peak (TFLOP/s): measured burst figure, else the fallback."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0, t1, gpu_indices):
        sel = [p for (t, p) in self.samples if t0 - 0.15 <= t <= t1 + 0.15 and p[0] in gpu_indices]
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(p[1]) for p in sel if num(p[1]) is not None]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for p in sel:
            for name, v in zip(names, p[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(sel[0][2]),
                "reasons": sorted(reasons), "samples": len(sel)}


# ------------------------------------------------------------------ workload

ROW_PARALLEL = ("out_proj", "o_proj", "down")


def build_weights(torch, shape, rank, world, device, seed=0):
    """Synthetic 4-bit g64 weights of one decode step, this rank's shard of each: with
    `world` > 1 the projections that feed a local nonlinearity (DeltaNet in_proj, attention
    q/k/v, MLP gate_up) keep 1/world of their output rows (column-parallel, no exchange), the
    projections that close a block (out_proj, o_proj, down) keep 1/world of their input
    columns (row-parallel, partial sums reduced over the ranks), and lm_head keeps 1/world of
    its rows (gathered).  Returns (name, N, K, local QLinear, kind) per projection, kind in
    "col", "row", "gather"."""
    from qvex.model import QLinear
    lins = []
    g = torch.Generator(device=device)
    for i, (name, N, K) in enumerate(shape.decode_linears()):
        kind = "col" if world == 1 else "row" if name.endswith(ROW_PARALLEL) else "gather" if name == "lm_head" else "col"
        g.manual_seed(seed * 100003 + i)
        # all 2^32 patterns equally likely => every 4-bit code uniform in 0..15
        w = torch.randint(-2 ** 31, 2 ** 31, (N, K // 8), dtype=torch.int64, device=device, generator=g).to(torch.int32)
        s = (torch.randn((N, K // 64), device=device, generator=g).abs() * 0.002).to(torch.bfloat16)
        if kind == "row":
            if K % (512 * world):
                raise ValueError(f"{name}: K={K} does not split over {world} ranks in 512-column slices")
            k = K // world
            w = w[:, rank * k // 8:(rank + 1) * k // 8].contiguous()
            s = s[:, rank * k // 64:(rank + 1) * k // 64].contiguous()
        else:
            if N % world:
                raise ValueError(f"{name}: N={N} does not split over {world} ranks")
            n = N // world
            w = w[rank * n:(rank + 1) * n].contiguous()
            s = s[rank * n:(rank + 1) * n].contiguous()
        b = (-8.0 * s.float()).to(torch.bfloat16)
        lins.append((name, N, K, QLinear(w, s, b, 64, 4), kind))
    return lins


def full_linear(torch, shape, index, device, seed=0):
    """Projection `index` of build_weights, unsharded (the same seeded generator)."""
    from qvex.model import QLinear
    name, N, K = shape.decode_linears()[index]
    g = torch.Generator(device=device)
    g.manual_seed(seed * 100003 + index)
    w = torch.randint(-2 ** 31, 2 ** 31, (N, K // 8), dtype=torch.int64, device=device, generator=g).to(torch.int32)
    s = (torch.randn((N, K // 64), device=device, generator=g).abs() * 0.002).to(torch.bfloat16)
    b = (-8.0 * s.float()).to(torch.bfloat16)
    return QLinear(w, s, b, 64, 4)


def gather_check(torch, dist, shape, lins, xin, full_out, world, device):
    """After the timed replays: every rank recomputes two projections unsharded with the
    single-GPU kernel.  lm_head (gathered rows) must match bit for bit (a row's arithmetic
    does not depend on how the rows are split); the first down projection (row-parallel,
    partial sums reduced over the ranks in rank order) within rel-L2 1e-3 and bit-identical
    on every rank.  Returns "ok" or the first mismatch."""
    names = [l[0] for l in lins]
    i_lm = len(lins) - 1
    i_down = next(i for i, n in enumerate(names) if n.endswith("down"))
    name, N, K, _, _ = lins[i_lm]
    ref = full_linear(torch, shape, i_lm, device)(xin["full"][K])
    got = full_out[i_lm]
    got = got.reshape(ref.shape) if got.dim() == 2 else got.permute(1, 0, 2).reshape(ref.shape)
    torch.cuda.synchronize()
    if not torch.equal(got.view(torch.int16), ref.view(torch.int16)):
        bad = int((got.view(torch.int16) != ref.view(torch.int16)).sum())
        return f"{name}: {bad} of {ref.numel()} outputs differ"
    del ref
    name, N, K, _, _ = lins[i_down]
    ref = full_linear(torch, shape, i_down, device)(xin["full"][K]).float()
    got = full_out[i_down].reshape(ref.shape)
    rel = float((got.float() - ref).norm() / ref.norm())
    if rel > 1e-3:
        return f"{name}: rel-L2 {rel:.2e} against the unsharded projection"
    parts = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(parts, got.contiguous())
    if not all(torch.equal(p.view(torch.int16), parts[0].view(torch.int16)) for p in parts):
        return f"{name}: the reduced output differs between ranks"
    return "ok"


def run_ours(args):
    import torch
    import torch.distributed as dist

    from qvex.shapes import Qwen35Shape, qlinear_bytes, qmv_bytes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    import qvex
    qvex.load_library()

    if args.profile and args.profile != "step":
        profile_case(torch, device, args.profile, max(args.warmup, 1))
        return

    shape = Qwen35Shape(layers=args.layers)
    M = args.m
    lins = build_weights(torch, shape, rank, world, device)
    Ks = sorted({K for _, _, K, _, _ in lins})
    g = torch.Generator(device=device)
    g.manual_seed(1234)
    xs = {K: torch.randn((M, K), device=device, generator=g).to(torch.bfloat16) for K in Ks}
    # row-parallel projections read this rank's slice of their input columns
    xs_row = {K: xs[K][:, rank * (K // world):(rank + 1) * (K // world)].contiguous() for K in Ks}
    xin = {"full": xs, "row": xs_row}
    inputs = [xs_row[K] if kind == "row" else xs[K] for _, _, K, _, kind in lins]
    local_out = [torch.empty((M, l.out_features), dtype=torch.bfloat16, device=device) for _, _, _, l, _ in lins]
    launches_per_step = len(lins)
    fused = world > 1 and args.gather == "fused"
    peer = None
    if fused:
        # lm_head's gather region and one reduce slot per row-parallel projection, mapped into
        # every rank (CUDA IPC); the exchanges run inside the projection kernels
        from qvex.core import qmv_fused
        from qvex.shard import PeerGather, qmv_allgather
        rows = [i for i, l in enumerate(lins) if l[4] == "row"]
        i_lm = len(lins) - 1
        peer = PeerGather([M * lins[i_lm][1] * 2], reduce=[(M, lins[i][1]) for i in rows])
        gdesc = peer.descriptor(peer.reserve(), lins[i_lm][1], rank * (lins[i_lm][1] // world))
        rdesc = {i: peer.reduce_descriptor(peer.reserve_reduce(), lins[i][1]) for i in rows}
        full_out = [torch.empty((M, N), dtype=torch.bfloat16, device=device) if kind == "row" else
                    peer.output(gdesc.slot, M, N) if kind == "gather" else None for _, N, _, _, kind in lins]
    else:
        full_out = [torch.empty((M, N), dtype=torch.bfloat16, device=device) if kind == "row" else
                    torch.empty((world, M, N // world), dtype=torch.bfloat16, device=device) if kind == "gather"
                    else None for _, N, _, _, kind in lins]

    def step_qmv():
        for (_, _, K, lin, kind), x, out in zip(lins, inputs, local_out):
            lin(x, out=out)

    def step_full():
        for i, ((_, _, K, lin, kind), x, out) in enumerate(zip(lins, inputs, local_out)):
            if kind == "col":
                lin(x, out=out)
            elif fused and kind == "row":
                qmv_fused(x, lin.w, lin.scales, lin.biases, gather=rdesc[i], out=full_out[i])
            elif fused:
                qmv_allgather(lin, x, gdesc)
            elif kind == "row":
                lin(x, out=full_out[i])
                dist.all_reduce(full_out[i])
            else:
                lin(x, out=out)
                dist.all_gather_into_tensor(full_out[i], out)

    if args.profile:
        for _ in range(max(args.warmup, 1)):
            step_full()
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"profile_run": True, "launches_per_step": launches_per_step}))
        if peer is not None:
            peer.close()
        if world > 1:
            dist.destroy_process_group()
        return

    # warm the kernels (occupancy queries, module load) before capture
    step_full()
    torch.cuda.synchronize()
    graph_full = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_full):
        step_full()
    graph_q = graph_full
    if world > 1:
        graph_q = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_q):
            step_qmv()

    def timed(graph, steps, warmup):
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.time()
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        t1 = time.time()
        ms = e0.elapsed_time(e1)
        if world > 1:
            dist.barrier()
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, t0, t1

    clocks = ClockSampler().start() if rank == 0 else None
    ms_total, t0, t1 = timed(graph_full, args.steps, args.warmup)
    if clocks:
        clocks.stop()
    ms_q, _, _ = timed(graph_q, args.steps, 3) if world > 1 else (ms_total, t0, t1)

    bytes_full = sum(qmv_bytes(M, N, K) for _, N, K, _, _ in lins)            # whole job, per step
    bytes_rank = sum(qmv_bytes(M, l.out_features, l.in_features) for _, _, _, l, _ in lins)  # this rank's
    weight_bytes = sum(qlinear_bytes(N, K) for _, N, K, _, _ in lins)
    ms_step = ms_total / args.steps
    value = bytes_full / (ms_step * 1e-3) / 1e9
    achieved = bytes_rank / (ms_q / args.steps * 1e-3) / 1e9   # per-GPU qmv bytes / per-GPU qmv time
    peak, peak_kind = peaks()

    # side measurement: lm_head qmv alone (572 MB, one launch), events around each launch
    lm = lins[-1][3]
    lm_out = local_out[-1]
    for _ in range(3):
        lm(xs[4096], out=lm_out)
    torch.cuda.synchronize()
    reps = 20
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in ev:
        a.record()
        lm(xs[4096], out=lm_out)
        b.record()
    torch.cuda.synchronize()
    lm_ms = statistics.median(a.elapsed_time(b) for a, b in ev)
    lm_gbs = qmv_bytes(M, lins[-1][1] // world, 4096) / (lm_ms * 1e-3) / 1e9

    # e2e through the public API: host x -> device, the captured QLinear calls, logits -> host,
    # synchronised every step (a decode loop needs the logits before the next token)
    pin_x = {K: xs[K].cpu().pin_memory() for K in Ks}
    logits_dev = full_out[-1] if world > 1 else local_out[-1]
    pin_y = torch.empty(logits_dev.shape, dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * 2 for t in pin_x.values())
    d2h = pin_y.numel() * 2
    e2e_steps = max(min(args.steps, 200), 10)
    stream = torch.cuda.current_stream()
    for i in range(e2e_steps + 3):
        if i == 3:
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            te0 = time.perf_counter()
        for K in Ks:
            xs[K].copy_(pin_x[K], non_blocking=True)
            if world > 1:  # this rank's input columns of the row-parallel projections
                xs_row[K].copy_(xs[K][:, rank * (K // world):(rank + 1) * (K // world)])
        graph_full.replay()
        pin_y.copy_(logits_dev, non_blocking=True)
        stream.synchronize()
    te1 = time.perf_counter()
    e2e_s = te1 - te0
    if world > 1:
        t = torch.tensor([e2e_s], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_val = bytes_full * e2e_steps / e2e_s / 1e9

    # multi-GPU correctness: the gathered outputs of the last replay against the unsharded
    # kernel on every rank, and the device status word (a bounded wait that gave up)
    check = None
    if world > 1:
        graph_full.replay()
        torch.cuda.synchronize()
        verdict = gather_check(torch, dist, shape, lins, xin, full_out, world, device)
        status = qvex._lib.device_status(torch.cuda.current_stream().cuda_stream)
        flags = [None] * world
        dist.all_gather_object(flags, (verdict, status))
        check = {"gather_check": "ok" if all(v == "ok" for v, _ in flags) else [v for v, _ in flags],
                 "device_status": max(st for _, st in flags),
                 "checked": "lm_head (gathered) bit for bit and the first down (row-parallel, reduced) within "
                            "rel-L2 1e-3 against the unsharded kernel on every rank, and bit-identical across ranks"}

    extra = {}
    if not args.no_extra and world == 1:
        for m2 in (2, 4, 8):
            xs2 = {K: torch.randn((m2, K), device=device, generator=g).to(torch.bfloat16) for K in Ks}
            outs2 = [torch.empty((m2, l.out_features), dtype=torch.bfloat16, device=device) for _, _, _, l, _ in lins]

            def step_m():
                for (_, _, K, lin, _), out in zip(lins, outs2):
                    lin(xs2[K], out=out)
            step_m()
            torch.cuda.synchronize()
            gm = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gm):
                step_m()
            ms_m, _, _ = timed(gm, max(args.steps // 4, 10), 3)
            bm = sum(qmv_bytes(m2, N, K) for _, N, K, _, _ in lins)
            extra[f"M={m2}"] = round(bm / (ms_m / max(args.steps // 4, 10) * 1e-3) / 1e9, 1)
            del gm

    configs = None
    if world == 1 and not args.no_configs:
        configs = measure_configs(torch, device, peak, tc_peak())
    model_dec = None
    if not args.no_model:
        model_dec = measure_model(torch, device, peak, world, rank, dist)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(torch, lins, xs, M, budget_s=3.0)

    if rank == 0:
        clk = clocks.summary(t0, t1, {str(local)}) if clocks else None
        rec = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u4 codes, bf16 x/y, fp32 acc",
            "data": "synthetic (seeded codes/scales/biases as config 0; x ~ N(0,1))",
            "config": {"workload": "config 1: all 145 4-bit g64 linears of one Qwen3.5-9B-shaped decode step",
                       "M": M, "layers": args.layers, "weight_bytes_per_step": weight_bytes,
                       "parallelism": ("single GPU" if world == 1 else
                                       f"tensor-parallel x{world}: in_proj/q/k/v/gate_up column-parallel (no exchange), "
                                       "out_proj/o_proj/down row-parallel with the all-reduce fused into the qmv kernel, "
                                       "lm_head gathered in-kernel (tagged words over NVLink; 65 exchanges per step)"
                                       if fused else f"tensor-parallel x{world}: row-parallel projections all-reduced "
                                       "and lm_head all-gathered by NCCL"),
                       "l2": "inputs larger than L2 (4.46 GB of weights per step)", "cuda_graph": True},
            "tok_per_s": round(1000.0 / ms_step, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic_per_launch(bytes_rank / launches_per_step),
                         "kernel": "qmv_stream_kernel (all 145 launches of the step, gaps included)"},
            "lm_head_qmv": {"gbs": round(lm_gbs, 1), "ms": round(lm_ms, 4), "frac": round(lm_gbs / peak, 4)},
            "qmv_gbs_by_m": extra,
            "e2e": {"value": round(e2e_val, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "tok_per_s": round(e2e_steps / e2e_s, 1),
                    "path": "pinned host x -> QLinear calls captured in a CUDA graph -> pinned host logits, sync/step"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if check:
            rec.update(check)
        if configs:
            rec["configs"] = configs
        if model_dec:
            rec["model_decode"] = model_dec
        if cpu:
            rec["cpu_baseline"] = cpu
        print(json.dumps(rec))
    del graph_full, graph_q
    if peer is not None:
        peer.close()
    if world > 1:
        dist.destroy_process_group()


def traffic_per_launch(algo_bytes_per_launch):
    """DRAM bytes per launch from the committed ncu summary (ratio of measured DRAM bytes
    to algorithmic bytes on the profiled case, applied to this launch size), or None."""
    p = ROOT / "profiles" / "qmv_traffic_ratio.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_over_algorithmic:"):
            return round(float(line.split(":", 1)[1]) * algo_bytes_per_launch)
    return None


# ------------------------------------------------------------------ CPU (reference arithmetic)

def _cpu_sample(torch, lins, xs, M, row_frac):
    """Host copies of the first `row_frac` of every linear's rows."""
    import numpy as np
    sample = []
    for name, N, K, lin, _ in lins:
        n = max(8, int(lin.out_features * row_frac))
        w = lin.w[:n].cpu().numpy().view(np.uint32)
        s = lin.scales[:n].view(torch.int16).cpu().numpy().view(np.uint16)
        b = lin.biases[:n].view(torch.int16).cpu().numpy().view(np.uint16)
        x = xs[K][:M].view(torch.int16).cpu().numpy().view(np.uint16)
        sample.append((x, w, s, b))
    return sample


def _time_cpu(sample, threads, budget_s, min_passes=1):
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    from qvex.shapes import qmv_bytes
    O.set_num_threads(threads)
    byts = sum(qmv_bytes(x.shape[0], w.shape[0], x.shape[1]) for x, w, _, _ in sample)
    for x, w, s, b in sample[:4]:  # warm
        O.qmv_fast(x, w, s, b)
    passes, t0 = 0, time.perf_counter()
    while True:
        for x, w, s, b in sample:
            O.qmv_fast(x, w, s, b)
        passes += 1
        el = time.perf_counter() - t0
        if passes >= min_passes and el >= budget_s:
            break
    return byts * passes / el / 1e9, passes, el, byts


def cpu_baseline(torch, lins, xs, M, budget_s):
    threads = host_threads()
    frac = 1 / 32
    sample = _cpu_sample(torch, lins, xs, M, frac)
    gbs, passes, el, byts = _time_cpu(sample, threads, budget_s)
    return {"value": round(gbs, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"first 1/32 of the rows of all 145 linears ({byts / 1e6:.0f} MB per pass), M={M}, "
                      f"{passes} passes in {el:.1f} s; oracle/qvex_oracle.c orc_qmv_fast (the reference qmv "
                      f"arithmetic, engine/kernels.py:146-174), OpenMP"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch  # only for seeded weight generation (CPU tensors)
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import oracle as O
    from qvex.shapes import Qwen35Shape, qmv_bytes
    shape = Qwen35Shape(layers=args.layers)
    frac = 1 / 64
    g = torch.Generator().manual_seed(0)
    sample = []
    for name, N, K in shape.decode_linears():
        n = max(8, int(N * frac))
        w = torch.randint(-2 ** 31, 2 ** 31, (n, K // 8), dtype=torch.int64, generator=g).to(torch.int32)
        s = (torch.randn((n, K // 64), generator=g).abs() * 0.002).to(torch.bfloat16)
        b = (-8.0 * s.float()).to(torch.bfloat16)
        x = torch.randn((args.m, K), generator=g).to(torch.bfloat16)
        sample.append((x.view(torch.int16).numpy().view(np.uint16), w.numpy().view(np.uint32),
                       s.view(torch.int16).numpy().view(np.uint16), b.view(torch.int16).numpy().view(np.uint16)))
    threads = host_threads()
    O.set_num_threads(threads)
    byts = sum(qmv_bytes(x.shape[0], w.shape[0], x.shape[1]) for x, w, _, _ in sample)

    def one_pass():
        for x, w, s, b in sample:
            O.qmv_fast(x, w, s, b)
    for _ in range(args.warmup):
        one_pass()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_pass()
    el = time.perf_counter() - t0
    value = byts * args.steps / el / 1e9
    rec = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u4 codes, bf16 x/y, fp32 acc",
        "data": "synthetic (seeded codes/scales/biases as config 0; x ~ N(0,1))",
        "config": {"workload": "config 1: all 145 4-bit g64 linears of one Qwen3.5-9B-shaped decode step",
                   "M": args.m, "layers": args.layers, "sample": "first 1/64 of the rows of every linear"},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"first 1/64 of the rows of all 145 linears ({byts / 1e6:.0f} MB per step); "
                                   "MLX (the reference's engine) is not installed, so the reference qmv arithmetic "
                                   "(engine/kernels.py:146-174) runs as the C oracle port orc_qmv_fast, OpenMP"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(rec))


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
