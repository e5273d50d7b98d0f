#!/usr/bin/env python
"""Benchmark of the const-max ring attention layer (Wan2.2-A14B 480x832x81 self-attention).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2|c1|c4]

One step = one self-attention layer through the public API ``wan_cp_self_attention`` (prologue
norms + const-max attention with the d-major epilogue) over this rank's S/N query rows, with K/V
rotated over the ring when N > 1. Default workload C2: S = 32760 tokens (latent 21x60x104, patch
1x2x2), 40 heads x 128, bf16; Q/K/V are a seeded random-init 5120 -> 3x5120 projection of N(0,1)
hidden states with RMSNorm on Q and K plus Wan 3-D RoPE (synthetic stand-in for the reference's
VBench prompts). Metric: whole-job attention TFLOP/s (4*H*S^2*D per layer) and ms/layer.

Under torchrun (N > 1) every rank runs one GPU of the ring (CP = N); times are device times
(CUDA events), max over ranks. ``--impl reference`` times the reference's own CPU attention path
(``_torch_attend``, restated in oracle/) on the host cores; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PKG = "vllm-omni-neuron_b200"
HEADS, HEAD_DIM, HIDDEN = 40, 128, 5120
CONFIGS = {
    "c1": dict(S=4096, latent=None, desc="C1: single-rank full self-attention, B=1 H=40 D=128 S=4096, Q/K/V~N(0,1)*0.5"),
    "c2": dict(S=32760, latent=(21, 60, 104), desc="C2: Wan2.2-A14B 480x832x81 self-attention, S=32760 (21x30x52 tokens), H=40 D=128"),
    "c3": dict(S=32760, latent=None, desc="C3: fused adaLN (LayerNorm eps 1e-6, shift/scale) + FP8 row quant + FP8 QKV projection, T=32760 H=5120 I=15360"),
    "c4": dict(S=75600, latent=(21, 90, 160), desc="C4: Wan2.2-A14B 720x1280x81 self-attention, S=75600 (21x45x80 tokens), H=40 D=128"),
    "c5": dict(S=32760, latent=(21, 60, 104), desc="C5: CFG-parallel Wan2.2-A14B transformer block (self-attn + cross-attn to 512 text tokens + FFN 5120-13824-5120 GELU-tanh), bf16, B=2 (cond/uncond) split CFGP=2 x CP=N/2 (N=1: one branch, CP=1)"),
    "ffn": dict(S=32760, latent=None, desc="Wan FFN of one block on the C2 token count: GELU_tanh(x @ Wu + bu) @ Wd + bd, x [32760, 5120], Wu [5120, 13824], Wd [13824, 5120], bf16"),
    "ffn_fp8": dict(S=32760, latent=None, desc="Wan FFN FP8 leaf (row_mx_mlp, ROW_MX) on the C2 token count: ROW e4m3 x [32760, 5120] -> up GEMM + GELU-tanh + MX-32 quant of the [32760, 13824] intermediate -> block-scaled down GEMM + per-channel scale + bias + gated residual"),
    "oproj": dict(S=32760, latent=None, desc="Output projection of one C2 self-attention layer (d-major [1,40,128,32760] @ [5120,5120] + bias) with the norm2 gated residual and adaLN (LayerNorm + FP8 row quant)"),
}
METRIC = "ring-attn TFLOP/s at S=32760 (one Wan2.2-A14B self-attention layer), CP=N"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------------------ workloads
def make_qkv(cfg: str, device, seed: int = 0):
    """Full-sequence token-major q, k, v [1, S, 40, 128] bf16 on `device` for a config."""
    import torch

    c = CONFIGS[cfg]
    S = c["S"]
    g = torch.Generator(device=device).manual_seed(seed)
    if c["latent"] is None:
        mk = lambda: (torch.randn(1, S, HEADS, HEAD_DIM, generator=g, device=device) * 0.5).to(torch.bfloat16)
        return mk(), mk(), mk()
    rope = importlib.import_module(PKG + ".rope")
    hidden = torch.randn(1, S, HIDDEN, generator=g, device=device).to(torch.bfloat16)
    w = (torch.randn(HIDDEN, 3 * HIDDEN, generator=g, device=device) * 0.02).to(torch.bfloat16)
    qkv = torch.matmul(hidden, w)  # bias 0 (wan2_2_transformer.py:1104)
    del hidden, w
    q, k, v = qkv.split(HIDDEN, dim=-1)

    def rms(x):  # DistributedRMSNorm at TP=1, gamma=1, eps=1e-6 (wan2_2_transformer.py:879-893)
        xf = x.float()
        return (xf / torch.sqrt((xf * xf).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)

    cos, sin = rope.wan_rotary_freqs(HEAD_DIM, (1, 2, 2), 1024, c["latent"], device=device)
    q = rope.apply_rotary_emb_wan(rms(q).unflatten(2, (HEADS, HEAD_DIM)), cos, sin).contiguous()
    k = rope.apply_rotary_emb_wan(rms(k).unflatten(2, (HEADS, HEAD_DIM)), cos, sin).contiguous()
    v = v.unflatten(2, (HEADS, HEAD_DIM)).contiguous()
    del qkv
    assert q.shape[1] == S
    return q, k, v


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples of one GPU while the timed region runs."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": mx,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ------------------------------------------------------------------------------ CPU legs
def cpu_attention_sample(q_rows, k_full, v_full, min_seconds: float):
    """Time the reference's CPU attention path (``_torch_attend``, wan2_2_transformer.py:640-650,
    restated in oracle/attention.py) on a bounded sample. Returns (TFLOP/s, seconds, flops)."""
    from oracle import attention as oat

    scale = 1.0 / math.sqrt(HEAD_DIM)
    flops_one = oat.attention_flops(1, q_rows.shape[1], q_rows.shape[2], k_full.shape[2], HEAD_DIM)
    t0 = time.perf_counter()
    n = 0
    while True:
        oat.torch_attend(q_rows, k_full, v_full, scale)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return flops_one * n / el / 1e12, el, flops_one * n


def cpu_sample_arrays(q, k, v, heads: int, rows: int):
    """[1, heads, rows, D] query sample and [1, heads, S, D] keys/values from device tensors."""
    import numpy as np

    qs = q[:, :rows, :heads].float().cpu().numpy()
    ks = k[:, :, :heads].float().cpu().numpy()
    vs = v[:, :, :heads].float().cpu().numpy()
    tr = lambda x: np.ascontiguousarray(np.transpose(x, (0, 2, 1, 3)))
    return tr(qs), tr(ks), tr(vs)


def cpu_cores() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = max((i.get("num_threads", 0) for i in threadpool_info()), default=0)
        if n:
            return int(n)
    except Exception:
        pass
    return os.cpu_count() or 1


# ------------------------------------------------------------------------------ main
def _claim_stdout():
    """Route everything libraries print (NCCL's version banner, warnings) to stderr; return a
    writer for the real stdout, which carries only the JSON result line."""
    real = os.dup(1)
    os.dup2(2, 1)
    out = os.fdopen(real, "w", buffering=1)

    def emit(obj):
        out.write(json.dumps(obj) + "\n")
        out.flush()

    return emit


def main():
    emit = _claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=list(CONFIGS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tokens", type=int, default=0, help="c3 / oproj / ffn / ffn_fp8: override the token count (small case for profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = CONFIGS[args.config]
    S = cfg["S"]
    flops_layer = 4.0 * HEADS * S * S * HEAD_DIM

    if args.impl == "reference":
        return run_reference(args, world, rank, cfg, flops_layer, emit)
    if args.config == "c3":
        return run_c3(args, emit)
    if args.config == "oproj":
        return run_oproj(args, emit)
    if args.config == "ffn":
        return run_ffn(args, emit)
    if args.config == "ffn_fp8":
        return run_ffn_fp8(args, emit)
    if args.config == "c5":
        return run_c5(args, world, rank, local_rank, emit)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    group = None
    if world > 1:
        from datetime import timedelta

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD
    if S % world:
        raise SystemExit(f"S={S} not divisible by {world}")
    s_loc = S // world

    pkg = importlib.import_module(PKG)
    pkg.build()
    lib = importlib.import_module(PKG + "._lib")

    q, k, v = make_qkv(args.config, dev, seed=0)
    sl = slice(rank * s_loc, (rank + 1) * s_loc)
    ql, kl, vl = (x[:, sl].contiguous() for x in (q, k, v))
    if rank != 0 or world > 1 or args.no_cpu_baseline:
        del q, k, v
        q = k = v = None
    torch.cuda.synchronize()
    scale = 1.0 / math.sqrt(HEAD_DIM)

    def step(qq, kk, vv):
        return pkg.wan_cp_self_attention(qq, kk, vv, scale, world, group, None)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-resident throughput
    for _ in range(args.warmup):
        out = step(ql, kl, vl)
    torch.cuda.synchronize()
    assert lib.device_status() == 0, "device status error during warm-up"
    sampler = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out = step(ql, kl, vl)
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    value = flops_layer / (ms / 1e3) / 1e12

    # ---------------- dominant kernel alone (events on the launching stream)
    L = lib.load()
    st = torch.cuda.current_stream().cuda_stream
    qn2 = torch.empty(HEADS, s_loc, dtype=torch.float32, device=dev)
    km = torch.empty(HEADS, dtype=torch.float32, device=dev)
    o_tmp = torch.empty(1, HEADS, HEAD_DIM, s_loc, dtype=torch.bfloat16, device=dev)
    lib.check(L.vomni_cm_prologue(ql.data_ptr(), kl.data_ptr(), 1, s_loc, HEADS, HEAD_DIM, qn2.data_ptr(), km.data_ptr(), st), "prologue")
    kern_steps = max(3, min(args.steps, 10))
    if True:  # the local-block pass: at N > 1 the largest single launch of the step
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(kern_steps)]
        for a, b in evs:
            a.record()
            lib.check(L.vomni_cm_attend(ql.data_ptr(), kl.data_ptr(), vl.data_ptr(), 1, s_loc, s_loc, 0, s_loc, HEADS, HEAD_DIM, scale,
                                        qn2.data_ptr(), km.data_ptr(), None, None, lib.CM_FINAL | lib.CM_OUT_DMAJOR, o_tmp.data_ptr(), None, st), "attend")
            b.record()
        torch.cuda.synchronize()
        kern_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
        kern_flops = 4.0 * HEADS * s_loc * s_loc * HEAD_DIM
    peaks = {}
    pk_path = ROOT / "MEASURED_PEAKS.json"
    if pk_path.exists():
        peaks = json.loads(pk_path.read_text())
    # The kernel is timed alone (a few back-to-back launches), so the burst cuBLAS figure is its peak.
    peak = peaks.get("bf16_tflops") or 1590.0
    peak_src = "measured (bf16_tflops, burst)" if peaks.get("bf16_tflops") else "fallback (1.59 PFLOP/s)"
    traffic = None
    tr_path = ROOT / "profiles" / "cm_attend_traffic.json"
    if tr_path.exists() and kern_flops:
        t = json.loads(tr_path.read_text())
        m = t.get("measured_launch", {})
        if s_loc == 32760 and world == 1 and m:
            # the C2 launch itself was captured: its DRAM bytes as measured
            traffic = int(m["dram_bytes_read"]) + int(m["dram_bytes_write"])
        else:
            # DRAM bytes per (token, head) of the captured launch, scaled to this launch
            traffic = round(t["dram_bytes_per_token_head"] * s_loc * HEADS)
    roof = None
    if kern_ms:
        ach = kern_flops / (kern_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 2), "peak": peak, "unit": "TFLOP/s", "frac": round(ach / peak, 4),
                "traffic": traffic, "kernel": "cm_attend_pair_kernel", "kernel_ms": round(kern_ms, 4), "peak_source": peak_src}

    # ---------------- exposed ring communication (N > 1): the same pass plan over local data only
    ring_info = None
    if world > 1:
        ring = importlib.import_module(PKG + ".ring")
        plan = ring.phase_plan(world)
        kg = torch.cat([kl] * (world - 1), dim=1).contiguous()
        vg = torch.cat([vl] * (world - 1), dim=1).contiguous()
        acc_o = torch.empty(HEADS, s_loc, HEAD_DIM, dtype=torch.float32, device=dev)
        acc_l = torch.empty(HEADS, s_loc, dtype=torch.float32, device=dev)

        def local_passes():
            lib.check(L.vomni_cm_prologue(ql.data_ptr(), kl.data_ptr(), 1, s_loc, HEADS, HEAD_DIM, qn2.data_ptr(), km.data_ptr(), st), "prologue")
            lib.check(L.vomni_cm_attend(ql.data_ptr(), kl.data_ptr(), vl.data_ptr(), 1, s_loc, s_loc, 0, s_loc, HEADS, HEAD_DIM, scale,
                                        qn2.data_ptr(), km.data_ptr(), acc_o.data_ptr(), acc_l.data_ptr(), 0, None, None, st), "pass0")
            for i, (first, count) in enumerate(plan[1:], start=1):
                fl = lib.CM_ACC_IN | lib.CM_OVERLAP | ((lib.CM_FINAL | lib.CM_OUT_DMAJOR) if i == len(plan) - 1 else 0)
                lib.check(L.vomni_cm_attend(ql.data_ptr(), kg.data_ptr(), vg.data_ptr(), 1, s_loc, (world - 1) * s_loc, first * s_loc,
                                            count * s_loc, HEADS, HEAD_DIM, scale, qn2.data_ptr(), km.data_ptr(), acc_o.data_ptr(),
                                            acc_l.data_ptr(), fl, o_tmp.data_ptr(), None, st), "pass")

        for _ in range(2):
            local_passes()
        torch.cuda.synchronize()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(args.steps):
            local_passes()
        g1.record()
        torch.cuda.synchronize()
        barrier()
        local_ms = max_over_ranks(g0.elapsed_time(g1)) / args.steps
        del kg, vg
        ring_info = {"passes": len(plan), "local_only_ms_per_step": round(local_ms, 4),
                     "exposed_comm_ms": round(ms - local_ms, 4), "exposed_comm_frac": round((ms - local_ms) / ms, 4),
                     "note": "exposed = ring step - the same prologue + pass plan over local K/V only (no copies, no all-reduce)"}

    # ---------------- end to end through the public API with host buffers: pinned host q/k/v in,
    # pinned host output back (the API streams head groups, overlapping PCIe copies with compute)
    qh, kh, vh = (x.cpu().pin_memory() for x in (ql, kl, vl))
    e2e_steps = max(3, min(args.steps, 10))
    e2e_out = {}

    def e2e_step():
        e2e_out["o"] = step(qh, kh, vh)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(e2e_steps):
        e2e_step()
    f1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1)) / e2e_steps
    o_dev = step(ql, kl, vl)
    torch.cuda.synchronize()
    assert e2e_out["o"].device.type == "cpu" and torch.equal(e2e_out["o"], o_dev.cpu()), "host-streamed result differs"
    del o_dev
    bi = 3 * s_loc * HEADS * HEAD_DIM * 2
    bo = s_loc * HEADS * HEAD_DIM * 2
    assert lib.device_status() == 0, "device status error"

    # ---------------- CPU baseline (rank 0, N == 1)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        heads_s, rows_s = 1, 512
        qs, ks, vs = cpu_sample_arrays(q, k, v, heads_s, rows_s)
        try:  # all host threads, also when a launcher pinned OMP_NUM_THREADS=1
            from threadpoolctl import threadpool_limits

            _pool = threadpool_limits(limits=os.cpu_count() or 1)  # noqa: F841
        except Exception:
            pass
        val, el, fl = cpu_attention_sample(qs, ks, vs, min_seconds=10.0)
        cpu = {"value": round(val, 5), "unit": "TFLOP/s", "cores": cpu_cores(), "kind": "port",
               "sample": f"_torch_attend restated (oracle/attention.py torch_attend, numpy fp32): {heads_s} head x {rows_s} query rows x {S} keys, repeated {el:.1f}s ({fl/1e9:.0f} GFLOP)"}

    launches_per_step = 2  # cm_norms_kernel + cm_attend_pair_kernel
    if world > 1:
        ring = importlib.import_module(PKG + ".ring")
        launches_per_step = 1 + len(ring.phase_plan(world))  # prologue + one attention pass per ring pass
    res = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded; random-init projection + RMSNorm + 3-D RoPE, no checkpoint/prompts)"
                if cfg["latent"] else "synthetic (seeded N(0,1)*0.5)",
        "config": attention_config(cfg, world, flops_layer),
        "roofline": roof,
        "cpu_baseline": cpu,
        "clocks": clocks,
        "e2e": {"value": round(flops_layer / (e2e_ms / 1e3) / 1e12, 3), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo},
        "gpu_launches": launches_per_step * args.steps,
    }
    if ring_info is not None:
        res["ring"] = ring_info
    if rank == 0:
        emit(res)
    if world > 1:
        pkg.destroy_rings()
        dist.destroy_process_group()


def run_c3(args, emit):
    """C3 block: adaLN + FP8 row quant (HBM-bound) then the FP8 QKV GEMM (tensor-bound) and the
    across-heads norm + RoPE apply (HBM-bound). Prints one JSON line with each kernel's roofline."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pkg = importlib.import_module(PKG)
    pkg.build()
    lib = importlib.import_module(PKG + "._lib")
    rope = importlib.import_module(PKG + ".rope")
    T, H, I = (args.tokens or 32760), HIDDEN, 3 * HIDDEN
    g = torch.Generator(device=dev).manual_seed(0)
    hidden = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    mods = torch.randn(6, H, generator=g, device=dev) * 0.1
    mul, add = (1 + mods[1]).to(torch.bfloat16), mods[0].to(torch.bfloat16)
    w = torch.randn(H, I, generator=g, device=dev) * 0.02
    wq, chan = pkg.quantize_qkv_weight(w, H, H)
    bias = torch.zeros(I, dtype=torch.bfloat16, device=dev)
    cos, sin = rope.wan_rotary_freqs(HEAD_DIM, (1, 2, 2), 1024, (21, 60, 104), device=dev)
    cos_rh, sin_rh = (x.reshape(-1, HEAD_DIM)[:T].contiguous() for x in rope.rope_rotate_half_caches(cos, sin))
    gamma = torch.ones(H, dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    L = lib.load()
    codes = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=dev)
    scales = torch.empty(T, dtype=torch.float32, device=dev)
    y = torch.empty(T, I, dtype=torch.bfloat16, device=dev)
    sumsq = torch.empty(T, 2 * H // HEAD_DIM, dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > L2: flushed between launches

    def adaln():
        lib.check(L.vomni_adaln_modulate(hidden.data_ptr(), None, mul.data_ptr(), add.data_ptr(), None, T, H, T, 1e-6, 0, 1, 1, 0,
                                         codes.data_ptr(), scales.data_ptr(), None, st), "adaln")

    def gemm():
        lib.check(L.vomni_qkv_fp8_gemm(codes.data_ptr(), scales.data_ptr(), wq.data_ptr(), chan.data_ptr(), bias.data_ptr(),
                                       T, H, I, H, H, y.data_ptr(), sumsq.data_ptr(), st), "gemm")

    # MX-32 variant (UE8M0 per 32 contraction values on activations and weights)
    wmx, _, wmx_sf = pkg.quantize_qkv_weight_mx32(w)
    mx_codes = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=dev)
    mx_scales = torch.empty(T, H // 32, dtype=torch.uint8, device=dev)
    mx_packed = torch.empty(L.vomni_mx_packed_scales_bytes(T, H), dtype=torch.uint8, device=dev)

    def adaln_mx():
        lib.check(L.vomni_adaln_modulate(hidden.data_ptr(), None, mul.data_ptr(), add.data_ptr(), None, T, H, T, 1e-6, 0, 2, 1,
                                         0, mx_codes.data_ptr(), mx_scales.data_ptr(), None, st), "adaln mx32")
        lib.check(L.vomni_mx_pack_scales(mx_scales.data_ptr(), T, H, mx_packed.data_ptr(), st), "pack")

    def gemm_mx():
        lib.check(L.vomni_qkv_mx32_gemm(mx_codes.data_ptr(), mx_packed.data_ptr(), wmx.data_ptr(), wmx_sf.data_ptr(),
                                        bias.data_ptr(), T, H, I, H, H, y.data_ptr(), sumsq.data_ptr(), st), "gemm mx32")

    def apply():
        lib.check(L.vomni_qk_norm_rope(y.data_ptr(), T, I, HEADS, HEADS, HEAD_DIM, sumsq.data_ptr(), 1e-6, gamma.data_ptr(),
                                       gamma.data_ptr(), cos_rh.data_ptr(), sin_rh.data_ptr(), st), "apply")

    def timeit(fn, n):
        ts = []
        for _ in range(n):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    for fn in (adaln, gemm, apply, adaln_mx, gemm_mx):
        for _ in range(args.warmup):
            fn()
    torch.cuda.synchronize()
    n = max(args.steps, 5)
    sampler = ClockSampler(0)
    sampler.start()
    t_ad, t_gm, t_ap = timeit(adaln, n), timeit(gemm, n), timeit(apply, n)
    t_admx, t_gmmx = timeit(adaln_mx, n), timeit(gemm_mx, n)
    clocks = sampler.stop()
    assert lib.device_status() == 0
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    bf16 = peaks.get("bf16_tflops", 1590.0)
    ad_bytes = 2 * T * H + T * H + 4 * T
    ap_bytes = 2 * (2 * T * 2 * H) + T * (2 * H // HEAD_DIM) * 4 + 2 * T * HEAD_DIM * 4
    gm_flops = 2.0 * T * H * I
    admx_bytes = 2 * T * H + T * H + 3 * (T * H // 32)  # bf16 in, codes out, scales out, re-tiled (read + write)
    res = {
        "metric": "C3 fused adaLN + FP8 row quant + FP8 QKV projection (ms per call, per kernel)",
        "value": round(t_ad + t_gm + t_ap, 4), "unit": "ms", "higher_is_better": False, "n_gpus": 1,
        "steps": n, "warmup": args.warmup, "dtype": "fp8 e4m3 (ROW scales) / bf16 I/O", "data": "synthetic",
        "config": {"workload": CONFIGS["c3"]["desc"], "T": T, "H": H, "I": I, "l2": "flushed (256 MB write) before each launch"},
        "kernels": {
            "adaln_rowquant": {"ms": round(t_ad, 4), "bytes": ad_bytes, "GB/s": round(ad_bytes / t_ad / 1e6, 1),
                               "frac_of_measured_hbm": round(ad_bytes / t_ad / 1e6 / hbm, 4)},
            "qkv_fp8_gemm": {"ms": round(t_gm, 4), "flops": gm_flops, "TFLOP/s": round(gm_flops / t_gm / 1e9, 1),
                             "frac_of_measured_bf16_burst_x2": round(gm_flops / t_gm / 1e9 / (2 * bf16), 4)},
            "qk_norm_rope": {"ms": round(t_ap, 4), "bytes": ap_bytes, "GB/s": round(ap_bytes / t_ap / 1e6, 1),
                             "frac_of_measured_hbm": round(ap_bytes / t_ap / 1e6 / hbm, 4)},
            "adaln_mx32quant_and_scale_pack": {"ms": round(t_admx, 4), "bytes": admx_bytes,
                                               "GB/s": round(admx_bytes / t_admx / 1e6, 1),
                                               "frac_of_measured_hbm": round(admx_bytes / t_admx / 1e6 / hbm, 4)},
            "qkv_mx32_gemm": {"ms": round(t_gmmx, 4), "flops": gm_flops, "TFLOP/s": round(gm_flops / t_gmmx / 1e9, 1),
                              "frac_of_measured_bf16_burst_x2": round(gm_flops / t_gmmx / 1e9 / (2 * bf16), 4)},
        },
        "mx32_path_ms": round(t_admx + t_gmmx + t_ap, 4),
        "clocks": clocks,
        "gpu_launches": 6 * n,
    }
    emit(res)


def run_oproj(args, emit):
    """The step after the self-attention: o-projection of the d-major attention output with the gated
    residual fused into its epilogue, then norm2 (adaLN LayerNorm + FP8 row quant), against the
    unfused order (plain projection, then adaLN with its own residual step)."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pkg = importlib.import_module(PKG)
    pkg.build()
    lib = importlib.import_module(PKG + "._lib")
    S, K, H = (args.tokens or 32760), HIDDEN, HIDDEN
    g = torch.Generator(device=dev).manual_seed(0)
    active = torch.randn(1, HEADS, HEAD_DIM, S, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(K, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(H, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    res = torch.randn(1, S, H, generator=g, device=dev).to(torch.bfloat16)
    gate = torch.randn(1, 1, H, generator=g, device=dev) * 0.3
    n2w = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
    n2b = (0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def proj():
        return pkg.wan_o_proj(active, w, bias)

    def fused():
        return pkg.o_proj_gated_residual(active, w, bias, res, gate)

    def fused_norm2():
        return pkg.attn_out_norm2(active, w, bias, res, gate, n2w, n2b, eps=1e-6, quant="row")

    def unfused_norm2():
        y = pkg.wan_o_proj(active, w, bias)
        return pkg.adaln_modulate(y, n2w, n2b, eps=1e-6, quant="row", residual=res, gate=gate)

    # FP8 (ROW) o-projection: per-token row quant of the d-major activation + FP8 ROW GEMM
    w8, w8_scale = pkg.quantize_qkv_weight(w.float(), H, 0)
    codes8 = torch.empty(S, K, dtype=torch.float8_e4m3fn, device=dev)
    scales8 = torch.empty(S, dtype=torch.float32, device=dev)
    L = lib.load()
    st = torch.cuda.current_stream().cuda_stream

    def fp8():
        return pkg.row_mx_o_proj(active, w8, w8_scale, bias)

    def fp8_quant():
        lib.check(L.vomni_oproj_rowquant(active.data_ptr(), 1, K, S, codes8.data_ptr(), scales8.data_ptr(), st), "rowquant")

    def timeit(fn, n):
        ts = []
        for _ in range(n):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    for fn in (proj, fused, fused_norm2, unfused_norm2, fp8, fp8_quant):
        for _ in range(args.warmup):
            fn()
    torch.cuda.synchronize()
    n = max(args.steps, 5)
    sampler = ClockSampler(0)
    sampler.start()
    t_p, t_f, t_fn, t_un = timeit(proj, n), timeit(fused, n), timeit(fused_norm2, n), timeit(unfused_norm2, n)
    t_8, t_8q = timeit(fp8, n), timeit(fp8_quant, n)
    clocks = sampler.stop()
    assert lib.device_status() == 0
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    bf16 = peaks.get("bf16_tflops", 1590.0)
    flops = 2.0 * S * K * H
    emit({
        "metric": "o-projection + norm2 after one C2 self-attention layer (ms per call)",
        "value": round(t_fn, 4), "unit": "ms", "higher_is_better": False, "n_gpus": 1, "steps": n,
        "warmup": args.warmup, "dtype": "bf16 GEMM (fp32 accumulate), fp8 e4m3 row quant out", "data": "synthetic",
        "config": {"workload": CONFIGS["oproj"]["desc"], "S": S, "K": K, "H": H, "l2": "flushed (256 MB write) before each call"},
        "kernels": {
            "oproj_gemm": {"ms": round(t_p, 4), "flops": flops, "TFLOP/s": round(flops / t_p / 1e9, 1),
                           "frac_of_measured_bf16_burst": round(flops / t_p / 1e9 / bf16, 4)},
            "oproj_gemm_gated_residual": {"ms": round(t_f, 4), "TFLOP/s": round(flops / t_f / 1e9, 1)},
            "fused_step": {"ms": round(t_fn, 4), "kernels": "gemm_bf16_pair_kernel<0,1> (residual epilogue) + adaln_kernel"},
            "unfused_step": {"ms": round(t_un, 4), "kernels": "gemm_bf16_pair_kernel<0,0> + adaln_kernel (residual step)"},
            "row_mx_o_proj_fp8": {"ms": round(t_8, 4), "TFLOP/s": round(flops / t_8 / 1e9, 1),
                                  "frac_of_2x_measured_bf16_burst": round(flops / t_8 / 1e9 / (2 * bf16), 4),
                                  "kernels": "oproj_rowquant_kernel + qkv_gemm_pair_kernel<0>"},
            "oproj_rowquant": {"ms": round(t_8q, 4), "bytes": S * K * 2 + S * K + S * 4,
                               "GB/s": round((S * K * 3 + S * 4) / t_8q / 1e6, 1),
                               "frac_of_measured_hbm": round((S * K * 3 + S * 4) / t_8q / 1e6 / peaks.get("hbm_gbs", 6650.0), 4)},
        },
        "clocks": clocks,
        "gpu_launches": 8 * n,
    })


def run_ffn(args, emit):
    """The block's FFN (two tcgen05 GEMMs, GELU-tanh fused into the first epilogue)."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pkg = importlib.import_module(PKG)
    pkg.build()
    lib = importlib.import_module(PKG + "._lib")
    T, H, I = (args.tokens or 32760), HIDDEN, 13824
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(1, T, H, generator=g, device=dev).to(torch.bfloat16)
    wu = (torch.randn(H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    bu = (torch.randn(1, I, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    bd = (torch.randn(1, H, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        pkg.wan_mlp(x, wu, wd, bu, bd)
    torch.cuda.synchronize()
    n = max(args.steps, 5)
    sampler = ClockSampler(0)
    sampler.start()
    ts = []
    for _ in range(n):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        pkg.wan_mlp(x, wu, wd, bu, bd)
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    clocks = sampler.stop()
    assert lib.device_status() == 0
    t = statistics.median(ts)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    bf16 = peaks.get("bf16_tflops", 1590.0)
    flops = 4.0 * T * H * I
    emit({
        "metric": "Wan FFN TFLOP/s (one block, C2 token count)", "value": round(flops / t / 1e9, 1), "unit": "TFLOP/s",
        "ms_per_step": round(t, 4), "higher_is_better": True, "n_gpus": 1, "steps": n, "warmup": args.warmup,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": CONFIGS["ffn"]["desc"], "T": T, "H": H, "I": I, "l2": "flushed (256 MB write) before each call"},
        "roofline": {"bound": "tensor", "achieved": round(flops / t / 1e9, 1), "peak": bf16, "unit": "TFLOP/s",
                     "frac": round(flops / t / 1e9 / bf16, 4), "peak_source": "measured (bf16_tflops burst)"},
        "clocks": clocks, "gpu_launches": 2 * n,
    })


def run_ffn_fp8(args, emit):
    """The FFN's FP8 leaf (row_mx_mlp): e4m3 ROW up GEMM with the GELU + MX-32 epilogue, block-scaled
    MX down GEMM with the closing gated residual."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pkg = importlib.import_module(PKG)
    pkg.build()
    lib = importlib.import_module(PKG + "._lib")
    T, H, I = (args.tokens or 32760), HIDDEN, 13824
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(T, H, generator=g, device=dev)
    rs = torch.clamp(x.abs().amax(1) / 448.0, min=1e-6)
    codes = (x / rs[:, None]).to(torch.float8_e4m3fn)
    del x
    uc, us, dc, ds = pkg.quantize_mlp_weights_row_mx(torch.randn(H, I, generator=g, device=dev) * 0.02,
                                                     torch.randn(I, H, generator=g, device=dev) * 0.02)
    bu = (torch.randn(I, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    bd = (torch.randn(H, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    res = torch.randn(1, T, H, generator=g, device=dev).to(torch.bfloat16)
    gate = torch.randn(1, 1, H, generator=g, device=dev) * 0.1
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        return pkg.row_mx_mlp((codes, rs), uc, dc, us, ds, bu, bd, residual=res, gate=gate)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    n = max(args.steps, 5)
    sampler = ClockSampler(0)
    sampler.start()
    ts = []
    for _ in range(n):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    clocks = sampler.stop()
    assert lib.device_status() == 0
    t = statistics.median(ts)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    fp8 = 2.0 * peaks.get("bf16_tflops", 1590.0)
    flops = 4.0 * T * H * I
    emit({
        "metric": "Wan FFN FP8 leaf TFLOP/s (row_mx_mlp, one block, C2 token count)", "value": round(flops / t / 1e9, 1),
        "unit": "TFLOP/s", "ms_per_step": round(t, 4), "higher_is_better": True, "n_gpus": 1, "steps": n,
        "warmup": args.warmup, "dtype": "e4m3 (fp32 accumulate, MX-32 intermediate)", "data": "synthetic",
        "config": {"workload": CONFIGS["ffn_fp8"]["desc"], "T": T, "H": H, "I": I,
                   "l2": "flushed (256 MB write) before each call"},
        "roofline": {"bound": "tensor", "achieved": round(flops / t / 1e9, 1), "peak": fp8, "unit": "TFLOP/s",
                     "frac": round(flops / t / 1e9 / fp8, 4),
                     "peak_source": "2 x measured bf16_tflops burst (dense fp8 rate = 2 x bf16 on B200)"},
        "clocks": clocks, "gpu_launches": 2 * n,
    })


def c5_block_flops(S: int, L: int = 512, I: int = 13824) -> float:
    """Algorithmic FLOPs of one block for one CFG branch (text K/V projection excluded: once per generation)."""
    H = HIDDEN
    return (4.0 * HEADS * S * S * HEAD_DIM + 2.0 * S * H * 3 * H + 2.0 * S * H * H + 2 * 2.0 * S * H * H
            + 4.0 * HEADS * S * L * HEAD_DIM + 4.0 * S * H * I)


def run_c5(args, world, rank, local_rank, emit):
    """Config 5: one transformer block per CFG branch. N=1: one branch at CP=1 (the single-GPU case);
    N>1: CFGP=2 x CP=N/2, ranks [0, N/2) run the cond branch and [N/2, N) the uncond one, each CP group
    a const-max ring over its own sequence shards (replica groups as get_cp_replica_groups builds them)."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        if world % 2:
            raise SystemExit("config c5 needs an even GPU count (CFGP=2)")
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    cp = max(world // 2, 1)
    branch = rank // cp if world > 1 else 0
    cp_rank = rank % cp
    groups = tuple(tuple(range(g * cp, (g + 1) * cp)) for g in range(2)) if world > 1 else None
    pkg = importlib.import_module(PKG)
    pkg.build()
    lib = importlib.import_module(PKG + "._lib")
    rope = importlib.import_module(PKG + ".rope")
    S, H, I, L = CONFIGS["c5"]["S"], HIDDEN, 13824, 512
    s_loc = S // cp
    g = torch.Generator(device=dev).manual_seed(1234)  # same weights on every rank
    rn = lambda *shape, s=0.02: (torch.randn(*shape, generator=g, device=dev) * s).to(torch.bfloat16)
    w = {
        "scale_shift_table": torch.randn(1, 6, H, generator=g, device=dev) / math.sqrt(H),
        "attn1.qkv_proj_weight": rn(H, 3 * H), "attn1.qkv_proj_bias": rn(3 * H),
        "attn1.norm_q.weight": 1 + rn(H, s=0.1), "attn1.norm_k.weight": 1 + rn(H, s=0.1),
        "attn1.o_proj_weight": rn(H, H), "attn1.o_proj_bias": rn(H),
        "norm2.weight": 1 + rn(H, s=0.1), "norm2.bias": rn(H),
        "attn2.q_proj_weight": rn(H, H), "attn2.q_proj_bias": rn(H), "attn2.norm_q.weight": 1 + rn(H, s=0.1),
        "attn2.k_proj_weight": rn(H, H), "attn2.k_proj_bias": rn(H), "attn2.norm_k.weight": 1 + rn(H, s=0.1),
        "attn2.v_proj_weight": rn(H, H), "attn2.v_proj_bias": rn(H),
        "attn2.o_proj_weight": rn(H, H), "attn2.o_proj_bias": rn(H),
        "ffn.up_weight": rn(H, I), "ffn.up_bias": rn(I), "ffn.down_weight": rn(I, H), "ffn.down_bias": rn(H),
    }
    bw = pkg.prepare_block_weights(w, HEADS)
    # this branch's inputs: hidden ~ N(0,1), text context ~ N(0,1) already projected to 5120 (the text
    # embedding runs once per generation, outside the block), timestep embedding ~ N(0, 0.1)
    gb = torch.Generator(device=dev).manual_seed(99 + branch)
    hidden = torch.randn(1, S, H, generator=gb, device=dev)[:, cp_rank * s_loc:(cp_rank + 1) * s_loc].to(torch.bfloat16).contiguous()
    ctx = torch.randn(1, L, H, generator=gb, device=dev).to(torch.bfloat16)
    temb = torch.randn(1, 6, H, generator=gb, device=dev) * 0.1
    kv = pkg.project_cross_kv(ctx, w["attn2.k_proj_weight"], w["attn2.k_proj_bias"], w["attn2.norm_k.weight"],
                              w["attn2.v_proj_weight"], w["attn2.v_proj_bias"], HEADS)
    cos, sin = rope.wan_rotary_freqs(HEAD_DIM, (1, 2, 2), 1024, CONFIGS["c5"]["latent"], device=dev)
    cos_rh, sin_rh = rope.rope_rotate_half_caches(cos, sin)
    cos_rh = cos_rh.reshape(S, HEAD_DIM)[cp_rank * s_loc:(cp_rank + 1) * s_loc].contiguous()
    sin_rh = sin_rh.reshape(S, HEAD_DIM)[cp_rank * s_loc:(cp_rank + 1) * s_loc].contiguous()

    def step():
        return pkg.wan_block_forward(hidden, temb, (cos_rh, sin_rh), kv, bw, cp_size=cp,
                                     cp_group=None, cp_replica_groups=groups)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out = step()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    assert lib.device_status() == 0 and torch.isfinite(out.float()).all()
    branches = 2 if world > 1 else 1
    flops = branches * c5_block_flops(S)
    if rank == 0:
        emit({
            "metric": "Wan2.2 transformer block TFLOP/s (whole job; CFGP=2 x CP=N/2)", "value": round(flops / ms / 1e9, 1),
            "unit": "TFLOP/s", "ms_per_step": round(ms, 4), "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights ~N(0,0.02), hidden/text ~N(0,1))",
            "config": {"workload": CONFIGS["c5"]["desc"], "S": S, "branches": branches, "cp": cp, "s_loc": s_loc,
                       "flops_per_branch": c5_block_flops(S), "l2": "inputs larger than L2"},
            "clocks": clocks,
        })
    if world > 1:
        pkg.destroy_rings()
        dist.destroy_process_group()


def attention_config(cfg, world: int, flops_layer: float) -> dict:
    """The `config` object of an attention line (c1 / c2 / c4), shared by both arms."""
    S = cfg["S"]
    s_loc = S // world
    return {
        "workload": cfg["desc"],
        "S": S, "heads": HEADS, "head_dim": HEAD_DIM, "cp": world, "s_loc": s_loc,
        "step": "one self-attention layer via wan_cp_self_attention (prologue + const-max attention, d-major out)",
        "l2": f"inputs larger than L2 (Q/K/V {3 * s_loc * HEADS * HEAD_DIM * 2 / 1e6:.0f} MB per rank per step)",
        "flops_per_layer": flops_layer,
    }


def run_reference(args, world, rank, cfg, flops_layer, emit):
    """The reference arm: the reference's own CPU attention path (``_torch_attend``,
    wan2_2_transformer.py:640-650, restated in oracle/attention.py because the reference module
    cannot be imported without the Neuron SDK) on the host cores. Each step is a bounded sample of
    the configured workload: head 0 x 1024 query rows of rank 0's shard against all S keys, drawn
    from the same seeded Q/K/V as the GPU arm. ``ms_per_step`` is the measured time of that sample;
    the full-layer time it implies is reported separately."""
    if rank != 0:
        return
    import numpy as np
    import torch

    # torchrun starts every rank with OMP_NUM_THREADS=1; the reference arm runs alone on rank 0 and
    # uses all host threads, as a CPU deployment of the reference would.
    try:
        from threadpoolctl import threadpool_limits

        _pool = threadpool_limits(limits=os.cpu_count() or 1)  # noqa: F841 (kept for the whole run)
    except Exception:
        pass
    torch.set_num_threads(os.cpu_count() or 1)
    S = cfg["S"]
    heads_s, rows_s = 1, 1024
    # Inputs: the GPU arm's seeded workload (make_qkv, plain torch ops), generated on a GPU when one
    # is visible only to save time; the timed attention runs on the host.
    gen_dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    q, k, v = make_qkv(args.config, gen_dev, seed=0)
    qs, ks, vs = cpu_sample_arrays(q, k, v, heads_s, min(rows_s, S // world))
    del q, k, v
    if gen_dev.type == "cuda":
        torch.cuda.empty_cache()
    for _ in range(args.warmup):
        cpu_attention_sample(qs, ks, vs, min_seconds=0.0)
    t0 = time.perf_counter()
    tot_fl = 0.0
    for _ in range(args.steps):
        _, _, fl = cpu_attention_sample(qs, ks, vs, min_seconds=0.0)
        tot_fl += fl
    el = time.perf_counter() - t0
    val = tot_fl / el / 1e12
    sample = (f"_torch_attend (wan2_2_transformer.py:640-650) restated in oracle/attention.py (numpy fp32): "
              f"head 0 x {qs.shape[2]} query rows of rank 0's shard x {S} keys per step, from the same seeded "
              f"Q/K/V as the GPU arm")
    res = {
        "metric": METRIC, "value": round(val, 6), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; random-init projection + RMSNorm + 3-D RoPE, no checkpoint/prompts)"
                if cfg["latent"] else "synthetic (seeded N(0,1)*0.5)",
        "config": attention_config(cfg, world, flops_layer),
        "impl": "reference",
        "restatement": "the reference's CPU attention path restated (its module needs the Neuron SDK to import)",
        "full_layer_ms_extrapolated": round(flops_layer / (val * 1e12) * 1e3, 1) if val else None,
        "cpu_baseline": {"value": round(val, 6), "unit": "TFLOP/s", "cores": cpu_cores(), "kind": "port", "sample": sample},
        "e2e": {"value": round(val, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(res)


if __name__ == "__main__":
    main()
