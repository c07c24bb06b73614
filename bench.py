#!/usr/bin/env python
"""Forward + backward throughput of one gated causal attention block on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|eager|triton]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N

One step = forward + backward of the block (fast_triton_attn.py:374-675) over
one batch of synthetic input already resident in HBM, through the public
autograd API; with N > 1 ranks the batch is sharded by sequence (B per rank
fixed: weak scaling) and the five weight gradients are all-reduced over NCCL
as one coalesced fp32 bucket (memory_efficient_attn_layer_b200.dp).

--impl reference : the reference path's CPU implementation timed on the host
                   cores (the eager block restated in oracle/eager.py), on a
                   bounded sample (one sequence of the workload per step).
--impl triton    : the reference's own GPU path, unmodified (fast_triton_attn.fused_attn, its Triton
                   kernels + ATen flash attention), imported from baseline/_ref, on the same
                   weights, tables and inputs; a comparator, like --impl eager.
--impl eager     : the reference's eager GPU equivalent (README.md:42-64:
                   checkpointed norm/projections/rotary + SDPA flash + gated
                   o_proj) in plain PyTorch, as an informative comparator.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd tokens/s per attn block"
# BASELINE.json configs (per GPU)
CONFIGS = {
    "c2": dict(B=128, T=2048, C=512, H=8, N=64, name="c2: 50M-class block B=128 T=2048 C=512 H=8 N=64"),
    "c3": dict(B=32, T=4096, C=1024, H=8, N=128, name="c3: wide block B=32 T=4096 C=1024 H=8 N=128"),
    "c4": dict(B=4, T=16384, C=2048, H=16, N=128, name="c4: long-context block B=4 T=16384 C=2048 H=16 N=128"),
    "c5": dict(B=128, T=2048, C=768, H=12, N=64, name="c5: DP block, global B=1024 T=2048 C=768 H=12 N=64 (B=128 per GPU at 8 GPUs)"),
}
LAUNCHES_PER_STAGE = {"bwd.memset": 0, "fwd.attention": 2}
# DRAM bytes per launch and per sequence, dram__bytes.sum from ncu captures of the c2 kernels at
# B=16 (every sequence is independent, so the traffic scales with B); the roofline's "traffic".
DRAM_BYTES_PER_SEQ = {
    "c2": {"bwd.attention_bwd": 287.0e6 / 16, "fwd.attention": 154.6e6 / 16,
           "bwd.attention_recompute": 179.1e6 / 16, "fwd.qkvg_gemm": 116.8e6 / 16,
           "bwd.qk_norm_rope_bwd": 216.5e6 / 16},
}


def model_flops(B, T, C, H, N):
    """Algorithmic fwd+bwd flops: 5 projections x (fwd, dgrad, wgrad) + causal attention (fwd 2, bwd 5)."""
    M = B * T
    return 30 * M * C * H * N + 7 * B * H * T * T * N


def stage_flops(B, T, C, H, N):
    M, HN = B * T, H * N
    attn_fwd = 2 * B * H * T * T * N
    return {
        "fwd.qkvg_gemm": 2 * M * C * 4 * HN, "fwd.attention": attn_fwd, "fwd.o_proj_gemm": 2 * M * HN * C,
        "bwd.qkvg_gemm": 2 * M * C * 4 * HN, "bwd.attention_recompute": attn_fwd, "bwd.dWo_gemm": 2 * M * C * HN,
        "bwd.dgate_gemm": 2 * M * C * HN, "bwd.attention_bwd": 5 * B * H * T * T * N,
        "bwd.dW_gemm": 2 * M * 4 * HN * C, "bwd.dx_gemm": 2 * M * 4 * HN * C,
    }


def stage_bytes(B, T, C, H, N):
    """Algorithmic HBM bytes of the bandwidth-bound stages."""
    M, HN = B * T, H * N
    return {
        # forward and backward recompute: only the inverse RMS is written (the projection GEMM and
        # the dAcc writers apply it; x_n is never stored)
        "fwd.rmsnorm": M * C * 2 + M * 4, "bwd.rmsnorm": M * C * 2 + M * 4,
        "bwd.qk_norm_rope_bwd": M * HN * (4 + 2 + 2 + 2 + 2 * 2) + 2 * B * H * T * 4,
        "bwd.rmsnorm_bwd": M * C * 2 * 3 + M * 4, "bwd.cast": 5 * HN * C * 6,
    }


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.rows = []  # (arrival time, fields)
        self.thread = None
        self.window = None

    def start(self):
        """Starts sampling early (nvidia-smi takes up to a second to come up).  Its output goes to a
        pseudo-terminal, so every sample line arrives (and is time-stamped) as it is taken."""
        import pty
        import threading

        try:
            master, slave = pty.openpty()
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=slave, stderr=subprocess.DEVNULL, close_fds=True)
            os.close(slave)
        except OSError:
            self.proc = None
            return

        def reader():
            try:
                with os.fdopen(master, "r", buffering=1, errors="replace") as f:
                    for line in f:
                        if line.count(",") >= 8:
                            self.rows.append((time.time(), line.strip().split(",")))
            except OSError:  # the terminal closes when nvidia-smi exits
                pass

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()

    def in_window(self, t0, t1):
        return sum(1 for t, _ in self.rows if t0 <= t <= t1)

    def mark(self, t0, t1, extended=False):
        """Host wall-clock bounds of the timed region (after device synchronisation); `extended` when
        the same steps kept running after it to collect samples."""
        self.window = (t0, t1)
        self.extended = extended

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        rows = [r for _, r in self.rows]
        used = "warm-up + timed steps"
        if self.window is not None:
            t0, t1 = self.window
            inside = [r for t, r in self.rows if t0 <= t <= t1 + 0.25]
            if len(inside) >= 2:
                rows = inside
                used = "timed steps + the same steps continued" if getattr(self, "extended", False) else "timed steps"
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        load = sorted(sm)[len(sm) // 4:] if sm else []  # drop ramp-up samples
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows), "window": used}


# --------------------------------------------------------------------------- inputs
def make_block_inputs(cfg, device, rank, requires_grad=True):
    from memory_efficient_attn_layer_b200 import Yarn

    B, T, C, H, N = (cfg[k] for k in ("B", "T", "C", "H", "N"))
    g = torch.Generator(device=device).manual_seed(0)  # weights replicated on every rank
    bound = 0.5 / math.sqrt(C)
    ws = [(torch.rand(H * N, C, device=device, generator=g) * 2 - 1) * bound for _ in range(4)]
    ws.append((torch.rand(C, H * N, device=device, generator=g) * 2 - 1) * bound)
    ws = [w.to(torch.bfloat16).requires_grad_(requires_grad) for w in ws]
    gx = torch.Generator(device=device).manual_seed(1000 + rank)  # this rank's shard of the batch
    x = torch.randn(B, T, C, device=device, generator=gx).to(torch.bfloat16)
    dy = torch.randn(B, T, C, device=device, generator=gx).to(torch.bfloat16)
    yarn = Yarn(N, T, device=device)
    return x, ws, yarn, dy


# --------------------------------------------------------------------------- CPU baseline
def cpu_sample(cfg, budget_s=12.0, min_reps=2):
    """Eager fp32 block on the host cores, one sequence of the workload per rep."""
    from oracle.eager import block_fwd_bwd, make_inputs

    torch.set_num_threads(os.cpu_count() or 1)
    inp = make_inputs(1, cfg["T"], cfg["C"], cfg["H"], cfg["N"], seed=0)
    block_fwd_bwd(inp, cfg["H"], cfg["N"])  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < min_reps or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        block_fwd_bwd(inp, cfg["H"], cfg["N"])
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": cfg["T"] / t, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"eager fp32 block fwd+bwd (oracle/eager.py) on 1 sequence of {cfg['T']} tokens "
                      f"(C={cfg['C']} H={cfg['H']} N={cfg['N']}), median of {len(times)} reps",
            "s_per_sequence": t}


# --------------------------------------------------------------------------- arms
def run_reference(args, cfg, rank, world):
    """CPU implementation of the path (oracle port) on the host cores; rank 0 only."""
    if rank != 0:
        return
    from oracle.eager import block_fwd_bwd, make_inputs

    torch.set_num_threads(os.cpu_count() or 1)
    inp = make_inputs(1, cfg["T"], cfg["C"], cfg["H"], cfg["N"], seed=0)
    for _ in range(args.warmup):
        block_fwd_bwd(inp, cfg["H"], cfg["N"])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        block_fwd_bwd(inp, cfg["H"], cfg["N"])
    dt = time.perf_counter() - t0
    value = args.steps * cfg["T"] / dt
    sample = (f"eager fp32 block fwd+bwd (oracle/eager.py, the reference's eager equivalent README.md:42-64) on one "
              f"sequence of {cfg['T']} tokens per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg["name"], "sample": "1 sequence per step", "B": 1, "T": cfg["T"], "C": cfg["C"],
                   "H": cfg["H"], "N": cfg["N"]},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def eager_block(x, ws, yarn, H, N, eps=1e-6):
    """README.md:42-64 in plain PyTorch on the GPU (comparator only)."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    B, T, C = x.shape
    wq, wk, wv, wg, wo = ws

    def norm(t):
        return F.rms_norm(t, (t.shape[-1],), eps=eps)

    def forward1(x):
        x = norm(x)
        q = F.linear(x, wq).view(B, T, H, N)
        k = F.linear(x, wk).view(B, T, H, N)
        v = F.linear(x, wv).view(B, T, H, N)
        g = F.linear(x, wg)
        return yarn.rotary(norm(q)), yarn.rotary(norm(k)), v, g

    q, k, v, g = torch.utils.checkpoint.checkpoint(forward1, x, use_reentrant=False)
    with sdpa_kernel(SDPBackend.FLASH_ATTENTION):
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
    o = o.transpose(1, 2).contiguous().view(B, T, H * N)
    return F.linear(o * torch.sigmoid(g), wo)


def reference_triton_block():
    """The reference's fused_attn (fast_triton_attn.py:681) from baseline/_ref, or None if absent."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "fast_triton_attn.py")):
        return None
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import fast_triton_attn

    return fast_triton_attn.fused_attn


def measure_block(fwd, x, dy, device, steps, warmup):
    """tokens/s, ms per step and activation memory of one block implementation (`fwd(x) -> y`) on the same
    device inputs: saved_for_backward = memory the forward leaves allocated besides its output,
    peak_fwd_bwd = peak allocation above the inputs during one forward + backward."""
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    m0 = torch.cuda.memory_allocated(device)
    xa = x.detach().requires_grad_(True)
    y = fwd(xa)
    torch.cuda.synchronize(device)
    saved = torch.cuda.memory_allocated(device) - m0 - y.numel() * y.element_size()
    y.backward(dy)
    torch.cuda.synchronize(device)
    peak = torch.cuda.max_memory_allocated(device) - m0
    del y, xa

    def step():
        y = fwd(x.detach().requires_grad_(True))
        y.backward(dy)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b) / steps
    return {"tokens_per_s": x.shape[0] * x.shape[1] / (ms / 1e3), "ms_per_step": ms,
            "saved_for_backward_gb": saved / 1e9, "peak_fwd_bwd_gb": peak / 1e9, "steps": steps}


def run_save_o_ablation(cfg, device, x, ws, yarn, dy, steps=10, warmup=3):
    """This build with save_o=True (the forward keeps the attention output, as the reference does, and the
    backward skips the attention recompute) on the same inputs: tokens/s, activation memory and the
    per-stage times of its backward."""
    from memory_efficient_attn_layer_b200 import FusedAttentionFunction, _lib

    H, N = cfg["H"], cfg["N"]
    wd = [w.detach() for w in ws]
    r = measure_block(lambda inp: FusedAttentionFunction.apply(inp, *wd, yarn.factor1, yarn.factor2, H, N, 1e-6,
                                                               True), x, dy, device, steps, warmup)
    _lib.profile_enable(True)
    for _ in range(3):
        y = FusedAttentionFunction.apply(x.detach().requires_grad_(True), *wd, yarn.factor1, yarn.factor2, H, N,
                                         1e-6, True)
        y.backward(dy)
    st = _lib.profile_read()
    _lib.profile_enable(False)
    r["stages_ms"] = {k: v[0] / v[1] for k, v in st.items() if k.startswith("bwd.")}
    r["what"] = "save_o=True: saved set x + O + row LSE (the reference's), no attention recompute in the backward"
    return r


def run_comparators(cfg, device, x, ws, yarn, dy, our_saved, our_peak, our_value, steps=10, warmup=3):
    """The reference's own GPU block (fast_triton_attn.fused_attn from baseline/_ref, unmodified: its Triton
    kernels and ATen flash attention) and the README's eager SDPA block, run in this process on the same
    weights, tables and device inputs as this build's line, with this build's figures beside them."""
    H, N = cfg["H"], cfg["N"]
    wd = [w.detach().clone().requires_grad_(True) for w in ws]
    out = {"ours": {"tokens_per_s": our_value, "saved_for_backward_gb": our_saved / 1e9,
                    "peak_fwd_bwd_gb": our_peak / 1e9}}
    ref = reference_triton_block()
    if ref is None:
        out["reference_triton"] = {"unavailable": "baseline/_ref/fast_triton_attn.py not installed"}
    else:
        lins = []
        for w in wd:
            lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False, device=device, dtype=w.dtype)
            lin.weight = torch.nn.Parameter(w.data, requires_grad=True)
            lins.append(lin)
        r = measure_block(lambda inp: ref(inp, *lins, yarn, H, N), x, dy, device, steps, warmup)
        r["path"] = "fast_triton_attn.fused_attn (baseline/_ref, unmodified)"
        out["reference_triton"] = r
        del lins
    e = measure_block(lambda inp: eager_block(inp, wd, yarn, H, N), x, dy, device, steps, warmup)
    e["path"] = "README.md:42-64 eager block (checkpointed projections + SDPA flash)"
    out["eager_sdpa"] = e
    rt = out["reference_triton"]
    if "tokens_per_s" in rt:
        out["speedup_vs_reference_triton"] = our_value / rt["tokens_per_s"]
        out["saved_ratio_vs_reference_triton"] = (our_saved / 1e9) / rt["saved_for_backward_gb"]
        out["peak_ratio_vs_reference_triton"] = (our_peak / 1e9) / rt["peak_fwd_bwd_gb"]
    return out


# --------------------------------------------------------------------------- model level
def run_stack(args, cfg, device):
    """The block's caller at model level (README.md:1, "-1GB of memory usage" on a 50M model): a stack of
    `--stack L` pre-norm residual layers x += attn(x) ; x += mlp(norm(x)) with a 4C ReLU^2 MLP, every
    layer's attention through `--impl` (ours / triton / eager) and the same MLP (torch).  Prints one
    JSON line with model-level fwd+bwd tokens/s and peak activation memory (not a bench line of the
    block metric)."""
    import torch.nn as nn
    import torch.nn.functional as F

    from memory_efficient_attn_layer_b200 import CausalSoftmaxAttention, Yarn

    B, T, C, H, N = (cfg[k] for k in ("B", "T", "C", "H", "N"))
    L = args.stack
    torch.manual_seed(0)
    attn = nn.ModuleList([CausalSoftmaxAttention(C, H, N) for _ in range(L)]).to(device=device, dtype=torch.bfloat16)
    for blk in attn:  # o_proj zero-init (README.md:35) would cut the gradient path: give it values
        nn.init.uniform_(blk.o_proj.weight, -0.5 / math.sqrt(H * N), 0.5 / math.sqrt(H * N))
    up = nn.ModuleList([nn.Linear(C, 4 * C, bias=False) for _ in range(L)]).to(device=device, dtype=torch.bfloat16)
    down = nn.ModuleList([nn.Linear(4 * C, C, bias=False) for _ in range(L)]).to(device=device, dtype=torch.bfloat16)
    yarn = Yarn(N, T, device=device)
    ref_fused = reference_triton_block() if args.impl == "triton" else None
    if args.impl == "triton" and ref_fused is None:
        print(json.dumps({"impl": "triton", "unavailable": "baseline/_ref/fast_triton_attn.py not installed"}))
        return

    def attention(l, h):
        blk = attn[l]
        if args.impl == "triton":
            return ref_fused(h, blk.q_proj, blk.k_proj, blk.v_proj, blk.g_proj, blk.o_proj, yarn, H, N)
        if args.impl == "eager":
            ws = [blk.q_proj.weight, blk.k_proj.weight, blk.v_proj.weight, blk.g_proj.weight, blk.o_proj.weight]
            return eager_block(h, ws, yarn, H, N)
        return blk(h, yarn)

    def model(h):
        for l in range(L):
            h = h + attention(l, h)
            h = h + down[l](F.relu(up[l](F.rms_norm(h, (C,), eps=1e-6))).square())
        return h

    g = torch.Generator(device=device).manual_seed(1000)
    x = torch.randn(B, T, C, device=device, generator=g).to(torch.bfloat16)
    dy = torch.randn(B, T, C, device=device, generator=g).to(torch.bfloat16)
    params = sum(p.numel() for m in (attn, up, down) for p in m.parameters())

    def step():
        y = model(x.detach().requires_grad_(True))
        y.backward(dy)
        for m in (attn, up, down):
            for p in m.parameters():
                p.grad = None

    step()
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    m0 = torch.cuda.memory_allocated(device)
    step()
    torch.cuda.synchronize(device)
    peak = torch.cuda.max_memory_allocated(device) - m0
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize(device)
    ms = t0.elapsed_time(t1) / args.steps
    print(json.dumps({
        "impl": args.impl, "metric": "model fwd+bwd tokens/s (stack of the block + MLP)", "value": B * T / (ms / 1e3),
        "unit": "tokens/s", "ms_per_step": ms, "layers": L, "params": params, "tokens_per_step": B * T,
        "peak_activation_gb": peak / 1e9, "config": {"workload": cfg["name"], "layer": "x += attn(x); x += "
                                                     "mlp(rmsnorm(x)), mlp = W2 relu(W1 x)^2, 4C hidden"},
    }), flush=True)


def run_gemm_e4m3(args, cfg, device):
    """e4m3 against bf16 operands in the same CTA-pair GEMM (mea_gemm_e4m3 / mea_gemm, K-major A and B, fp32
    out) on the block's long GEMM shapes at this config: the FP8-projection row's measurement.  Prints one
    JSON line (not a bench line of the block metric)."""
    import ctypes

    from memory_efficient_attn_layer_b200 import _lib

    L = _lib.lib()
    B, T, C, H, N = (cfg[k] for k in ("B", "T", "C", "H", "N"))
    M, HN = B * T, H * N
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    st = lambda: ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    rows = []
    for (m, n, k, what) in [(M, C, 4 * HN, "dx = dAcc [W_q;W_k;W_v;W_g] shape"), (M, 4 * HN, C, "q/k/v/g projection shape")]:
        out = torch.empty(m, n, device=device)
        res = {"shape": what, "M": m, "N": n, "K": k}
        for kind in ("bf16", "e4m3"):
            if kind == "bf16":
                a = torch.randn(m, k, device=device).bfloat16()
                b = torch.randn(n, k, device=device).bfloat16()
                fn = lambda: _lib.check(L.mea_gemm(m, n, k, P(a), k, 0, P(b), k, 0, P(out), n, 0, None, st()))
            else:
                a = torch.randn(m, k, device=device).to(torch.float8_e4m3fn)
                b = torch.randn(n, k, device=device).to(torch.float8_e4m3fn)
                fn = lambda: _lib.check(L.mea_gemm_e4m3(m, n, k, P(a), k, P(b), k, P(out), n, 0, None, st()))
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                fn()
            e1.record()
            torch.cuda.synchronize(device)
            ms = e0.elapsed_time(e1) / args.steps
            res[kind] = {"ms": ms, "tflops": 2 * m * n * k / (ms / 1e3) / 1e12}
            del a, b
        res["speedup"] = res["bf16"]["ms"] / res["e4m3"]["ms"]
        rows.append(res)
    print(json.dumps({"probe": "e4m3 vs bf16 operands, CTA-pair tcgen05 GEMM, fp32 output",
                      "config": cfg["name"], "rows": rows}), flush=True)


def run_gpu(args, cfg, rank, world, device):
    import torch.distributed as dist

    from memory_efficient_attn_layer_b200 import FusedAttentionFunction, _lib
    from memory_efficient_attn_layer_b200.dp import allreduce_grads, overlap_grad_allreduce

    B, T, C, H, N = (cfg[k] for k in ("B", "T", "C", "H", "N"))
    tokens_rank = B * T
    clocks = ClockSampler(device.index if device.index is not None else 0)
    clocks.start()  # samples are kept for the timed window only (marked below)
    x, ws, yarn, dy = make_block_inputs(cfg, device, rank)
    eager = args.impl in ("eager", "triton")  # comparators: no library profiler
    ref_fused = None
    if args.impl == "triton":
        ref_fused = reference_triton_block()
        if ref_fused is None:
            clocks.stop()
            if rank == 0:
                print(json.dumps({"impl": "triton", "unavailable": "baseline/_ref/fast_triton_attn.py not installed"}))
            return
        lins = []
        for w in ws:  # nn.Linear views of the same weight tensors (the reference reads .weight)
            lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False, device=device, dtype=w.dtype)
            lin.weight = torch.nn.Parameter(w.data, requires_grad=True)
            lins.append(lin)
        ws = [lin.weight for lin in lins]

    def fwd(inp):
        if ref_fused is not None:
            return ref_fused(inp, *lins, yarn, H, N)
        if eager:
            return eager_block(inp, ws, yarn, H, N)
        return FusedAttentionFunction.apply(inp, *ws, yarn.factor1, yarn.factor2, H, N, 1e-6)

    # --optim: the step ends with the sharded AdamW update (reduce-scatter of the fp32 weight gradients the
    # backward hands over directly, the fused update kernel on this rank's shard, all-gather of the bf16
    # weights) instead of an all-reduce.
    opt, opt_ev = None, []
    if args.optim:
        if eager:
            raise SystemExit("--optim runs with --impl ours")
        from memory_efficient_attn_layer_b200.optim import ShardedAdamW

        opt = ShardedAdamW(ws, lr=1e-4, weight_decay=1e-2)

    # Our block exchanges its weight gradients inside its own backward (the
    # all-reduce of each part starts as soon as the library marks it final);
    # the comparators exchange theirs after the backward.
    overlap = world > 1 and not eager and opt is None

    def exchange_ctx():
        return overlap_grad_allreduce() if overlap else contextlib.nullcontext()

    def opt_step(timed=False):
        if not timed:
            opt.step()
            return
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        opt.step()
        b.record()
        opt_ev.append((a, b))

    def step(inp, grad, timed=False):
        if opt is not None:
            opt.zero_grad()
        with exchange_ctx():
            y = fwd(inp)
            y.backward(grad)
        if opt is not None:
            opt_step(timed)
        elif world > 1 and not overlap:
            allreduce_grads(ws)
        for w in ws:
            w.grad = None
        return y

    # ---- activation memory: what the forward keeps for the backward, and the fwd+bwd peak
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    m0 = torch.cuda.memory_allocated(device)
    xa = x.detach().requires_grad_(True)
    y = fwd(xa)
    torch.cuda.synchronize(device)
    saved = torch.cuda.memory_allocated(device) - m0 - y.numel() * y.element_size()
    y.backward(dy)
    torch.cuda.synchronize(device)
    peak = torch.cuda.max_memory_allocated(device) - m0
    del y, xa
    for w in ws:
        w.grad = None

    # ---- device-timed steps (inputs resident in HBM; x is 2*B*T*C bytes > L2)
    for _ in range(args.warmup):
        step(x, dy)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    if not eager:
        _lib.profile_enable(True)
    if overlap:
        from memory_efficient_attn_layer_b200.fused_attn import record_exchange_waits

        record_exchange_waits(True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    ev0.record()
    for _ in range(args.steps):
        step(x, dy, timed=True)
    ev1.record()
    torch.cuda.synchronize(device)
    t_wall1 = time.time()
    ms = ev0.elapsed_time(ev1)
    stages = {}
    if not eager:
        stages = _lib.profile_read()
        _lib.profile_enable(False)
    exchange_wait = None
    if overlap:
        waits = record_exchange_waits(False)
        if waits:
            exchange_wait = {"ms_per_step": sum(waits) / len(waits), "max_ms": max(waits), "steps": len(waits),
                             "what": "time the caller's stream waited at the end of the backward for the "
                                     "side stream's all-reduce of the weight gradients (0 = fully overlapped)"}
    # A short timed region can end before nvidia-smi has taken enough samples in it: then the same steps
    # keep running (untimed, at most 2 s) until it has five, and the clocks cover that span too.
    # Every rank runs the same number of these steps (their collectives must pair up).
    while True:
        need = clocks.proc is not None and clocks.in_window(t_wall0, time.time()) < 5 and time.time() - t_wall1 < 2.0
        if world > 1:
            f = torch.tensor([1 if need else 0], device=device, dtype=torch.int32)
            dist.all_reduce(f, op=dist.ReduceOp.MAX)
            need = bool(f.item())
        if not need:
            break
        step(x, dy)
        torch.cuda.synchronize(device)
    clocks.mark(t_wall0, time.time(), extended=time.time() - t_wall1 > 0.01)
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = world * tokens_rank * args.steps / (ms / 1e3)

    # ---- end to end through the public API: every step's x and dy come from pinned host memory and
    # its loss goes back to the host.  Inputs are double-buffered: step i+1's host->device copy runs on
    # a copy stream while step i computes (as a data loader feeding a training step would), each copy
    # ordered after the step that last read its buffer.
    xh = x.detach().cpu().pin_memory()
    dyh = dy.detach().cpu().pin_memory()
    loss_h = torch.empty(1, dtype=torch.float32).pin_memory()
    # enough steps that the pipeline's fill (the first copy, exposed, and the last step's compute) is a
    # small share of the timed region
    e2e_steps = max(30, args.steps // 4)
    comp = torch.cuda.current_stream(device)
    copy_stream = torch.cuda.Stream(device)
    xbuf = [torch.empty_like(x) for _ in range(2)]
    dybuf = [torch.empty_like(dy) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def e2e_copy(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            if i >= 2:
                copy_stream.wait_event(consumed[b])
            xbuf[b].copy_(xh, non_blocking=True)
            dybuf[b].copy_(dyh, non_blocking=True)
            copied[b].record(copy_stream)

    def e2e_step(i, n):
        b = i % 2
        if i + 1 < n:
            e2e_copy(i + 1)
        comp.wait_event(copied[b])
        if opt is not None:
            opt.zero_grad()
        with exchange_ctx():
            y = fwd(xbuf[b])
            loss = (y * dybuf[b]).sum(dtype=torch.float32)
            loss.backward()
        consumed[b].record(comp)
        if opt is not None:
            opt.step()
        elif world > 1 and not overlap:
            allreduce_grads(ws)
        for w in ws:
            w.grad = None
        loss_h.copy_(loss.detach().view(1), non_blocking=True)

    def e2e_run(n):
        e2e_copy(0)
        for i in range(n):
            e2e_step(i, n)

    e2e_run(2)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    e2e_run(e2e_steps)
    e1.record(comp)
    torch.cuda.synchronize(device)
    ems = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ems], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e_value = world * tokens_rank * e2e_steps / (ems / 1e3)

    if rank != 0:
        return
    peaks = load_peaks()
    F_step = model_flops(B, T, C, H, N)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: x, dy ~ N(0,1); weights ~ U(+-0.5/sqrt(C)) replicated; rotary tables for N, T",
        "config": {"workload": cfg["name"], "B_per_gpu": B, "global_batch": B * world, "T": T, "C": C, "H": H,
                   "N": N, "parallelism": f"dp{world}" if world > 1 else "single",
                   "grad_exchange": ("nccl all-reduce overlapped with the backward" if overlap else
                                     "nccl reduce-scatter + all-gather around the sharded AdamW step"
                                     if opt is not None else "nccl all-reduce after the backward")
                   if world > 1 else None,
                   "optimizer": ("ShardedAdamW in every step: fp32 weight gradients straight from the backward, "
                                 "reduce-scatter, fused AdamW kernel on this rank's shard, all-gather of the "
                                 "bf16 weights") if opt is not None else None,
                   "l2": f"inputs larger than L2 (x is {2 * B * T * C / 1e6:.0f} MB per GPU), no flush"},
    }
    if eager:
        line["impl"] = args.impl
    # The burst peak (a GEMM timed alone) for kernels and for timed regions shorter than the few seconds
    # the sustained figure was measured over; the sustained peak for seconds-long timed regions.
    long_region = ms >= 2000.0
    step_peak = peaks["bf16_tflops_sustained"] if long_region else peaks["bf16_tflops"]
    line["tensor_pipe_frac_step"] = {
        "achieved_tflops": F_step / (ms_step / 1e3) / 1e12, "peak_tflops": step_peak,
        "frac": F_step / (ms_step / 1e3) / 1e12 / step_peak,
        "flops_per_step": F_step,
        "peak_source": peaks["source"] + (" sustained (timed region >= 2 s)" if long_region
                                          else " burst (timed region < 2 s)")}
    line["activation_gb"] = {"saved_for_backward": saved / 1e9, "peak_fwd_bwd": peak / 1e9}
    if stages:
        sf, sb = stage_flops(B, T, C, H, N), stage_bytes(B, T, C, H, N)
        table = {}
        for name, (tot, cnt) in stages.items():
            avg = tot / cnt
            row = {"ms": avg, "share": tot / sum(v[0] for v in stages.values())}
            if name in sf:
                row["tflops"] = sf[name] / (avg / 1e3) / 1e12
            if name in sb:
                row["gbs"] = sb[name] / (avg / 1e3) / 1e9
            table[name] = row
        line["stages"] = table
        top = max(stages, key=lambda k: stages[k][0])
        avg = stages[top][0] / stages[top][1]
        per_seq = DRAM_BYTES_PER_SEQ.get(cfg.get("key", ""), {}).get(top)
        traffic = per_seq * B if per_seq else None
        if top in sf:
            ach = sf[top] / (avg / 1e3) / 1e12
            line["roofline"] = {"kernel": top, "bound": "tensor", "achieved": ach,
                                "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                                "frac": ach / peaks["bf16_tflops"], "traffic": traffic,
                                "peak_source": peaks["source"] + " burst (a kernel of a few ms)",
                                "algorithmic": f"{sf[top]:.4g} flop per launch"}
        else:
            ach = sb[top] / (avg / 1e3) / 1e9
            line["roofline"] = {"kernel": top, "bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"],
                                "unit": "GB/s", "frac": ach / peaks["hbm_gbs"], "traffic": traffic,
                                "peak_source": peaks["source"]}
        line["gpu_launches"] = sum(cnt * LAUNCHES_PER_STAGE.get(n, 1) for n, (_, cnt) in stages.items())
        if opt is not None:
            line["gpu_launches"] += args.steps  # one mea_adamw_step kernel per step
    if opt is not None:
        o_ms = sum(a.elapsed_time(b) for a, b in opt_ev) / len(opt_ev)
        n_shard = opt.layout.shard
        o_bytes = 30 * n_shard  # fp32 w, m, v, g read (16 B); w, m, v written (12 B); bf16 w written (2 B)
        line["optimizer"] = {"ms_per_step": o_ms, "share_of_step": o_ms / ms_step, "weights": opt.layout.numel,
                             "shard": n_shard, "update_bytes": o_bytes,
                             "update_gbs_upper_bound": o_bytes / (o_ms / 1e3) / 1e9,
                             "note": "ms_per_step spans opt.step() (at N>1 the reduce-scatter and all-gather too); "
                                     "the GB/s figure divides the update kernel's bytes by that whole span"}
    line["e2e"] = {"value": e2e_value, "unit": "tokens/s",
                   "h2d_bytes_per_step": world * (x.numel() * x.element_size() + dy.numel() * dy.element_size()),
                   "d2h_bytes_per_step": world * 4,
                   "path": {"ours": "FusedAttentionFunction.apply", "triton": "reference fast_triton_attn.fused_attn",
                            "eager": "eager README block"}[args.impl]
                           + " + loss=(y*dy).sum() + backward; every step's x and dy "
                           "copied in from pinned host memory (double-buffered: the next step's copy overlaps this "
                           "step's compute) and its loss copied out"}
    if exchange_wait is not None:
        line["exchange_wait"] = exchange_wait
    line["clocks"] = clk
    if world == 1 and not eager and not args.no_comparators:
        line["save_o_ablation"] = run_save_o_ablation(cfg, device, x, ws, yarn, dy)
        line["comparators"] = run_comparators(cfg, device, x, ws, yarn, dy, saved, peak, value)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sample(cfg)
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference", "eager", "triton"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-comparators", action="store_true",
                    help="skip the in-process GPU comparators (reference Triton block, eager SDPA block)")
    ap.add_argument("--batch", type=int, default=0,
                    help="per-GPU batch override (smaller cases for profiler captures; not a bench line)")
    ap.add_argument("--optim", action="store_true",
                    help="end every step with the ShardedAdamW update (reduce-scatter, fused AdamW kernel, "
                         "all-gather) instead of the gradient all-reduce")
    ap.add_argument("--gemm-e4m3", action="store_true",
                    help="probe: the e4m3 GEMM against the bf16 one on this config's GEMM shapes (one GPU; not a "
                         "bench line)")
    ap.add_argument("--stack", type=int, default=0,
                    help="model-level mode: a stack of this many block + MLP layers (memory and tokens/s of the "
                         "caller; one GPU; not a bench line)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    cfg = dict(CONFIGS[args.config], key=args.config)
    if args.batch > 0:
        cfg["B"] = args.batch
        cfg["name"] += f" [batch override B={args.batch}]"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        if args.stack > 0:
            if world > 1:
                raise SystemExit("--stack runs on one GPU")
            run_stack(args, cfg, device)
            return
        if args.gemm_e4m3:
            run_gemm_e4m3(args, cfg, device)
            return
        run_gpu(args, cfg, rank, world, device)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
