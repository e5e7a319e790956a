"""Benchmark of the B200 QLoRA hot path (driver contract: one JSON line on rank 0).

Workload: one Qwen2.5-1.5B decoder layer's seven NF4
projections (q 1536->1536, k/v 1536->256, o 1536->1536, gate/up 1536->8960,
down 8960->1536), NF4/block64 + double-quant/block256 weights ~N(0, 0.02),
LoRA r=16 alpha=32 on every projection, T=3300 packed fp16 tokens ~N(0, 1),
fused residual add-RMSNorm (eps 1e-6, gamma ~N(1, 0.1)) before attention and
before the MLP, the MLP itself as the fused gate/up -> SwiGLU -> down chain,
forward plus backward (dX of every projection, LoRA dA/dB, norm gradients).
Attention is outside the hot path: its output is a synthetic input of o_proj,
and the upstream gradients of q, k, v and of the layer output are synthetic.
One step = that layer forward + backward on one micro-batch.

value     = algorithmic NF4-GEMM FLOPs of the step (fwd 2MNK+2MKr+2MrN,
            dX 2MNK+2MNr+2MrK per projection) / device time, whole job;
e2e       = the same through the public API with every input copied from
            pinned host memory and the layer-input gradient read back;
roofline  = the fused NF4 GEMM (dominant kernel) timed alone with CUDA events
            against the measured dense bf16 peak;
ce        = fused linear CE fwd+bwd tokens/s at configs[3] (T=3300,
            V=151936, H=1536, 63% ignored);
cpu_baseline = the reference's path restated on the host (oracle/cpu_path.py).

Multi-GPU (torchrun, NCCL): each rank runs its own micro-batch (data parallel,
weak scaling) and the LoRA gradients are all-reduced every step.

Other workloads (their own JSON line): --workload stack times configs[2] (the
28-layer stack over 64 synthetic variable-length batches, data parallel, strong
scaling); --workload sweep times configs[4] (Qwen2.5-7B shapes, M from 1 to
16384, weights N-split across the ranks).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, INTER, KV = 1536, 8960, 256
RANK_R, ALPHA = 16, 32
T_TOKENS = 3300
EPS = 1e-6
PROJ = [("q", HIDDEN, HIDDEN), ("k", KV, HIDDEN), ("v", KV, HIDDEN), ("o", HIDDEN, HIDDEN),
        ("gate", INTER, HIDDEN), ("up", INTER, HIDDEN), ("down", HIDDEN, INTER)]
METRIC = "NF4 dequant-GEMM TFLOP/s (% peak) fwd+bwd at Qwen2.5-1.5B shapes; CE tokens/s"
L2_FLUSH_BYTES = 256 << 20


def proj_flops(m, n, k, r):
    fwd = 2 * m * n * k + 2 * m * k * r + 2 * m * r * n
    dx = 2 * m * n * k + 2 * m * n * r + 2 * m * r * k
    return fwd, dx


def step_flops(m):
    return sum(sum(proj_flops(m, n, k, RANK_R)) for _, n, k in PROJ)


def nf4_weight_bytes(n, k):
    """Packed codes, uint8 absmax per 64, fp32 absmax2 per 16384 elements, code table, offset."""
    return n * k // 2 + n * k // 64 + 4 * ((n * k + 16383) // 16384) + 1024 + 4


def pass_bytes(m):
    """Algorithmic HBM bytes of one layer's GEMM pass (12 launches): per launch the
    weight(s), the activation read, the output(s) written, the LoRA factors and the
    rank-r operand.  q/k/v/o: forward and dX each.  MLP: gate/up forward (both
    weights, X, gate|up and act written), down forward, down dX (dY and gate|up
    read, dgate|dup written), two-weight dX (dgate|dup read, dX written)."""
    r, h, n = RANK_R, HIDDEN, INTER
    total = 0
    for _, no, ki in PROJ[:4]:
        one = nf4_weight_bytes(no, ki) + 2 * m * ki + 2 * m * no + 2 * r * (ki + no) + 2 * m * r
        total += 2 * one
    wgu = 2 * nf4_weight_bytes(n, h)
    total += wgu + 2 * m * h + 3 * 2 * m * n + 2 * (2 * r) * (h + 2 * n) + 2 * m * 2 * r      # gate/up + SwiGLU
    total += nf4_weight_bytes(h, n) + 2 * m * n + 2 * m * h + 2 * r * (n + h) + 2 * m * r     # down
    total += nf4_weight_bytes(h, n) + 2 * m * h + 2 * 2 * m * n + 2 * 2 * m * n + 2 * r * (n + h) + 2 * m * r  # down dX
    total += wgu + 2 * 2 * m * n + 2 * m * h + 2 * (2 * r) * h + 2 * m * 2 * r                # gate/up dX
    return total


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one 12-launch GEMM
# pass, from a separate ncu capture of `bench.py --kernel-case gemm_pass --warmup 1
# --steps 1` (-k regex:pair_kernel -s 12 -c 12; ncu cannot run inside the timed
# bench).  A static figure: it is reported as such and describes the kernels of
# the capture it came from (624.9 MB read + 227.2 MB written).
PASS_TRAFFIC_NCU = {3300: 852130560}


def static_pass_traffic(m):
    return PASS_TRAFFIC_NCU.get(m)


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples the SM clock and the clock-event (throttle) reasons of the GPU the
    process uses through NVML (read-only): once when the timed region starts,
    every millisecond from a background thread while it runs, and once when it
    ends.  The NVML handle is found by the device's UUID (NVML's indices need not
    match CUDA's under CUDA_VISIBLE_DEVICES), then its PCI bus id, then its index."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index, period=0.001):
        self.index, self.period = index, period
        self.samples, self.max_mhz, self.reasons = [], None, set()
        self.handle = None

    def _handle(self, pynvml):
        import torch
        props = torch.cuda.get_device_properties(self.index)
        uuid = getattr(props, "uuid", None)
        if uuid is not None:
            try:
                text = str(uuid)
                return pynvml.nvmlDeviceGetHandleByUUID(text if text.startswith("GPU-") else "GPU-" + text)
            except Exception:
                pass
        try:
            bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _sample(self):
        import pynvml
        self.samples.append(pynvml.nvmlDeviceGetClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        mask = pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        for name, bit in self.REASONS.items():
            if mask & bit:
                self.reasons.add(name)

    def _run(self):
        while not self.stop.is_set():
            self._sample()
            self.stop.wait(self.period)

    def __enter__(self):
        import threading
        self.stop = threading.Event()
        self.thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.handle = self._handle(pynvml)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self._sample()
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
        return self

    def __exit__(self, *exc):
        self.stop.set()
        if self.thread is not None:
            self.thread.join(timeout=5)
        if self.handle is not None:
            try:
                self._sample()
            except Exception:
                pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------ layer
def build_layer(torch, device, seed):
    from soupsuck_b200.quantize import quantize_nf4
    g = torch.Generator(device=device).manual_seed(seed)
    layer = {}
    for name, n, k in PROJ:
        w = (torch.randn((n, k), device=device, generator=g) * 0.02).to(torch.float16)
        packed, st = quantize_nf4(w)
        a = ((torch.rand((RANK_R, k), device=device, generator=g) * 2 - 1) / math.sqrt(k)).requires_grad_()
        b = (torch.randn((n, RANK_R), device=device, generator=g) * 0.01).requires_grad_()
        layer[name] = (packed, st, a, b)
    layer["gamma_in"] = (1 + 0.1 * torch.randn(HIDDEN, device=device, generator=g)).to(torch.float16)
    layer["gamma_post"] = (1 + 0.1 * torch.randn(HIDDEN, device=device, generator=g)).to(torch.float16)
    return layer


def input_shapes(t):
    return {"residual": (t, HIDDEN), "mlp_prev": (t, HIDDEN), "attn": (t, HIDDEN),
            "g_q": (t, HIDDEN), "g_k": (t, KV), "g_v": (t, KV), "g_out": (t, HIDDEN)}


DIFF_INPUTS = ("residual", "attn", "mlp_prev")


def layer_step(torch, layer, inp, streams=None):
    """Forward + backward of the hot path of one decoder layer (public API calls).

    add-RMSNorm, q/k/v, o, add-RMSNorm, then the MLP as the fused
    gate/up(+SwiGLU) -> down chain (``nf4_swiglu_mlp``), residual add; backward
    from synthetic upstream gradients of q, k, v and the layer output.  With
    ``streams`` (two side streams) the projections that do not depend on each
    other run concurrently: o_proj (its input is a layer input) on one side
    stream, q/k/v on the other.  Autograd runs every backward node on the
    stream of its forward, so the backward overlaps the same way; all streams are
    joined before returning."""
    from soupsuck_b200.kernels import add_rms_norm, nf4_lora_linear, nf4_swiglu_mlp
    s = ALPHA / RANK_R

    def proj(name, x):
        packed, st, a, b = layer[name]
        return nf4_lora_linear(x, packed, st, a, b, s)

    def mlp(x):
        return nf4_swiglu_mlp(x, layer["gate"], layer["up"], layer["down"], s)

    grads = [inp["g_q"], inp["g_k"], inp["g_v"], inp["g_out"]]
    if streams is None:
        s1, y1 = add_rms_norm(inp["residual"], inp["mlp_prev"], layer["gamma_in"], EPS)
        q, k, v = proj("q", y1), proj("k", y1), proj("v", y1)
        o = proj("o", inp["attn"])
        s2, y2 = add_rms_norm(s1, o, layer["gamma_post"], EPS)
        out = s2 + mlp(y2)
        torch.autograd.backward([q, k, v, out], grads)
        return inp["residual"].grad
    main = torch.cuda.current_stream()
    sa, sb = streams
    sa.wait_stream(main)
    sb.wait_stream(main)
    with torch.cuda.stream(sb):
        o = proj("o", inp["attn"])
    s1, y1 = add_rms_norm(inp["residual"], inp["mlp_prev"], layer["gamma_in"], EPS)
    sa.wait_stream(main)
    with torch.cuda.stream(sa):
        q, k, v = proj("q", y1), proj("k", y1), proj("v", y1)
    main.wait_stream(sb)
    s2, y2 = add_rms_norm(s1, o, layer["gamma_post"], EPS)
    out = s2 + mlp(y2)
    main.wait_stream(sa)
    torch.autograd.backward([q, k, v, out], grads)
    main.wait_stream(sa)
    main.wait_stream(sb)
    return inp["residual"].grad


def lora_params(layer):
    ps = []
    for name, _, _ in PROJ:
        ps.extend(layer[name][2:4])
    return ps


# ------------------------------------------------------------------ CPU reference
def _cpu_projections(layer):
    from oracle.cpu_path import CpuProjection
    return [CpuProjection(layer[name][0], layer[name][1], layer[name][2], layer[name][3],
                          ALPHA / RANK_R) for name, _, _ in PROJ]


def run_cpu_sample(torch, layer, budget_s, rows=T_TOKENS):
    """cpu_baseline: the reference path restated on the host, on the same
    configs[1] rows as the GPU step (every pass dequantizes each weight twice)."""
    from oracle.cpu_path import threads, time_projections
    sec, flops = time_projections(_cpu_projections(layer), rows, budget_s=budget_s)
    return {"value": flops / sec / 1e12, "unit": "TFLOP/s", "cores": threads(), "kind": "port",
            "same_config": rows == T_TOKENS,
            "sample": f"fwd+dX of the 7 projections on all {rows} rows of configs[1] per pass "
                      f"(dequant via the C oracle on {threads()} threads + torch fp32 matmul), "
                      f"{sec:.3f} s per pass"}


def run_reference(args, torch):
    """--impl reference: the reference's path restated on the host cores (the
    oracle port; the reference itself is Triton for sm_75 behind bitsandbytes),
    on the same configs[1] workload as the GPU arm; rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    layer = build_layer(torch, "cpu", seed=0)
    from oracle.cpu_path import threads, time_projections
    projs = _cpu_projections(layer)
    rows = args.tokens
    time_projections(projs, rows, budget_s=0.0, min_reps=1)
    per = []
    flops = None
    for _ in range(args.steps):
        sec, flops = time_projections(projs, rows, budget_s=0.0, min_reps=1)
        per.append(sec)
    total = sum(per)
    value = flops * len(per) / total / 1e12
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000 * total / len(per), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"configs[1]: 7 NF4+LoRA(r=16) projections fwd+dX on {rows} rows "
                                   f"(the GEMM work of the GPU arm's layer step)", "tokens": rows,
                       "same_config": rows == T_TOKENS},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads(), "kind": "port",
                             "sample": f"all {rows} rows x 7 projections fwd+dX per step"},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU timing helpers
def mlp_calls(torch, layer, device, t, rnd):
    """(label, launch) pairs of the fused MLP's four GEMM launches at T = t with
    LoRA (rank-32 step for the gate/up pair, rank 16 for down)."""
    import ctypes

    from soupsuck_b200 import _lib
    from soupsuck_b200.kernels.nf4_gemm import _weight_struct, nf4_linear_raw
    calls = []
    stream = _lib.stream_of(device)
    wg = _weight_struct(layer["gate"][0], layer["gate"][1])
    wu = _weight_struct(layer["up"][0], layer["up"][1])
    dp, ds, da_, db_ = layer["down"]
    wd = _weight_struct(dp, ds)
    x, dy = rnd(t, HIDDEN), rnd(t, HIDDEN)
    z2, b_gu, u2, at_cat = rnd(t, 2 * RANK_R), rnd(2 * INTER, 2 * RANK_R), rnd(t, 2 * RANK_R), rnd(HIDDEN, 2 * RANK_R)
    zd, bd16, ud, atd = rnd(t, RANK_R), db_.detach().half().contiguous(), rnd(t, RANK_R), da_.detach().half().t().contiguous()
    gate_up, act, dgu = rnd(t, 2 * INTER), rnd(t, INTER), rnd(t, 2 * INTER)
    dx = torch.empty((t, HIDDEN), device=device, dtype=torch.float16)
    nbytes = _lib.query("sb_nf4_linear_dx2_workspace_bytes", t, INTER, HIDDEN)
    ws = torch.empty(max(nbytes, 1), device=device, dtype=torch.uint8)
    calls.append(("gate/up fwd + SwiGLU", lambda: _lib.call("sb_nf4_mlp_gate_up_fwd", x.data_ptr(), t, ctypes.byref(wg), ctypes.byref(wu),
                                   z2.data_ptr(), b_gu.data_ptr(), 2 * RANK_R, gate_up.data_ptr(), act.data_ptr(),
                                   stream)))
    calls.append(("down fwd", lambda: nf4_linear_raw(act, dp, ds, lora_a=zd, lora_b=bd16)))
    calls.append(("down dX + SwiGLU'", lambda: _lib.call("sb_nf4_mlp_down_dx", dy.data_ptr(), t, ctypes.byref(wd), ud.data_ptr(),
                                   atd.data_ptr(), RANK_R, gate_up.data_ptr(), dgu.data_ptr(), stream)))
    calls.append(("gate/up dX (two weights)", lambda: _lib.call("sb_nf4_linear_dx2", dgu.data_ptr(), t, ctypes.byref(wg), ctypes.byref(wu),
                                   u2.data_ptr(), at_cat.data_ptr(), 2 * RANK_R, dx.data_ptr(), ws.data_ptr(),
                                   nbytes, stream)))
    return calls


def gemm_roofline(torch, layer, device, t, passes=10, warm=3):
    """Time the fused NF4 GEMM launches of one layer step back to back with CUDA
    events on their stream: forward and dX of q, k, v, o (LoRA fused) and the
    MLP's four launches -- gate/up with the SwiGLU epilogue, down, down dX with
    the SwiGLU-derivative epilogue, and the two-weight gate/up dX (rank-32 LoRA
    step for the gate/up pair).  Returns (FLOPs, seconds per pass, launches)."""
    import ctypes

    from soupsuck_b200 import _lib
    from soupsuck_b200.kernels.nf4_gemm import _weight_struct, nf4_linear_raw
    calls = []
    flops = 0
    gen = torch.Generator(device=device).manual_seed(5)
    rnd = lambda *shape: torch.randn(shape, device=device, dtype=torch.float16, generator=gen)
    for name, n, k in PROJ[:4]:
        packed, st, a, b = layer[name]
        x, dy, za = rnd(t, k), rnd(t, n), rnd(t, RANK_R)
        bt = b.detach().half().contiguous()
        at = a.detach().half().t().contiguous()
        calls.append((f"{name} fwd", lambda x=x, p=packed, s=st, za=za, bt=bt:
                      nf4_linear_raw(x, p, s, lora_a=za, lora_b=bt)))
        calls.append((f"{name} dX", lambda dy=dy, p=packed, s=st, za=za, at=at:
                      nf4_linear_raw(dy, p, s, transpose=True, lora_a=za, lora_b=at)))
    calls += mlp_calls(torch, layer, device, t, rnd)
    flops = step_flops(t)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    for _ in range(warm):
        for _, c in calls:
            c()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream(device)
    times = []
    for _ in range(passes):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        for _, c in calls:
            c()
        e1.record(cur)
        e1.synchronize()
        times.append(e0.elapsed_time(e1) / 1000.0)
    sec = statistics.median(times)
    # Each launch alone (L2 flushed before it), for the per-kernel breakdown.
    per_launch = {}
    for label, c in calls:
        samples = []
        for _ in range(max(3, passes // 2)):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            c()
            e1.record(cur)
            e1.synchronize()
            samples.append(e0.elapsed_time(e1) * 1000.0)
        per_launch[label] = round(statistics.median(samples), 1)
    return flops, sec, len(calls), per_launch


def ce_benchmark(torch, device, steps, tokens=T_TOKENS, warm=2):
    from soupsuck_b200.kernels import fused_linear_cross_entropy
    t, h, v = tokens, HIDDEN, 151936
    g = torch.Generator(device=device).manual_seed(4)
    hidden = torch.randn((t, h), device=device, dtype=torch.float16, generator=g).requires_grad_()
    weight = (torch.randn((v, h), device=device, generator=g) * 0.02).to(torch.float16)
    targets = torch.randint(v, (t,), device=device, generator=g)
    mask = torch.rand(t, device=device, generator=g) < 0.63
    targets[mask] = -100
    valid = int((targets != -100).sum().item())

    def once():
        loss = fused_linear_cross_entropy(hidden, weight, targets, validate=False)[0]
        loss.sum().backward()
        hidden.grad = None

    for _ in range(warm):
        once()
    torch.cuda.synchronize()
    times = []
    for _ in range(max(1, min(steps, 10))):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        once()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) / 1000.0)
    sec = statistics.median(times)
    flops = 2 * t * v * h + 4 * valid * v * h
    return {"tokens_per_s": t / sec, "ms_per_step": 1000 * sec, "tflops": flops / sec / 1e12,
            "config": {"tokens": t, "vocab": v, "hidden": h, "labelled": valid}}


def kernel_case(args, torch):
    """--kernel-case: a small, self-checking launch of one kernel family for ncu
    captures (a few launches, well under a GB on the device).  Exits 0 only if
    no kernel reported a device error."""
    from soupsuck_b200 import _lib
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    t = args.tokens
    if args.kernel_case in ("nf4_fwd", "nf4_dx"):
        from soupsuck_b200.kernels.nf4_gemm import nf4_linear_raw
        from soupsuck_b200.quantize import quantize_nf4
        g = torch.Generator(device=device).manual_seed(0)
        n, k = args.case_n, args.case_k
        w = (torch.randn((n, k), device=device, generator=g) * 0.02).to(torch.float16)
        packed, st = quantize_nf4(w)
        za = torch.randn((t, RANK_R), device=device, dtype=torch.float16, generator=g)
        if args.kernel_case == "nf4_fwd":
            x = torch.randn((t, k), device=device, dtype=torch.float16, generator=g)
            lb = (torch.randn((n, RANK_R), device=device, generator=g) * 0.01).half()
            call = lambda: nf4_linear_raw(x, packed, st, lora_a=za, lora_b=lb)
        else:
            x = torch.randn((t, n), device=device, dtype=torch.float16, generator=g)
            la = (torch.randn((k, RANK_R), device=device, generator=g) * 0.01).half()
            call = lambda: nf4_linear_raw(x, packed, st, transpose=True, lora_a=za, lora_b=la)
        for _ in range(args.warmup + args.steps):
            call()
    elif args.kernel_case == "mlp":
        layer = build_layer(torch, device, seed=0)
        gen = torch.Generator(device=device).manual_seed(5)
        rnd = lambda *shape: torch.randn(shape, device=device, dtype=torch.float16, generator=gen)
        calls = mlp_calls(torch, layer, device, t, rnd)
        for _ in range(args.warmup + args.steps):
            for _, c in calls:
                c()
    elif args.kernel_case == "gemm_pass":
        layer = build_layer(torch, device, seed=0)
        gemm_roofline(torch, layer, device, t, passes=args.steps, warm=args.warmup)
    elif args.kernel_case == "layer":
        layer = build_layer(torch, device, seed=0)
        gen = torch.Generator(device=device).manual_seed(1000)
        inp = {name: torch.randn(shp, device=device, dtype=torch.float16, generator=gen)
               for name, shp in input_shapes(t).items()}
        for name in DIFF_INPUTS:
            inp[name].requires_grad_()
        for _ in range(args.warmup + args.steps):
            for name in DIFF_INPUTS:
                inp[name].grad = None
            layer_step(torch, layer, inp)
    elif args.kernel_case == "ce":
        ce_benchmark(torch, device, args.steps, tokens=t, warm=args.warmup)
    torch.cuda.synchronize()
    err = _lib.take_device_error(device)
    print(json.dumps({"kernel_case": args.kernel_case, "tokens": t, "device_error": err,
                      "launches": _lib.launch_count()}))
    return 1 if err else 0


# ------------------------------------------------------------------ 7B shape sweep
SWEEP_HIDDEN, SWEEP_INTER, SWEEP_KV = 3584, 18944, 512
SWEEP_PROJ = [("q", SWEEP_HIDDEN, SWEEP_HIDDEN), ("k", SWEEP_KV, SWEEP_HIDDEN), ("v", SWEEP_KV, SWEEP_HIDDEN),
              ("o", SWEEP_HIDDEN, SWEEP_HIDDEN), ("gate", SWEEP_INTER, SWEEP_HIDDEN),
              ("up", SWEEP_INTER, SWEEP_HIDDEN), ("down", SWEEP_HIDDEN, SWEEP_INTER)]
SWEEP_M = (1, 16, 128, 4096, 16384)


def run_sweep(args, torch):
    """Qwen2.5-7B projection shapes, M in {1, 16, 128, 4096, 16384}, NF4 forward and
    dX of the seven projections (no LoRA), weights N-split across the ranks with an
    all-gather of Y and an all-reduce of dX when launched on several GPUs.  Reported
    per M: whole-job TFLOP/s and the HBM rate of the algorithmic bytes (packed
    weight + absmax + activations in and out)."""
    import datetime

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    from soupsuck_b200 import _lib
    from soupsuck_b200.distributed import allreduce_sum, nf4_row_shard
    from soupsuck_b200.kernels.nf4_gemm import nf4_linear_raw
    from soupsuck_b200.quantize import quantize_nf4
    import torch.distributed as dist

    g = torch.Generator(device=device).manual_seed(0)
    weights = []
    for name, n, k in SWEEP_PROJ:
        w = (torch.randn((n, k), device=device, generator=g) * 0.02).to(torch.float16)
        packed, st = quantize_nf4(w)
        del w
        sh = nf4_row_shard(packed, st, rank, world) if world > 1 else None
        weights.append((name, n, k, packed, st, sh))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    peak_burst, _, hbm, _ = measured_peaks()
    results = []
    for m in SWEEP_M:
        calls, flops, nbytes = [], 0, 0
        for name, n, k, packed, st, sh in weights:
            x = torch.randn((m, k), device=device, dtype=torch.float16, generator=g)
            dy = torch.randn((m, n), device=device, dtype=torch.float16, generator=g)
            if sh is None:
                calls.append(lambda x=x, p=packed, s=st: nf4_linear_raw(x, p, s))
                calls.append(lambda dy=dy, p=packed, s=st: nf4_linear_raw(dy, p, s, transpose=True))
            else:
                rows = sh.row1 - sh.row0
                dy_loc = dy[:, sh.row0:sh.row1].contiguous()
                # Equal row shards (every sweep width divides by N): the ranks' Y
                # blocks are gathered straight into one [N, m, rows] buffer, which is
                # Y itself at m = 1 and Y after one column-block interleave otherwise.
                assert n % world == 0 and rows == n // world
                buf = torch.empty((world * m, rows), device=device, dtype=torch.float16)

                def fwd(x=x, sh=sh, rows=rows, buf=buf):
                    dist.all_gather_into_tensor(buf, nf4_linear_raw(x, sh.packed, sh.state))
                    if m == 1:
                        return buf.view(1, world * rows)
                    return buf.view(world, m, rows).permute(1, 0, 2).reshape(m, world * rows)

                def dxf(dy_loc=dy_loc, sh=sh):
                    return allreduce_sum(nf4_linear_raw(dy_loc, sh.packed, sh.state, transpose=True))

                calls += [fwd, dxf]
            flops += 2 * (2 * m * n * k)
            wbytes = nf4_weight_bytes(n, k)
            nbytes += 2 * (wbytes + 2 * m * k + 2 * m * n)
        for _ in range(max(args.warmup, 3)):
            for c in calls:
                c()
        torch.cuda.synchronize()
        # The pass is replayed from a CUDA graph (with its NCCL collectives on N
        # GPUs), so host launch overhead -- which exceeds the kernels' own time at
        # M <= 16 -- stays out of the timing.
        graph = None
        if not args.no_graph:
            side = torch.cuda.Stream(device)
            side.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(side):
                for c in calls:
                    c()
            torch.cuda.current_stream(device).wait_stream(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for c in calls:
                    c()
            graph.replay()
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        marks = []
        stream = torch.cuda.current_stream(device)
        for _ in range(max(3, min(args.steps, 10))):  # queued back to back, read at the end
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if graph is not None:
                graph.replay()
            else:
                for c in calls:
                    c()
            e1.record(stream)
            marks.append((e0, e1))
        torch.cuda.synchronize()
        times = [e0.elapsed_time(e1) / 1000.0 for e0, e1 in marks]
        del graph
        sec = statistics.median(times)
        if world > 1:
            tt = torch.tensor([sec], device=device, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            sec = float(tt.item())
        results.append({"M": m, "ms_per_pass": 1000 * sec, "tflops": flops / sec / 1e12,
                        "pct_peak": 100 * flops / sec / 1e12 / (peak_burst * world),
                        "hbm_gbs": nbytes / sec / 1e9, "pct_hbm": 100 * nbytes / sec / 1e9 / (hbm * world),
                        "projection_calls": len(calls), "cuda_graph": not args.no_graph})
    err = _lib.take_device_error(device)
    if rank == 0:
        print(json.dumps({"metric": "NF4 dequant-GEMM fwd+dX at Qwen2.5-7B shapes (configs[4])",
                          "n_gpus": world, "dtype": "f16", "data": "synthetic",
                          "parallelism": f"N-split x{world}" if world > 1 else "single GPU",
                          "l2": "flushed before every timed pass", "sweep": results, "device_error": err}),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------ 28-layer stack, DP
STACK_LAYERS, STACK_BATCHES, STACK_ROWS, STACK_LEN = 28, 64, 4, (64, 512)
STACK_BUCKET = 128


def stack_lengths():
    """Real token count of each of the 64 synthetic batches (4 right-padded rows of
    seeded lengths U[64, 512], unpadded to packed T)."""
    import numpy as np
    rng = np.random.default_rng(2026)
    lens = rng.integers(STACK_LEN[0], STACK_LEN[1] + 1, size=(STACK_BATCHES, STACK_ROWS))
    return [int(x) for x in lens.sum(axis=1)]


def stack_step(torch, layers, x, delta, g_out, g_kv, side=None):
    """Forward + backward of the 28-layer projection stack on one packed batch.
    Attention is outside the hot path: o_proj reads q in place of the attention
    output (same shape).  The MLP is the fused gate/up -> SwiGLU -> down chain.
    With ``side`` (a stream) k/v run beside q, forward and (autograd keeps each
    backward node on its forward's stream) backward."""
    from soupsuck_b200.kernels import add_rms_norm, nf4_lora_linear, nf4_swiglu_mlp
    s = ALPHA / RANK_R

    def proj(layer, name, inp):
        packed, st, a, b = layer[name]
        return nf4_lora_linear(inp, packed, st, a, b, s)

    main = torch.cuda.current_stream()
    res, dlt = x, delta
    outs, grads = [], []
    for layer in layers:
        s1, y1 = add_rms_norm(res, dlt, layer["gamma_in"], EPS)
        if side is not None:
            # Tensors that cross streams are recorded on the stream that reads them,
            # so the allocator does not hand their memory to the allocating stream
            # while the other still uses it (autograd frees them mid-backward).
            side.wait_stream(main)
            with torch.cuda.stream(side):
                k, v = proj(layer, "k", y1), proj(layer, "v", y1)
            y1.record_stream(side)
        else:
            k, v = proj(layer, "k", y1), proj(layer, "v", y1)
        q = proj(layer, "q", y1)
        o = proj(layer, "o", q)
        s2, y2 = add_rms_norm(s1, o, layer["gamma_post"], EPS)
        mlp = nf4_swiglu_mlp(y2, layer["gate"], layer["up"], layer["down"], s)
        outs += [k, v]
        grads += [g_kv, g_kv]
        res, dlt = s2, mlp
    outs.append(res + dlt)
    grads.append(g_out)
    if side is not None:
        main.wait_stream(side)
    torch.autograd.backward(outs, grads)
    if side is not None:
        main.wait_stream(side)


def run_stack(args, torch):
    """the full 28-layer Qwen2.5-1.5B projection stack over 64 synthetic
    batches, data parallel.  Rank r takes batches r, r + N, ...; one step runs all of
    them (forward + backward, LoRA gradients accumulated) and all-reduces the LoRA
    gradients once.  Each batch's packed length is padded up to a multiple of 128
    rows (zero rows) so that one CUDA graph per length bucket serves every batch
    of that bucket; FLOPs count the real tokens only."""
    import datetime

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    from soupsuck_b200 import _lib

    layers = [build_layer(torch, device, seed=100 + i) for i in range(STACK_LAYERS)]
    params = [p for layer in layers for p in lora_params(layer)]
    lengths = stack_lengths()
    mine = list(range(rank, STACK_BATCHES, world))
    buckets = sorted({-(-lengths[b] // STACK_BUCKET) * STACK_BUCKET for b in mine})
    g = torch.Generator(device=device).manual_seed(7 + rank)
    tmax = buckets[-1]
    base = {"x": torch.randn((tmax, HIDDEN), device=device, dtype=torch.float16, generator=g),
            "d": torch.randn((tmax, HIDDEN), device=device, dtype=torch.float16, generator=g),
            "go": torch.randn((tmax, HIDDEN), device=device, dtype=torch.float16, generator=g),
            "gkv": torch.randn((tmax, KV), device=device, dtype=torch.float16, generator=g)}
    acc = [torch.zeros_like(p) for p in params]
    kv_stream = None if args.no_streams else torch.cuda.Stream(device)

    def inputs(t):
        x = base["x"][:t].clone().requires_grad_()
        d = base["d"][:t].clone().requires_grad_()
        return x, d, base["go"][:t].contiguous(), base["gkv"][:t].contiguous()

    # Warm-up eagerly once per bucket (configures kernels before capture).
    for t in buckets:
        for p in params:
            p.grad = None
        stack_step(torch, layers, *inputs(t), side=kv_stream)
    torch.cuda.synchronize()
    graphs = {}
    if not args.no_graph:
        side = torch.cuda.Stream(device)
        for t in buckets:
            ins = inputs(t)
            side.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(side):
                for p in params:
                    p.grad = None
                stack_step(torch, layers, *ins, side=kv_stream)
            torch.cuda.current_stream(device).wait_stream(side)
            torch.cuda.synchronize()
            for p in params:
                p.grad = None
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                stack_step(torch, layers, *ins, side=kv_stream)
            graphs[t] = (gr, [p.grad for p in params], ins)
        torch.cuda.synchronize()

    def allreduce(tensors):
        if dist is None:
            return
        flat = torch.cat([x.reshape(-1) for x in tensors])
        dist.all_reduce(flat)
        flat.div_(world)
        off = 0
        for x in tensors:
            x.copy_(flat[off:off + x.numel()].view_as(x))
            off += x.numel()

    def step():
        for a_ in acc:
            a_.zero_()
        for b in mine:
            t = -(-lengths[b] // STACK_BUCKET) * STACK_BUCKET
            if graphs:
                gr, gg, _ = graphs[t]
                gr.replay()
            else:
                for p in params:
                    p.grad = None
                stack_step(torch, layers, *inputs(t), side=kv_stream)
                gg = [p.grad for p in params]
            torch._foreach_add_(acc, gg)
        allreduce(acc)

    for _ in range(max(1, min(args.warmup, 2))):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    stream = torch.cuda.current_stream(device)
    times = []
    nsteps = max(1, min(args.steps, 3))
    with ClockSampler(local) as clocks:
        for _ in range(nsteps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1) / 1000.0)
    sec = statistics.median(times)
    if dist is not None:
        tt = torch.tensor([sec], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        sec = float(tt.item())
    tokens = sum(lengths)
    padded = sum(-(-x // STACK_BUCKET) * STACK_BUCKET for x in lengths)
    flops = sum(step_flops(x) for x in lengths) * STACK_LAYERS
    peak_burst, peak_sust, _, _ = measured_peaks()
    err = _lib.take_device_error(device)
    if rank == 0:
        print(json.dumps({
            "metric": "NF4 dequant-GEMM TFLOP/s fwd+bwd, 28-layer Qwen2.5-1.5B stack (configs[2])",
            "value": flops / sec / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": nsteps,
            "ms_per_step": 1000 * sec, "tokens_per_s": tokens / sec, "higher_is_better": True,
            "scaling": "strong", "dtype": "f16", "data": "synthetic (seeded lengths U[64,512], 4 rows x 64 batches)",
            "pct_peak": 100 * flops / sec / 1e12 / (peak_sust * world),
            "peak": "sustained bf16 (MEASURED_PEAKS.json)",
            "config": {"workload": "configs[2]: 28 layers x 7 NF4+LoRA(r=16) projections (MLP as the fused gate/up+SwiGLU -> down chain) + 2 add-RMSNorm, fwd+bwd",
                       "batches": STACK_BATCHES, "tokens": tokens, "padded_rows": padded,
                       "bucket_rows": STACK_BUCKET, "cuda_graph": bool(graphs), "graphs": len(graphs),
                       "streams": "k/v on a side stream" if kv_stream is not None else "one stream",
                       "parallelism": f"dp{world}"},
            "clocks": clocks.summary(), "device_error": err}), flush=True)
    del graphs
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=T_TOKENS)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-streams", action="store_true",
                    help="run the layer's projections one after another on one stream")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ce", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--workload", choices=["layer", "sweep", "stack"], default="layer",
                    help="layer: configs[1] (the headline line); sweep: configs[4] 7B shapes; "
                         "stack: configs[2] 28-layer stack, data parallel")
    ap.add_argument("--kernel-case", choices=["nf4_fwd", "nf4_dx", "gemm_pass", "mlp", "layer", "ce"],
                    help="run a small launch of one kernel family (for ncu) instead of the bench")
    ap.add_argument("--case-n", type=int, default=INTER)
    ap.add_argument("--case-k", type=int, default=HIDDEN)
    args = ap.parse_args()

    import torch

    if args.kernel_case:
        return kernel_case(args, torch)
    if args.workload == "sweep":
        return run_sweep(args, torch)
    if args.workload == "stack":
        return run_stack(args, torch)

    if args.impl == "reference":
        return run_reference(args, torch)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)

    from soupsuck_b200 import _lib
    t = args.tokens
    layer = build_layer(torch, device, seed=0)
    params = lora_params(layer)
    shapes = input_shapes(t)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    dev_in = {}
    for name, shp in shapes.items():
        dev_in[name] = torch.randn(shp, device=device, dtype=torch.float16, generator=g)
    for name in DIFF_INPUTS:
        dev_in[name].requires_grad_()

    def zero_grads():
        for p in params:
            p.grad = None
        for name in DIFF_INPUTS:
            dev_in[name].grad = None

    def allreduce_grads():
        """Average the LoRA gradients over the ranks: one flat fp32 buffer (one
        concatenation launch), one NCCL all-reduce, one scale.  Inside a captured
        step this is part of the graph, so it runs right behind the backward with
        no host round trip.  Returns the averaged flat buffer (None on one GPU)."""
        if dist is None:
            return None
        flat = torch.cat([p.grad.reshape(-1) for p in params])
        dist.all_reduce(flat)
        flat.mul_(1.0 / world)
        return flat

    streams = None if args.no_streams else (torch.cuda.Stream(device), torch.cuda.Stream(device))

    def device_step():
        zero_grads()
        layer_step(torch, layer, dev_in, streams)
        allreduce_grads()

    # Warm-up (also configures kernels before any capture).
    for _ in range(max(args.warmup, 3)):
        device_step()
    torch.cuda.synchronize()

    # Two input sets, each with its own captured step: the timed device loop replays
    # the first; the end-to-end loop alternates them so that the host->device copy
    # of the next step's inputs overlaps the current step.
    sets = [dev_in]
    graphs, graph_grads, graph_out = [], [], []
    launches_per_step = None
    if not args.no_graph:
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(2):
                device_step()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize()
        second = {k: v.detach().clone() for k, v in dev_in.items()}
        for name in DIFF_INPUTS:
            second[name].requires_grad_()
        sets.append(second)
        for inputs in sets:
            for p in params:
                p.grad = None
            for name in DIFF_INPUTS:
                inputs[name].grad = None
            g_ = torch.cuda.CUDAGraph()
            before = _lib.launch_count()
            with torch.cuda.graph(g_):
                layer_step(torch, layer, inputs, streams)
                flat = allreduce_grads()
            launches_per_step = _lib.launch_count() - before
            graphs.append(g_)
            graph_grads.append(flat if flat is not None else [p.grad for p in params])
            graph_out.append(inputs["residual"].grad)
        for g_ in graphs:
            for _ in range(2):
                g_.replay()
        torch.cuda.synchronize()
        # Only the `graphs` list may own the captured steps: they hold NCCL work and
        # must all be released before the process group is destroyed.
        del g_
    graph = graphs[0] if graphs else None

    def run_step():
        # With a graph the LoRA gradients (and, on N GPUs, their all-reduced
        # average) live in the graph's pool and are overwritten by every replay.
        if graph is not None:
            graph.replay()
        else:
            device_step()

    if launches_per_step is None:
        before = _lib.launch_count()
        run_step()
        torch.cuda.synchronize()
        launches_per_step = _lib.launch_count() - before

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    # One untimed flush + step: the flush buffer's first write maps its pages, and
    # on N GPUs a first step behind it would make the other ranks' all-reduce wait.
    flush.zero_()
    run_step()
    # ---- timed region: K steps, L2 flushed before each (outside the events).  The
    # steps are queued back to back and read once at the end: a host round trip
    # per step would let the ranks' hosts drift apart, and on N GPUs every rank's
    # all-reduce would then wait for the latest host's launch.
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    marks = []
    with ClockSampler(local) as clocks:
        if dist is not None:
            # The ranks' hosts leave the barrier at different times; one small
            # all-reduce queued ahead of the first step lines the GPUs up, so the
            # first step's in-graph all-reduce does not wait for the latest host.
            dist.all_reduce(torch.zeros(1, device=device))
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run_step()
            e1.record(stream)
            marks.append((e0, e1))
        torch.cuda.synchronize()
    step_times = [e0.elapsed_time(e1) / 1000.0 for e0, e1 in marks]
    if dist is not None:
        dist.barrier()
    local_total = sum(step_times)
    total = local_total
    rank_steps = None
    if dist is not None:
        tt = torch.tensor([local_total], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total = float(tt.item())
        # Every rank's own mean / fastest / slowest step (ms), the slowest step's
        # index and the median SM clock: with the all-reduce inside each step,
        # ranks that wait for a slower one show it in their mean.
        mhz = clocks.summary()["sm_mhz"]
        mine = torch.tensor([1000 * local_total / args.steps, 1000 * min(step_times), 1000 * max(step_times),
                             float(step_times.index(max(step_times))), float(mhz) if mhz is not None else -1.0],
                            device=device, dtype=torch.float64)
        every = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        rank_steps = [[round(float(x), 4) for x in e.tolist()] for e in every]
    sec_per_step = total / args.steps
    flops = step_flops(t) * world
    value = flops / sec_per_step / 1e12
    dev_err = _lib.take_device_error(device)

    # ---- end-to-end through the public API with host buffers: every step copies
    # its inputs from pinned host memory and reads the layer-input gradient back.
    # With graphs the steps alternate between the two input sets: the copy of step
    # i+1's inputs (on a copy stream) and the read-back of step i-1's result (on a
    # second copy stream, the other PCIe direction) overlap step i; a set's inputs
    # and result buffer are reused only after its previous read-back has finished.
    host = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in dev_in.items()}
    for k in host:
        host[k].copy_(dev_in[k].detach())
    out_host = [torch.empty((t, HIDDEN), dtype=torch.float16, pin_memory=True) for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = out_host[0].numel() * out_host[0].element_size()
    copy_stream = torch.cuda.Stream(device)
    back_stream = torch.cuda.Stream(device)
    e2e_steps = max(3, min(args.steps, 10))

    def e2e_run(n):
        if graph is None:
            for _ in range(n):
                for k, hv in host.items():
                    with torch.no_grad():
                        dev_in[k].copy_(hv, non_blocking=True)
                run_step()
                out_host[0].copy_(dev_in["residual"].grad, non_blocking=True)
            return
        done = [None, None]
        copy_stream.wait_stream(stream)
        back_stream.wait_stream(stream)
        for i in range(n):
            j = i % len(sets)
            if done[j] is not None:
                copy_stream.wait_event(done[j])
                stream.wait_event(done[j])
            with torch.cuda.stream(copy_stream), torch.no_grad():
                for k, hv in host.items():
                    sets[j][k].copy_(hv, non_blocking=True)
            copied = torch.cuda.Event()
            copied.record(copy_stream)
            stream.wait_event(copied)
            graphs[j].replay()
            computed = torch.cuda.Event()
            computed.record(stream)
            back_stream.wait_event(computed)
            with torch.cuda.stream(back_stream):
                out_host[j].copy_(graph_out[j], non_blocking=True)
            done[j] = torch.cuda.Event()
            done[j].record(back_stream)
        stream.wait_stream(copy_stream)
        stream.wait_stream(back_stream)

    e2e_run(2)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e2e_times = []
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        e2e_run(e2e_steps)
        e1.record(stream)
        e1.synchronize()
        e2e_times.append(e0.elapsed_time(e1) / 1000.0 / e2e_steps)
    e2e_local = sum(e2e_times) / len(e2e_times)
    e2e_sec = e2e_local
    if dist is not None:
        tt = torch.tensor([e2e_local], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_sec = float(tt.item())
    e2e_value = flops / e2e_sec / 1e12

    # The captured steps hold NCCL work: release them before the process group.
    torch.cuda.synchronize()
    used_graph = graph is not None
    graph = None
    graphs.clear()
    graph_grads.clear()
    import gc
    gc.collect()
    torch.cuda.synchronize()
    if rank != 0:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    peak_burst, peak_sust, hbm, peak_kind = measured_peaks()
    gflops, gsec, glaunch, per_launch = gemm_roofline(torch, layer, device, t)
    achieved = gflops / gsec / 1e12
    ce = None if args.no_ce else ce_benchmark(torch, device, args.steps)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = run_cpu_sample(torch, layer, args.cpu_budget)
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * sec_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) NF4 weights)",
        "config": {"workload": "configs[1]: Qwen2.5-1.5B layer, 7 NF4+LoRA(r=16) projections + 2 add-RMSNorm "
                               "+ SwiGLU (fused MLP), fwd+bwd",
                   "tokens_per_gpu": t, "global_tokens": t * world,
                   "parallelism": f"dp{world}" + (" + LoRA-grad NCCL all-reduce" if world > 1 else ""),
                   "l2": "flushed (256 MiB write) before every timed step, outside the events",
                   "cuda_graph": used_graph,
                   "streams": "o and q/k/v on two side streams" if streams else "one stream"},
        "pct_peak": 100.0 * value / (peak_burst * world),
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": 1000 * e2e_sec,
                "pipelining": "next step's host->device copy and the previous step's device->host read-back (one copy stream each) overlap the current step (two input sets)"
                              if used_graph else "none"},
        "gpu_launches": int(launches_per_step) * args.steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_burst, "unit": "TFLOP/s",
                     "frac": achieved / peak_burst, "traffic": static_pass_traffic(t),
                     "traffic_source": "static ncu figure (DRAM bytes per pass of the 12 launches, "
                                       "captured separately from this run)",
                     "algorithmic_bytes": pass_bytes(t),
                     "kernel": "pair_kernel<NF4> (cta_group::2): q/k/v/o fwd+dX, MLP gate/up+SwiGLU, down, "
                               "down dX+SwiGLU', gate/up two-weight dX; LoRA fused",
                     "peak_source": f"{peak_kind} bf16 dense burst (MEASURED_PEAKS.json)",
                     "launches": glaunch, "ms_per_pass": 1000 * gsec, "per_launch_us": per_launch},
        "clocks": clocks.summary(),
        "device_error": dev_err,
    }
    if rank_steps is not None:
        line["rank_step_ms"] = {"fields": ["mean ms", "min ms", "max ms", "index of the slowest step",
                                           "median SM MHz"], "ranks": rank_steps}
    if ce is not None:
        line["ce"] = ce
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
