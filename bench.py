#!/usr/bin/env python
"""Benchmark of the B200 quaternion linear forward.

Metric: QuaternionLinear microseconds per call (bf16), with the fraction of
the HBM (decode) or tensor-core (prefill) roofline.  One *step* is one call of
the layer on one batch of seeded synthetic input.

Default workload (N=1): the decode layer in=out=4096 bf16, M=1 token, fused
bias [4096] and LoRA rank 32 (the decode configuration of the reference's
benchmark set).  The same run reports, as top-level keys ending the line, the
metric's other halves -- "decode_m16" and "prefill_m2048" (in=4096 ->
out=11008, M=2048) -- and under "also" the fp32 1024 layer, the 5120 -> 27648
layer at M in {1, 16, 512, 8192} and the 48 linears of the GPT-2-small-shaped
stack.  Every kernel number has cuBLAS dense of the same logical shape beside
it, timed the same way.

Timing: W untimed warm-up steps, then exactly K steps captured in one CUDA
graph and replayed once between CUDA events (device time), bracketed by a
barrier and torch.cuda.synchronize() on both sides; the max over ranks is
reported.  Consecutive steps rotate through enough copies of the weights
(and inputs) to exceed the 126 MB L2, so every step streams its weights from
HBM.  "e2e" times K calls of the C ABI's host-buffer entry (qlin_forward_host):
every step copies the input from pinned host memory, runs the layer and
reads the output back; "e2e_module" does the same through the public module
API (torch copies around the module call).

With torchrun (N>1) the headline is the 5120 -> 27648 layer column-partitioned
over the N ranks (out/4 quaternion rows each) at --shard-m tokens (8192 by
default), the full output assembled on every rank inside the timed region
(strong scaling); the same layer unpartitioned on one GPU, the other token
counts and independent decode replicas are extra keys.

CPU baselines (rank 0, N=1): the unmodified reference module
(QuaternionLinear + LoRAQuaternionLinear on CPU torch, installed under
baseline/_ref) -- `--impl reference` prints it as its own line -- and the
oracle's numpy restatement of the reference K1 operator, both under one sample
policy (cpu_sample).
"""

from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = "quaternion-based-math-1_b200"
L2_BYTES = 126 * 2**20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

WORKLOADS = {
    "decode_m1": dict(fn="decode_4096", M=1, bound="hbm"),
    "decode_m16": dict(fn="decode_4096", M=16, bound="hbm"),
    "prefill_m2048": dict(fn="prefill_11008", M=2048, bound="tensor"),
    # the fp32 layer in=out=1024 at M=128 (CUDA-core fp32 path)
    "fp32_m128": dict(fn="fp32_1024", M=128, bound="fp32"),
    # the large layer in=5120 -> out=27648 on one GPU (the sharded sweep's N=1 points)
    "large_m1": dict(fn="sharded_27648", M=1, bound="hbm"),
    "large_m16": dict(fn="sharded_27648", M=16, bound="hbm"),
    "large_m512": dict(fn="sharded_27648", M=512, bound="tensor"),
    "large_m8192": dict(fn="sharded_27648", M=8192, bound="tensor"),
}
DEFAULT = "decode_m1"
# FP32 CUDA-core peak (no measured figure exists): 148 SMs x 128 lanes x 2
# FLOP x 1.965 GHz, nominal.
FP32_NOMINAL_TFLOPS = 74.4


def _pkg():
    if REPO not in sys.path:
        sys.path.insert(0, REPO)
    return importlib.import_module(PKG), importlib.import_module(f"{PKG}.workloads")


def _oracle():
    p = os.path.join(REPO, "oracle")
    if p not in sys.path:
        sys.path.insert(0, p)
    import oracle  # the CPU restatement: timed baseline only

    return oracle


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def _traffic(workload):
    """DRAM bytes per launch of the workload's main kernel from the ncu
    summary table in profiles/ (None when no capture is recorded)."""
    path = os.path.join(REPO, "profiles", "dram_traffic_per_launch.md")
    try:
        with open(path) as f:
            for line in f:
                cells = [c.strip() for c in line.strip().strip("|").split("|")]
                if len(cells) >= 4 and cells[0] == workload and cells[2].isdigit():
                    return int(cells[2]), f"profiles/{cells[3]}"
    except OSError:
        pass
    return None, None


def _layer(wl, name):
    spec = WORKLOADS[name]
    return getattr(wl, spec["fn"])(spec["M"])


def algorithmic_work(lay):
    """(bytes, flops) one call must move / perform, from the layer's shapes."""
    es = 2 if lay.dtype != "f32" else 4
    M, K, N = lay.M, 4 * lay.K_g, 4 * lay.N_g
    nbytes = es * (4 * lay.N_g * lay.K_g + M * K + M * N)
    flops = 2.0 * M * N * K
    if lay.bias is not None:
        nbytes += es * N
    if lay.lora_a is not None:
        r = lay.lora_a.shape[0]
        nbytes += es * (r * K + N * r)
        flops += 2.0 * M * r * (K + N)
    return nbytes, flops


def workload_config(name, lay, ncopy):
    return {
        "workload": f"qlinear_{4 * lay.K_g}x{4 * lay.N_g}_{lay.dtype}_m{lay.M}"
                    + ("_bias" if lay.bias is not None else "")
                    + (f"_lora{lay.lora_a.shape[0]}" if lay.lora_a is not None else ""),
        "name": name,
        "M": lay.M,
        "in_features": 4 * lay.K_g,
        "out_features": 4 * lay.N_g,
        "lora_rank": 0 if lay.lora_a is None else int(lay.lora_a.shape[0]),
        "bias": lay.bias is not None,
        "seed": lay.meta.get("seed"),
        "inputs": "seeded synthetic N(0,1) activations, N(0,1/in) weights (variance), "
                  "bias N(0,0.02), LoRA N(0,0.01)",
        "l2": f"inputs larger than L2: {ncopy} rotating copies of weights/inputs",
    }


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in getattr(self, "lines", []):
            f = [c.strip() for c in ln.split(",")]
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
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# device timing
# ---------------------------------------------------------------------------

def _ncopy(lay, min_bytes=2 * L2_BYTES):
    """Copies of a workload's weights and inputs that the timed steps rotate
    through so that together they exceed L2 (at least two)."""
    nbytes, _ = algorithmic_work(lay)
    return max(2, min(64, math.ceil(min_bytes / max(nbytes, 1))))


def _device_case(qb, lay, torch, dev, min_bytes=2 * L2_BYTES, flags=0, algo=0, packed=False):
    """Device copies rotated to exceed L2, preallocated outputs and workspace.
    packed: the calls go through qlin_forward_packed with the packed weight
    cache only (no planar weights)."""
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[lay.dtype]
    ncopy = _ncopy(lay, min_bytes)

    def t(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dt)

    base = dict(x=t(lay.x), w=[t(a) for a in lay.weights], b=t(lay.bias), la=t(lay.lora_a),
                lb=t(lay.lora_b))
    copies = [base]
    for _ in range(ncopy - 1):
        copies.append({k: (None if v is None else ([a.clone() for a in v] if isinstance(v, list)
                                                    else v.clone()))
                       for k, v in base.items()})
    M, K_g, N_g = lay.M, lay.K_g, lay.N_g
    rank = 0 if lay.lora_a is None else lay.lora_a.shape[0]
    ys = [torch.empty(M, 4 * N_g, dtype=dt, device=dev) for _ in range(ncopy)]
    ws_bytes = qb._lib.workspace_size(dt, M, K_g, N_g, rank)
    # a zero-filled workspace reused by every call (QLIN_FLAG_ZEROED_WORKSPACE):
    # decode-sized K splits are then summed inside the main kernel
    ws = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    flags |= qb._lib.FLAG_ZEROED_WORKSPACE
    lib = qb._lib.load()
    code = qb._lib.dtype_code(dt)
    stream_of = qb._lib.stream_handle

    if packed:
        for c in copies:
            c["wq"] = qb.pack_quaternion_weights(*c["w"])
            c["w"] = None
        torch.cuda.empty_cache()

    def call(i):
        c = copies[i % ncopy]
        y = ys[i % ncopy]
        if packed:
            st = lib.qlin_forward_packed(code, c["x"].data_ptr(), 4 * K_g, c["wq"].data_ptr(), K_g, None, None,
                                         None, None, K_g, c["b"].data_ptr() if c["b"] is not None else None,
                                         c["la"].data_ptr() if c["la"] is not None else None,
                                         c["lb"].data_ptr() if c["lb"] is not None else None,
                                         rank, float(lay.lora_scale), y.data_ptr(), 4 * N_g, M, K_g, N_g,
                                         ws.data_ptr(), ws_bytes, flags, stream_of(dev))
            if st != 0:
                qb._lib.check(st, "qlin_forward_packed")
            return
        st = lib.qlin_forward_ex(code, c["x"].data_ptr(), 4 * K_g, *(w.data_ptr() for w in c["w"]), K_g,
                                 c["b"].data_ptr() if c["b"] is not None else None,
                                 c["la"].data_ptr() if c["la"] is not None else None,
                                 c["lb"].data_ptr() if c["lb"] is not None else None,
                                 rank, float(lay.lora_scale), y.data_ptr(), 4 * N_g, M, K_g, N_g,
                                 ws.data_ptr(), ws_bytes, algo, flags, stream_of(dev))
        if st != 0:
            qb._lib.check(st, "qlin_forward")

    with torch.cuda.device(dev):
        plan = qb._lib.plan(dt, M, K_g, N_g, rank, flags=flags)
    if algo == qb._lib.ALGO_TC and plan["algo"] != "tcgen05":
        plan = {"algo": "tcgen05 (forced)"}
    return call, ncopy, copies, ys, plan


def _settle(torch, dev, fn, seconds=0.5):
    """Untimed repetitions of fn for about `seconds`: the first timed region
    of a process otherwise runs before the GPU has left its idle clocks
    (measured: 15-25% slower decode calls)."""
    end = time.time() + seconds
    while time.time() < end:
        fn()
        torch.cuda.synchronize(dev)


def time_device(qb, lay, torch, dev, K, W, dist=None, flags=0, algo=0, packed=False):
    call, ncopy, copies, ys, plan = _device_case(qb, lay, torch, dev, flags=flags, algo=algo, packed=packed)
    for i in range(W):
        call(i)
    torch.cuda.synchronize(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        call(0)  # stream warm-up before capture
    torch.cuda.current_stream(dev).wait_stream(side)
    with torch.cuda.graph(graph):
        for i in range(K):
            call(i)
    _settle(torch, dev, graph.replay)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    graph.replay()
    end.record()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    ms = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del graph
    return ms, ncopy, plan


def time_stack(qb, wl, torch, dev, R, W):
    """All 48 quaternion linears of one forward of the GPT-2-small-shaped
    stack (12 blocks x qkv/proj/fc/fc2, M = 8 x 1024 tokens, bf16), captured
    as one CUDA graph of 48 qlin_forward_ex calls and replayed R times.
    Each layer reads its own weights and an N(0,1) activation of its input
    width; the whole footprint (about 200 MB) exceeds L2."""
    layers = wl.gpt2_stack()
    lib = qb._lib.load()
    code = qb._lib.dtype_code(torch.bfloat16)
    M = layers[0].M
    xs, ys = {}, {}
    calls = []
    flops = 0.0
    for lay in layers:
        fin, fout = 4 * lay.K_g, 4 * lay.N_g
        if fin not in xs:
            xs[fin] = torch.from_numpy(lay.x).to(dev, torch.bfloat16)
        if fout not in ys:
            ys[fout] = torch.empty(M, fout, dtype=torch.bfloat16, device=dev)
        w = [torch.from_numpy(a).to(dev, torch.bfloat16) for a in lay.weights]
        nws = qb._lib.workspace_size(torch.bfloat16, M, lay.K_g, lay.N_g, 0)
        ws = torch.zeros(max(nws, 256), dtype=torch.uint8, device=dev)
        calls.append((xs[fin], w, ys[fout], lay.K_g, lay.N_g, ws, nws))
        flops += 2.0 * M * fin * fout
    stream_of = qb._lib.stream_handle

    def forward():
        for x, w, y, K_g, N_g, ws, nws in calls:
            st = lib.qlin_forward_ex(code, x.data_ptr(), 4 * K_g, *(a.data_ptr() for a in w), K_g,
                                     None, None, None, 0, 0.0, y.data_ptr(), 4 * N_g, M, K_g, N_g,
                                     ws.data_ptr(), nws, 0, qb._lib.FLAG_ZEROED_WORKSPACE, stream_of(dev))
            if st != 0:
                qb._lib.check(st, "qlin_forward")

    for _ in range(W):
        forward()
    torch.cuda.synchronize(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        forward()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        forward()
    _settle(torch, dev, graph.replay, 0.3)
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(R):
        graph.replay()
    e.record()
    torch.cuda.synchronize(dev)
    us = s.elapsed_time(e) * 1e3 / R
    plans = {f"{4 * k}x{4 * n}": qb._lib.plan(torch.bfloat16, M, k, n, 0)
             for (_, _, _, k, n, _, _) in calls[:4]}
    del graph
    return us, flops, len(calls), plans


def time_converted_gpt2(qb, torch, dev, R, W, M=8 * 1024):
    """The 48 quaternion linears of a converted GPT-2-small: a transformers
    GPT2LMHeadModel built from its config (12 blocks, d=768, 12 heads, MLP
    3072; random init, seed 0 -- no checkpoints offline) in bf16, whose
    c_attn / c_proj / c_fc / c_proj projections convert_model (the
    reference's matrix method) replaced with QuaternionLinear layers (the
    least-squares quaternion components of each dense weight, biases kept).
    One forward of every converted layer through the module API (fused
    bias) on N(0,1) activations of M = 8 x 1024 tokens, captured as one CUDA
    graph and replayed R times.  Returns (us per forward, FLOP, layers)."""
    import transformers

    torch.manual_seed(0)
    cfg = transformers.GPT2Config(n_layer=12, n_embd=768, n_head=12, n_positions=1024, n_inner=3072)
    model = transformers.GPT2LMHeadModel(cfg).to(dev, torch.bfloat16).eval()
    _, records = qb.convert_model(model)
    layers = [model.get_submodule(r.name) for r in records]
    g = torch.Generator(device="cpu").manual_seed(1)
    xs = {}
    flops = 0.0
    for layer in layers:
        if layer.in_features not in xs:
            xs[layer.in_features] = torch.randn(M, layer.in_features, generator=g).to(dev, torch.bfloat16)
        flops += 2.0 * M * layer.in_features * layer.out_features

    def forward():
        for layer in layers:
            layer(xs[layer.in_features])

    with torch.inference_mode():
        for _ in range(W):
            forward()
        torch.cuda.synchronize(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            forward()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            forward()
        _settle(torch, dev, graph.replay, 0.3)
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(R):
            graph.replay()
        e.record()
        torch.cuda.synchronize(dev)
    del graph, model
    return s.elapsed_time(e) * 1e3 / R, flops, len(layers)


def _time_ranks(torch, dev, dist, call, steps, W):
    """Device time per call of call(i) on every rank, max over ranks: steps
    calls captured in one CUDA graph (eager launches if capture is refused)."""
    for i in range(W):
        call(i)
    torch.cuda.synchronize(dev)
    mode = "graph"
    graph = None
    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            call(0)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(steps):
                call(i)
    except Exception:  # capture refused: time eager launches
        graph = None
        mode = "eager"
        torch.cuda.synchronize(dev)
    dist.barrier()
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    if graph is not None:
        graph.replay()
    else:
        for i in range(steps):
            call(i)
    e.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([s.elapsed_time(e) * 1e3 / steps], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del graph
    torch.cuda.synchronize(dev)
    return float(t.item()), mode


def time_sharded(qb, wl, torch, dev, dist, world, rank, W, cases):
    """The large layer (in=5120 -> out=27648) column-partitioned over the
    torchrun world: rank r runs the kernel on its out/4 rows (N_g/world of
    6912).  Two ways to assemble [M, 27648] on every rank are timed: NCCL
    (all-gather of the [M, 4*N_g/world] outputs over NVLink, then for M > 1
    the column-gather kernel) and fused (qlin_forward_allgather: entry flag
    barrier, the epilogue stores into every rank's output over NVLink, exit
    flag barrier).  Each is captured in a CUDA graph (eager launches if
    capture is refused); device time, max over ranks.  Weight shards rotate
    across more than L2.  `cases` is a list of (M, steps).  The fused
    roofline target is the slower of the shard's compute (or HBM) time and
    its NVLink traffic at 770 GB/s per direction: (world - 1) shards' outputs
    leave each rank (peer stores) and, multicast or not, arrive at each rank."""
    lib = qb._lib.load()
    code = qb._lib.dtype_code(torch.bfloat16)
    stream_of = qb._lib.stream_handle
    peaks_ref, _ = _peaks()
    out = {}
    for M, steps in cases:
        lay = wl.sharded_27648(M)
        N_g, K_g = lay.N_g, lay.K_g
        n = -(-N_g // world)
        b0, b1 = min(rank * n, N_g), min(rank * n + n, N_g)
        shard_bytes = 4 * n * K_g * 2
        ncopy = max(2, min(32, math.ceil(2 * L2_BYTES / shard_bytes)))
        shards = []
        for _ in range(ncopy):
            ws_ = []
            for a in lay.weights:
                t = torch.zeros(n, K_g, dtype=torch.bfloat16, device=dev)
                t[:b1 - b0].copy_(torch.from_numpy(a[b0:b1]))
                ws_.append(t)
            shards.append(ws_)
        x = torch.from_numpy(lay.x).to(dev, torch.bfloat16)
        y_loc = torch.empty(M, 4 * n, dtype=torch.bfloat16, device=dev)
        flat = torch.empty(world * M, 4 * n, dtype=torch.bfloat16, device=dev)
        y_full = torch.empty(M, 4 * n * world, dtype=torch.bfloat16, device=dev)
        nws = qb._lib.workspace_size(torch.bfloat16, M, K_g, n, 0)
        wsb = torch.zeros(max(nws, 256), dtype=torch.uint8, device=dev)

        def call(i):
            w = shards[i % ncopy]
            st = lib.qlin_forward_ex(code, x.data_ptr(), 4 * K_g, *(a.data_ptr() for a in w), K_g, None, None,
                                     None, 0, 0.0, y_loc.data_ptr(), 4 * n, M, K_g, n, wsb.data_ptr(), nws, 0,
                                     qb._lib.FLAG_ZEROED_WORKSPACE, stream_of(dev))
            if st != 0:
                qb._lib.check(st, "qlin_forward")
            dist.all_gather_into_tensor(flat, y_loc)
            if M > 1:
                qb._lib.check(lib.qlin_gather_columns(code, flat.data_ptr(), y_full.data_ptr(), world, M, 4 * n,
                                                      4 * n * world, stream_of(dev)), "qlin_gather_columns")

        # the same shard computation with the all-gather fused into the
        # epilogue: outputs stored into every rank's full output over NVLink
        po = qb.PeerOutputs(M, 4 * n * world, torch.bfloat16, dev)

        def call_fused(i):
            w = shards[i % ncopy]
            st = lib.qlin_forward_allgather(code, x.data_ptr(), 4 * K_g, *(a.data_ptr() for a in w), K_g, None,
                                            None, None, 0, 0.0, M, K_g, n, wsb.data_ptr(), nws,
                                            qb._lib.FLAG_ZEROED_WORKSPACE, world, rank, po._outs, 4 * n * world,
                                            4 * n * rank, po._flags, po.epoch.data_ptr(), stream_of(dev))
            if st != 0:
                qb._lib.check(st, "qlin_forward_allgather")

        # and with one multicast store per output piece (NVLink multicast
        # through NVSwitch), where every rank has it
        ok = torch.tensor([int(qb.MulticastOutputs.available(dev))], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        mco = qb.MulticastOutputs(M, 4 * n * world, torch.bfloat16, dev) if ok.item() else None

        def call_mc(i):
            w = shards[i % ncopy]
            st = lib.qlin_forward_allgather_mc(code, x.data_ptr(), 4 * K_g, *(a.data_ptr() for a in w), K_g, None,
                                               None, None, 0, 0.0, M, K_g, n, wsb.data_ptr(), nws,
                                               qb._lib.FLAG_ZEROED_WORKSPACE, world, rank, mco.out.data_ptr(),
                                               mco.mc, 4 * n * world, 4 * n * rank, mco._flags,
                                               mco.epoch.data_ptr(), stream_of(dev))
            if st != 0:
                qb._lib.check(st, "qlin_forward_allgather_mc")

        us, mode = _time_ranks(torch, dev, dist, call, steps, W)
        us_f, mode_f = _time_ranks(torch, dev, dist, call_fused, steps, W)
        same = bool(torch.equal(po.out, y_full if M > 1 else flat.view(M, -1)))
        us_mc = same_mc = None
        if mco is not None:
            us_mc, _ = _time_ranks(torch, dev, dist, call_mc, steps, W)
            same_mc = bool(torch.equal(mco.out, po.out))
        nbytes = 2 * (4 * n * K_g + M * 4 * K_g + M * 4 * n)
        flops = 2.0 * M * 4 * K_g * 4 * n
        best = min(v for v in (us, us_f, us_mc) if v is not None)
        if M <= 16:
            a = nbytes / (best * 1e-6) / 1e9
            roof = {"bound": "hbm", "achieved_per_gpu": a, "unit": "GB/s", "peak": peaks_ref["hbm_gbs"],
                    "frac_per_gpu": a / peaks_ref["hbm_gbs"], "basis": "shard bytes per GPU"}
        else:
            a = flops / (best * 1e-6) / 1e12
            roof = {"bound": "tensor", "achieved_per_gpu": a, "unit": "TFLOP/s", "peak": peaks_ref["bf16_tflops"],
                    "frac_per_gpu": a / peaks_ref["bf16_tflops"], "basis": "shard FLOP per GPU"}
        egress = (world - 1) * M * 4 * n * 2  # bytes each rank stores to its peers
        t_nvl = egress / 770e9 * 1e6          # at the measured 770 GB/s peer copy, per direction
        # multicast sends each rank's columns over its links once, but every
        # rank still receives the other ranks' columns: the same ingress bound
        t_nvl_mc = t_nvl
        t_cmp = (nbytes / (peaks_ref["hbm_gbs"] * 1e9) if M <= 16 else flops / (peaks_ref["bf16_tflops"] * 1e12)) * 1e6
        launches = qb._lib.plan(torch.bfloat16, M, K_g, n, 0, flags=qb._lib.FLAG_ZEROED_WORKSPACE)["launches"]
        out[M] = {"us_nccl": us, "us_fused": us_f, "steps": steps, "timing": [mode, mode_f], "shard_rows": n,
                  "fused_equals_nccl": same, "roofline": roof,
                  "fused_target_us": max(t_nvl, t_cmp), "fused_frac_of_target": max(t_nvl, t_cmp) / us_f,
                  "nvlink_us": t_nvl, "launches_fused": launches + 2}
        if us_mc is not None:
            out[M].update({"us_fused_mc": us_mc, "mc_equals_fused": same_mc,
                           "mc_target_us": max(t_nvl_mc, t_cmp), "mc_frac_of_target": max(t_nvl_mc, t_cmp) / us_mc})
        del shards, x, y_loc, flat, y_full, wsb, mco
        torch.cuda.empty_cache()
    return out


def time_sharded_e2e(qb, wl, torch, dev, dist, world, M, K, W):
    """K calls of the column-partitioned 5120->27648 layer through the public
    module (ColumnParallelQuaternionLinear: its fused NVLink all-gather for
    M >= 64), each with the input copied from pinned host memory and the
    full output read back to pinned host memory; max over ranks."""
    lay = wl.sharded_27648(M)
    full = qb.QuaternionLinear(5120, 27648, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        for name, a in zip(("wr", "wi", "wj", "wk"), lay.weights):
            getattr(full, name).copy_(torch.from_numpy(a))
    mod = qb.ColumnParallelQuaternionLinear.from_full(full)
    del full
    torch.cuda.empty_cache()
    x_host = torch.from_numpy(lay.x).to(torch.bfloat16).pin_memory()
    y_host = torch.empty(M, 27648, dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty(M, 5120, dtype=torch.bfloat16, device=dev)

    def step():
        x_dev.copy_(x_host, non_blocking=True)
        y = mod(x_dev)
        y_host.copy_(y, non_blocking=True)

    with torch.inference_mode():
        for _ in range(W):
            step()
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(K):
            step()
        e.record()
        torch.cuda.synchronize(dev)
    t = torch.tensor([s.elapsed_time(e) * 1e3 / K], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), M * 5120 * 2, M * 27648 * 2


def time_dense(lay, torch, dev, K, W):
    """cuBLAS x @ W^T of the same logical shape (context only), captured in
    one CUDA graph and replayed between CUDA events exactly like our calls."""
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[lay.dtype]
    M, Kf, N = lay.M, 4 * lay.K_g, 4 * lay.N_g
    wbytes = N * Kf * dt.itemsize
    ncopy = max(2, min(32, math.ceil(2 * L2_BYTES / (wbytes + dt.itemsize * M * (Kf + N)))))
    g = torch.Generator(device="cpu").manual_seed(0)
    ws = [(torch.randn(N, Kf, generator=g) / math.sqrt(Kf)).to(dev, dt) for _ in range(ncopy)]
    xs = [torch.randn(M, Kf, generator=g).to(dev, dt) for _ in range(ncopy)]
    ys = [torch.empty(M, N, device=dev, dtype=dt) for _ in range(ncopy)]

    def call(i):
        torch.matmul(xs[i % ncopy], ws[i % ncopy].t(), out=ys[i % ncopy])

    for i in range(W):
        call(i)
    torch.cuda.synchronize(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        call(0)
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(K):
            call(i)
    _settle(torch, dev, graph.replay, 0.3)
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize(dev)
    del graph
    return s.elapsed_time(e) * 1e3 / K


def time_e2e_abi(qb, lay, torch, dev, K, W):
    """K calls of the C ABI's host-buffer entry (qlin_forward_host, through
    the package's CPython binding of it): every step copies x from page-locked
    host memory to the device, runs the layer and copies y back to
    page-locked host memory, all on the stream; the device weights rotate
    over copies larger than L2 as in the device timing."""
    _, ncopy, copies, _, _ = _device_case(qb, lay, torch, dev)
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[lay.dtype]
    M, K_g, N_g = lay.M, lay.K_g, lay.N_g
    rank = 0 if lay.lora_a is None else lay.lora_a.shape[0]
    lib = qb._lib.load()
    code = qb._lib.dtype_code(dt)
    x_host = torch.from_numpy(lay.x).to(dt).pin_memory()
    y_host = torch.empty(M, 4 * N_g, dtype=dt).pin_memory()
    n = ctypes.c_size_t(0)
    qb._lib.check(lib.qlin_host_workspace_size(code, M, K_g, N_g, rank, ctypes.byref(n)), "qlin_host_workspace_size")
    ws = torch.zeros(max(n.value, 256), dtype=torch.uint8, device=dev)
    fn = qb._lib._fast.forward_host if qb._lib._fast is not None else lib.qlin_forward_host
    stream = qb._lib.stream_handle(dev)
    flags = qb._lib.FLAG_ZEROED_WORKSPACE
    args = []
    for c in copies:
        args.append((code, x_host.data_ptr(), 4 * K_g, *(w.data_ptr() for w in c["w"]), K_g,
                     c["b"].data_ptr() if c["b"] is not None else None,
                     c["la"].data_ptr() if c["la"] is not None else None,
                     c["lb"].data_ptr() if c["lb"] is not None else None, rank, float(lay.lora_scale),
                     y_host.data_ptr(), 4 * N_g, M, K_g, N_g, ws.data_ptr(), n.value, 0, flags, stream))

    def step(i):
        st = fn(*args[i % ncopy])
        if st != 0:
            qb._lib.check(st, "qlin_forward_host")

    for i in range(W):
        step(i)
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(K):
        step(i)
    e.record()
    torch.cuda.synchronize(dev)
    es = x_host.element_size()
    return s.elapsed_time(e) * 1e3 / K, M * 4 * K_g * es, M * 4 * N_g * es


def time_e2e(qb, lay, torch, dev, K, W):
    """K steps through the public module API with host input and host output."""
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[lay.dtype]
    nbytes, _ = algorithmic_work(lay)
    ncopy = max(2, min(32, math.ceil(2 * L2_BYTES / max(nbytes, 1))))
    fin, fout = 4 * lay.K_g, 4 * lay.N_g
    layers = []
    for c in range(ncopy):
        base = qb.QuaternionLinear(fin, fout, bias=lay.bias is not None, device=dev, dtype=dt)
        with torch.no_grad():
            for n, a in zip(("wr", "wi", "wj", "wk"), lay.weights):
                getattr(base, n).copy_(torch.from_numpy(a))
            if lay.bias is not None:
                base.bias.copy_(torch.from_numpy(lay.bias))
        mod = base
        if lay.lora_a is not None:
            mod = qb.LoRAQuaternionLinear(base, rank=lay.lora_a.shape[0])
            with torch.no_grad():
                mod.lora_A.copy_(torch.from_numpy(lay.lora_a))
                mod.lora_B.copy_(torch.from_numpy(lay.lora_b))
        mod.eval()
        layers.append(mod)
    x_host = torch.from_numpy(lay.x).to(dt).pin_memory()
    y_host = torch.empty(lay.M, fout, dtype=dt).pin_memory()
    x_dev = torch.empty(lay.M, fin, dtype=dt, device=dev)

    def step(i):
        x_dev.copy_(x_host, non_blocking=True)
        y = layers[i % ncopy](x_dev)
        y_host.copy_(y, non_blocking=True)

    with torch.inference_mode():
        for i in range(W):
            step(i)
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(K):
            step(i)
        e.record()
        torch.cuda.synchronize(dev)
    es = x_host.element_size()
    return s.elapsed_time(e) * 1e3 / K, lay.M * fin * es, lay.M * fout * es


# ---------------------------------------------------------------------------
# CPU baselines, one sample policy for both: the unmodified reference module
# (installed under baseline/_ref) and the oracle's numpy restatement of K1
# ---------------------------------------------------------------------------

def _reference_modules():
    """(QuaternionLinear, LoRAQuaternionLinear) of the unmodified reference
    package installed under baseline/_ref, or None when it is absent."""
    root = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(root, "quaternion")):
        return None
    if root not in sys.path:
        sys.path.insert(0, root)
    try:
        from quaternion.linear import QuaternionLinear  # the reference package (CPU torch)
        from quaternion.lora import LoRAQuaternionLinear
    except ImportError:
        return None
    return QuaternionLinear, LoRAQuaternionLinear


def reference_cpu_call(lay):
    """The reference's own module path on CPU torch, in the layer's dtype:
    QuaternionLinear.forward (quaternion/linear.py:120-124), wrapped in
    LoRAQuaternionLinear.forward (quaternion/lora.py:60-63) when the layer has
    LoRA.  Returns call(rows) or None when the reference is not installed."""
    mods = _reference_modules()
    if mods is None:
        return None
    import torch

    QL, LQL = mods
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[lay.dtype]
    base = QL(4 * lay.K_g, 4 * lay.N_g, bias=lay.bias is not None, dtype=dt)
    with torch.no_grad():
        for n, a in zip(("wr", "wi", "wj", "wk"), lay.weights):
            getattr(base, n).copy_(torch.from_numpy(a))
        if lay.bias is not None:
            base.bias.copy_(torch.from_numpy(lay.bias))
    mod = base
    if lay.lora_a is not None:
        mod = LQL(base, rank=lay.lora_a.shape[0])
        with torch.no_grad():
            mod.lora_A.copy_(torch.from_numpy(lay.lora_a))
            mod.lora_B.copy_(torch.from_numpy(lay.lora_b))
    mod.eval()
    x = torch.from_numpy(lay.x).to(dt)

    def call(rows):
        with torch.inference_mode():
            return mod(x[: len(rows)])

    return call


def cpu_port_call(oracle, lay, rows):
    """quaternion/planar.py:39-61 (+ bias, + lora.py:60-63) in float32 BLAS."""
    x = lay.x[rows]
    y = oracle.quaternion_linear_naive(x, *lay.weights, dtype=np.float32)
    if lay.bias is not None:
        y = y + lay.bias
    if lay.lora_a is not None:
        y = y + np.float32(lay.lora_scale) * ((x @ lay.lora_a.T) @ lay.lora_b.T)
    return y


def cpu_sample(fn, M, steps, warmup, budget_s):
    """The one CPU sample policy: a step runs fn on the first `rows` tokens,
    rows = M unless one call of M tokens would exceed 0.25 s (then as many
    tokens as fit, the time scaled to M); `warmup` untimed steps, then up to
    `steps` timed ones, stopping once `budget_s` has passed (at least 3).
    Returns (us per call of M tokens, timed steps, rows)."""
    probe = min(M, 8)
    t0 = time.perf_counter()
    fn(np.arange(probe))
    per_row = max((time.perf_counter() - t0) / probe, 1e-7)
    rows_n = M if per_row * M <= 0.25 else max(1, min(M, int(0.25 / per_row)))
    rows = np.arange(rows_n)
    for _ in range(warmup):
        fn(rows)
    times = []
    t_start = time.perf_counter()
    while len(times) < steps:
        t0 = time.perf_counter()
        fn(rows)
        times.append(time.perf_counter() - t0)
        if len(times) >= 3 and time.perf_counter() - t_start > budget_s:
            break
    return statistics.median(times) * (M / rows_n) * 1e6, len(times), rows_n


def cpu_baselines(lay, steps, warmup, budget_s):
    """(primary, port): the reference module on CPU torch (kind "reference")
    when installed, else the port; and the port itself (kind "port")."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    oracle = _oracle()
    try:
        from threadpoolctl import threadpool_limits
        ctx = threadpool_limits(limits=threads)
    except ImportError:  # pragma: no cover
        ctx = None
    port_us, n, rows = cpu_sample(lambda r: cpu_port_call(oracle, lay, r), lay.M, steps, warmup, budget_s)
    port = {"value": port_us, "unit": "us/call", "cores": threads, "kind": "port",
            "sample": f"{n} calls of the oracle's numpy/OpenBLAS float32 restatement of the reference K1 "
                      f"operator (+bias, +LoRA) on {rows} of {lay.M} token rows, scaled to the batch"}
    if ctx is not None and hasattr(ctx, "unregister"):
        ctx.unregister()
    ref_fn = reference_cpu_call(lay)
    if ref_fn is None:
        return port, port
    ref_us, n, rows = cpu_sample(ref_fn, lay.M, steps, warmup, budget_s)
    ref = {"value": ref_us, "unit": "us/call", "cores": threads, "kind": "reference",
           "sample": f"{n} calls of the unmodified reference module (QuaternionLinear"
                     f"{' + LoRAQuaternionLinear' if lay.lora_a is not None else ''}, CPU torch "
                     f"{torch.__version__}, {lay.dtype}) on {rows} of {lay.M} token rows, scaled to the batch"}
    return ref, port


# ---------------------------------------------------------------------------

def _roofline(bound, nbytes, flops, us, peaks, peak_src=None, launches=None, workload=None):
    if bound == "hbm":
        a = nbytes / (us * 1e-6) / 1e9
        r = {"bound": "hbm", "achieved": a, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": a / peaks["hbm_gbs"]}
    elif bound == "fp32":
        a = flops / (us * 1e-6) / 1e12
        r = {"bound": "fp32 CUDA cores", "achieved": a, "peak": FP32_NOMINAL_TFLOPS, "unit": "TFLOP/s",
             "frac": a / FP32_NOMINAL_TFLOPS, "peak_source": "nominal"}
    else:
        a = flops / (us * 1e-6) / 1e12
        r = {"bound": "tensor", "achieved": a, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
             "frac": a / peaks["bf16_tflops"]}
    if workload is not None:
        traffic, tsrc = _traffic(workload)
        r["traffic"] = traffic
        r["traffic_source"] = tsrc
        r["basis"] = (f"{nbytes} algorithmic bytes" if bound == "hbm" else f"{flops:.4g} dense-equivalent FLOP") + \
            f" per call / device time per call ({launches} launches per call)"
    if peak_src is not None and "peak_source" not in r:
        r["peak_source"] = peak_src
    return r


def _entry(qb, wl, torch, dev, name, K, W, peaks, with_clocks=False):
    """Compact record of one secondary workload: device us/call, roofline,
    cuBLAS dense of the same logical shape (same graph-replay timing)."""
    lay = _layer(wl, name)
    bound = WORKLOADS[name]["bound"]
    kk = K if bound == "hbm" else max(3, min(K, 100))
    if with_clocks:
        with ClockSampler(dev.index) as clk:
            ms, _, plan = time_device(qb, lay, torch, dev, kk, W)
        clocks = clk.summary()
    else:
        ms, _, plan = time_device(qb, lay, torch, dev, kk, W)
        clocks = None
    us = ms * 1e3 / kk
    nb, fl = algorithmic_work(lay)
    if name == "prefill_m2048":
        pms, _, _ = time_device(qb, lay, torch, dev, kk, W, packed=True)
        packed_us = pms * 1e3 / kk
    else:
        packed_us = None
    e = {"value": us, "unit": "us/call", "steps": kk, "launches": plan["launches"], "algo": plan["algo"],
         "roofline": _roofline(bound, nb, fl, us, peaks, None, plan["launches"], name),
         "dense_cublas_us": time_dense(lay, torch, dev, kk, W)}
    if clocks is not None:
        e["clocks"] = clocks
    if packed_us is not None:
        e["packed_weights_us_per_call"] = packed_us
    return e


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=DEFAULT, choices=sorted(WORKLOADS))
    ap.add_argument("--no-extra", action="store_true", help="skip the secondary workloads")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--shard-m", type=int, default=8192,
                    help="tokens of the column-partitioned headline at --gpus N > 1")
    args = ap.parse_args()
    K, W = args.steps, max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    qb, wl = _pkg()
    metric = "QuaternionLinear us/call (bf16), % of HBM/TC roofline"

    if args.impl == "reference":
        if rank != 0:
            return
        lay = _layer(wl, args.workload)
        ref, port = cpu_baselines(lay, K, W, budget_s=60.0)
        # the same config record as the device arm's (it does not rotate
        # copies, but the workload is identical)
        cfg = dict(workload_config(args.workload, lay, _ncopy(lay)), parallelism="single")
        print(json.dumps({
            "impl": "reference", "metric": metric, "value": ref["value"], "unit": "us/call",
            "n_gpus": args.gpus, "steps": K, "warmup": W, "ms_per_step": ref["value"] / 1e3,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": f"{lay.dtype} (CPU)", "data": "synthetic", "config": cfg,
            "cpu_baseline": ref, "cpu_port": port,
            "e2e": {"value": ref["value"], "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return

    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        torch.cuda.set_device(local)
        # keep stdout to the one JSON line: whatever the communicator set-up
        # prints (NCCL's version banner) goes to stderr
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                     device_id=torch.device("cuda", local))
            tdist.barrier()
            torch.cuda.synchronize(local)
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
        dist = tdist
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks, peak_src = _peaks()

    if dist is not None:
        result = main_partitioned(qb, wl, torch, dev, dist, world, rank, K, W, args.shard_m, metric, peaks,
                                  peak_src)
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(result), flush=True)
        return

    lay = _layer(wl, args.workload)
    nbytes, flops = algorithmic_work(lay)
    with ClockSampler(local) as clk:
        ms, ncopy, plan = time_device(qb, lay, torch, dev, K, W)
    launches = plan["launches"]
    us_call = ms * 1e3 / K
    bound = WORKLOADS[args.workload]["bound"]
    result = {
        "metric": metric, "value": us_call, "unit": "us/call", "n_gpus": 1,
        "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": lay.dtype, "data": "synthetic",
        "config": dict(workload_config(args.workload, lay, ncopy), parallelism="single"),
        "roofline": _roofline(bound, nbytes, flops, us_call, peaks, peak_src, launches, args.workload),
        "clocks": clk.summary(),
        "gpu_launches": K * launches,
        "plan": plan,
    }
    # Same workload with the weights declared static (inference): each call
    # streams its weights while the previous call's kernels finish.
    sms, _, _ = time_device(qb, lay, torch, dev, K, W, flags=qb._lib.FLAG_STATIC_WEIGHTS)
    result["static_weights_us_per_call"] = sms * 1e3 / K
    # the same calls on the packed weight cache only (qlin_forward_packed;
    # null where the layer's kernel needs the planar weights)
    try:
        pms, _, _ = time_device(qb, lay, torch, dev, K, W, packed=True)
        result["packed_weights_us_per_call"] = pms * 1e3 / K
    except RuntimeError:
        result["packed_weights_us_per_call"] = None
    # end to end with host buffers: through the C ABI's host entry (the
    # reference-facing boundary a non-Python host binds), and through the
    # Python module API (copies by torch around the module call)
    e2e_us, h2d, d2h = time_e2e_abi(qb, lay, torch, dev, K, W)
    result["e2e"] = {"value": e2e_us, "unit": "us/call", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                     "through": "qlin_forward_host (C ABI, pinned host x and y)"}
    m_us, h2d, d2h = time_e2e(qb, lay, torch, dev, K, W)
    result["e2e_module"] = {"value": m_us, "unit": "us/call", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                            "through": "LoRAQuaternionLinear / QuaternionLinear forward, torch copies"}
    result["dense_cublas_us"] = time_dense(lay, torch, dev, K, W)
    if rank == 0:
        ref, port = cpu_baselines(lay, K, W, budget_s=args.cpu_budget)
        result["cpu_baseline"] = ref
        result["cpu_port"] = port
    if not args.no_extra:
        also = {}
        for name in ("fp32_m128", "large_m1", "large_m16", "large_m512", "large_m8192"):
            if name != args.workload:
                also[name] = _entry(qb, wl, torch, dev, name, K, W, peaks)
        sus, sflops, ncalls, _ = time_stack(qb, wl, torch, dev, 20, W)
        a = sflops / (sus * 1e-6) / 1e12
        also["gpt2_stack"] = {"us_per_forward": sus, "linears": ncalls, "M": 8192,
                              "roofline": {"bound": "tensor", "achieved": a, "peak": peaks["bf16_tflops"],
                                           "unit": "TFLOP/s", "frac": a / peaks["bf16_tflops"]}}
        try:
            cus, cflops, cn = time_converted_gpt2(qb, torch, dev, 20, W)
            a = cflops / (cus * 1e-6) / 1e12
            also["gpt2_converted"] = {
                "us_per_forward": cus, "linears": cn, "M": 8192, "bias": True,
                "weights": "transformers GPT-2-small (random init, seed 0) converted by convert_model (matrix)",
                "roofline": {"bound": "tensor", "achieved": a, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                             "frac": a / peaks["bf16_tflops"]}}
        except ImportError:  # transformers absent
            pass
        result["also"] = also
        # the metric's other halves, last so that they end the line
        for name in ("decode_m16", "prefill_m2048"):
            if name != args.workload:
                result[name] = _entry(qb, wl, torch, dev, name, K, W, peaks, with_clocks=True)
    print(json.dumps(result), flush=True)


def main_partitioned(qb, wl, torch, dev, dist, world, rank, K, W, M, metric, peaks, peak_src):
    """--gpus N > 1: the 5120 -> 27648 layer column-partitioned over the N
    ranks (out/4 rows per rank) at M tokens, the full output assembled on
    every rank inside the timed region (strong scaling: the layer and batch
    are fixed, N GPUs share them).  value = device us per call, max over
    ranks, of the path the module takes at this M (fused NVLink all-gather
    for M >= 64, else NCCL)."""
    with ClockSampler(dev.index) as clk:
        head = time_sharded(qb, wl, torch, dev, dist, world, rank, W, [(M, K)])[M]
    clocks = clk.summary()
    fused = M >= 64
    mc = fused and head.get("us_fused_mc") is not None
    us = (head["us_fused_mc"] if mc else head["us_fused"]) if fused else head["us_nccl"]
    lay = wl.sharded_27648(M)
    n = head["shard_rows"]
    flops = 2.0 * M * 4 * lay.K_g * 4 * n
    nbytes = 2 * (4 * n * lay.K_g + M * 4 * lay.K_g + M * 4 * n)
    roof = _roofline("tensor" if M > 16 else "hbm", nbytes, flops, us, peaks, peak_src)
    roof["basis"] = "one rank's shard FLOP (or bytes) / call time incl. the output all-gather"
    if fused:
        # the fused call's target: the slower of the shard's compute and its NVLink egress
        target = head["mc_target_us"] if mc else head["fused_target_us"]
        roof["target_us"] = target
        roof["frac_of_target"] = target / us
    # the same layer unpartitioned on this GPU (the N = 1 point of the sweep)
    one_ms, _, _ = time_device(qb, lay, torch, dev, K, W, dist)
    single_us = one_ms * 1e3 / K
    e2e_us, h2d, d2h = time_sharded_e2e(qb, wl, torch, dev, dist, world, M, min(K, 20), W)
    others = time_sharded(qb, wl, torch, dev, dist, world, rank, W,
                          [(m, 200 if m <= 16 else 20) for m in (1, 16, 512, 8192) if m != M])
    # independent decode replicas (one per GPU), max over ranks
    dlay = _layer(wl, "decode_m1")
    dms, _, _ = time_device(qb, dlay, torch, dev, K, W, dist)
    launches = head["launches_fused"] if fused else None
    return {
        "metric": metric, "value": us, "unit": "us/call", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": us / 1e3, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"qlinear_5120x27648_bf16_m{M}_column_partitioned", "M": M,
                   "in_features": 5120, "out_features": 27648, "shard_rows_per_gpu": n,
                   "parallelism": f"column{world} (out/4 quaternion rows) + "
                                  + (("fused NVLink multicast all-gather" if mc else "fused NVLink all-gather")
                                     if fused else "NCCL all-gather"),
                   "inputs": "seeded synthetic N(0,1) activations, N(0,1/in) weights (variance)",
                   "l2": "inputs larger than L2: rotating weight shard copies"},
        "roofline": roof,
        "clocks": clocks,
        "gpu_launches": K * (launches or 2),
        "e2e": {"value": e2e_us, "unit": "us/call", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "single_gpu_us_per_call": single_us,
        "decode_replicas_us_per_call": dms * 1e3 / K,
        "sharded_other_m": {f"m{m}": v for m, v in others.items()},
        "partitioned": head,
    }


if __name__ == "__main__":
    main()
