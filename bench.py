#!/usr/bin/env python
"""Benchmark of the W4A16 g128 dequant-GEMM (and its M sweep) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Metric: W4A16 g128 GEMM us/call and % of the HBM / tensor
roofline at M = 16 / 128 / 4096, 1-8 GPUs.  The headline workload is the
benchmark's compute-bound configuration, x fp16 [4096, 14336] . W [14336, 4096]
(K=14336, N=4096, group 128, asymmetric int4, scales U[0.002, 0.02], zeros
U{0..15}); the other M values are reported in ``sweep``.  A step is one call of
the op.  Inputs are synthetic and seeded, with the benchmark's distributions.

For N > 1 GPUs (torchrun, one rank per GPU) the weight is column-sharded:
total work is fixed ("strong" scaling) and the time is the max over ranks.
With ``--gather peer`` (the default) the GEMM epilogue stores every tile into
all ranks' outputs over NVLink (one kernel per rank and call); with
``--gather nccl`` the local output is all-gathered over NCCL and permuted.

Timing: W untimed warm-up calls, then exactly K calls captured in a CUDA graph
(every N; NCCL collectives are captured too), bracketed by barrier + synchronize, timed
with CUDA events on the launching stream.  Calls rotate over enough copies of
the weights (and activations) that the working set exceeds the 126 MB L2, so
every call streams from HBM.  SM clocks and throttle reasons are sampled with
NVML during the timed regions.

``e2e`` is the same call through the public module with host buffers: every
step copies x and the weights from pinned host memory and reads y back;
consecutive steps overlap over the full-duplex link (the next step's copies
run while this step computes and reads back).

``--impl reference`` times the reference module's op sequence (a torch-CPU
restatement of QUANT_REF.forward, oracle/reference_port.py) on the host cores
for the same workload; each step is a column sample of the call, scaled to a
whole call.  Under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

K_DIM, N_DIM, GROUP = 14336, 4096, 128
HEADLINE_M = 4096
SWEEP_M = (16, 128, 1024, 4096)
L2_BYTES = 126 * 2**20
NCU_TRAFFIC = {4096: 209_088_512}  # 186.118912 MB read + 22.969600 MB written
METRIC = "W4A16 g128 GEMM us/call & % HBM/tensor roofline at M=16/128/4096, 1-8 GPU"


def algorithmic_bytes(M, N, K, group):
    return K * N // 2 + 2 * (K // group) * N * 2 + M * K * 2 + M * N * 2


def flops(M, N, K):
    return 2 * M * N * K


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "tflops": float(d["bf16_tflops"]),
                "tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """Polls NVML (SM clock, throttle reasons) every ~5 ms while `active`."""

    REASONS = {
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index: int):
        self.samples = []
        self.reasons = set()
        self.active = False
        self.max_mhz = None
        self._stop = False
        self.nv = None
        try:
            import pynvml
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device_index)
            bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.nv = pynvml
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as e:  # NVML unavailable: report nothing rather than guess
            self.nv = None
            self.err = str(e)

    def sample(self):
        """One sample now (also called right after the timed work is enqueued,
        while the GPU runs it, so short timed regions get at least one)."""
        if self.nv is None:
            return
        try:
            mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
            r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            self.samples.append(mhz)
            for bit, name in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def _run(self):
        while not self._stop:
            if self.active:
                self.sample()
            time.sleep(0.005)

    def summary(self):
        self._stop = True
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------- inputs
def make_weights(seed: int, device, K=K_DIM, N=N_DIM, group=GROUP):
    g = torch.Generator(device=device).manual_seed(seed)
    nib = torch.randint(0, 16, (K, N), generator=g, device=device, dtype=torch.int32)
    packed = torch.zeros(K, N // 8, dtype=torch.int32, device=device)
    for i in range(8):
        packed |= nib[:, i::8] << (4 * i)
    scales = (torch.rand(K // group, N, generator=g, device=device) * 0.018 + 0.002).half()
    zeros = torch.randint(0, 16, (K // group, N), generator=g, device=device).half()
    return packed, scales, zeros


def make_x(M: int, seed: int, device, K=K_DIM):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(M, K, generator=g, device=device).half()


# ---------------------------------------------------------------------------- our arm
def barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_calls(fn, n_sets, steps, warmup, world, sampler, use_graph):
    """Per-call device time (ms) of `steps` calls rotating over `n_sets` input
    sets, max over ranks."""
    for i in range(max(warmup, 1)):
        fn(i % n_sets)
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if use_graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(steps):
                fn(i % n_sets)
        g.replay()  # untimed: the first replay uploads the graph
        barrier(world)
        sampler.active = True
        s.record()
        g.replay()
        e.record()
        sampler.sample()  # the replay is enqueued and running
        torch.cuda.synchronize()
        sampler.active = False
    else:
        barrier(world)
        sampler.active = True
        s.record()
        for i in range(steps):
            fn(i % n_sets)
        e.record()
        sampler.sample()
        torch.cuda.synchronize()
        sampler.active = False
    barrier(world)
    return max_over_ranks(s.elapsed_time(e) / steps, world)


def run_ours(args, world, rank, device, peaks):
    import kernelbench_harbor_b200 as pkg
    pkg.build()
    from kernelbench_harbor_b200 import ops, parallel
    from kernelbench_harbor_b200.modules import ModelNew

    sampler = ClockSampler(device.index)
    use_graph = True  # NCCL collectives are captured in the graph too
    n_local = N_DIM // world
    w_bytes = K_DIM * n_local // 2 + 2 * (K_DIM // GROUP) * n_local * 2
    sweep = {}
    model = None
    if world > 1:
        model = (parallel.PeerGatherW4A16(GROUP) if args.gather == "peer"
                 else parallel.ColumnShardedW4A16(GROUP))
    parity = {}
    for M in sorted(set(args.sweep) | {args.m}):
        set_bytes = w_bytes + M * K_DIM * 2
        n_sets = max(2, -(-2 * L2_BYTES // set_bytes))  # working set > 2x L2
        sets = []
        for i in range(n_sets):
            q, s_, z = make_weights(1000 + i, device)
            if world > 1:
                q, s_, z = parallel.shard_weights(q, s_, z, world, rank)
            sets.append((make_x(M, 2000 + i, device), q, s_, z))
        torch.cuda.synchronize()
        if world > 1:
            fn = lambda i: model(*sets[i])  # noqa: E731
        else:
            fn = lambda i: ops.w4a16_gemm(*sets[i], GROUP)  # noqa: E731
        ms = time_calls(fn, n_sets, args.steps, args.warmup, world, sampler, use_graph)
        us = ms * 1e3
        if world > 1:
            parity[M] = sharded_parity(model, sets[0], world)
            # the same shards through the plain single-GPU entry point (no
            # peer stores, no cross-rank ordering): the compute part of the
            # fused-gather time
            ms_local = time_calls(lambda i: ops.w4a16_gemm(*sets[i], GROUP), n_sets, args.steps, args.warmup,
                                  world, sampler, use_graph)
        ab = algorithmic_bytes(M, N_DIM, K_DIM, GROUP)
        fl = flops(M, N_DIM, K_DIM)
        t_hbm = ab / (peaks["hbm_gbs"] * 1e9 * world)
        t_ten = fl / (peaks["tflops"] * 1e12 * world)
        bound = "hbm" if t_hbm >= t_ten else "tensor"
        sweep[M] = {"us_per_call": round(us, 3), "GB_s": round(ab / (us * 1e-6) / 1e9, 1),
                    "TFLOP_s": round(fl / (us * 1e-6) / 1e12, 1), "bound": bound,
                    "roofline_frac": round((t_hbm if bound == "hbm" else t_ten) / (us * 1e-6), 4),
                    "l2": f"{n_sets} rotating input sets of {set_bytes / 2**20:.0f} MiB"}
        if world > 1:
            sweep[M]["shard_gemm_only_us"] = round(ms_local * 1e3, 3)
        if world == 1 and M <= 16:
            # the same calls with weight prefetch across the launch boundary
            # (programmatic dependent launch; weights are never written here)
            prev = ops.set_weight_prefetch(True)
            ms_p = time_calls(fn, n_sets, args.steps, args.warmup, world, sampler, use_graph)
            ops.set_weight_prefetch(prev)
            us_p = ms_p * 1e3
            sweep[f"{M}_weight_prefetch"] = {
                "us_per_call": round(us_p, 3), "GB_s": round(ab / (us_p * 1e-6) / 1e9, 1),
                "roofline_frac": round(t_hbm / (us_p * 1e-6), 4), "bound": "hbm",
                "note": "b200q_set_weight_prefetch(1): each call streams its first weight tiles while "
                        "the previous call finishes", "l2": sweep[M]["l2"]}
        del sets
        torch.cuda.empty_cache()

    e2e = None
    if not args.no_e2e:
        # the public module with HOST buffers: H2D of every forward input and
        # D2H of y inside the timed region, each step
        # (N > 1: each rank copies its 1/N of x's rows and its weight shard
        # from the host, x is all-gathered over NCCL, and each rank reads back
        # its 1/N of y's rows: the hosts together move x, W and y once)
        M = args.m
        q, s_, z = make_weights(1000, device)
        if world > 1:
            q, s_, z = parallel.shard_weights(q, s_, z, world, rank)
        x = make_x(M, 2000, device)
        rows = slice(rank * M // world, (rank + 1) * M // world)
        hx = x[rows].contiguous().cpu().pin_memory()
        hq, hs, hz = (t.cpu().pin_memory() for t in (q, s_, z))
        hy = torch.empty((rows.stop - rows.start, N_DIM), dtype=torch.float16).pin_memory()
        mod = model if world > 1 else ModelNew()
        x_full = torch.empty((M, K_DIM), dtype=torch.float16, device=device)
        # Consecutive steps overlap over the full-duplex PCIe link: step i+1's
        # host-to-device copies (copy stream, double-buffered device inputs)
        # run while step i computes and reads y back (its own stream).  All
        # compute stays on one stream, so the fused-gather module's shared
        # peer buffers are never used by two calls at once.
        comp = torch.cuda.current_stream(device)
        h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
        bufs = [[torch.empty_like(t, device=device) for t in (hx, hq, hs, hz)] for _ in range(2)]
        hys = [hy, torch.empty_like(hy).pin_memory()]
        loaded = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]
        computed = [torch.cuda.Event() for _ in range(2)]
        read = [torch.cuda.Event() for _ in range(2)]
        ybuf = [None, None]
        for k in range(2):  # every event starts recorded
            for ev in (consumed[k], read[k]):
                ev.record(comp)

        def load(i):
            k = i % 2
            with torch.cuda.stream(h2d):
                h2d.wait_event(consumed[k])  # the step two back finished reading slot k
                for d, h in zip(bufs[k], (hx, hq, hs, hz)):
                    d.copy_(h, non_blocking=True)
                loaded[k].record(h2d)

        def compute(i):
            k = i % 2
            comp.wait_event(loaded[k])
            comp.wait_event(read[k])  # the step two back has read its y out of ybuf[k]
            dx, dq, ds, dz = bufs[k]
            if world > 1:
                dist.all_gather_into_tensor(x_full, dx)
                dx = x_full
            ybuf[k] = mod(dx, dq, ds, dz)[rows].clone()
            consumed[k].record(comp)
            computed[k].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(computed[k])
                hys[k].copy_(ybuf[k], non_blocking=True)
                read[k].record(d2h)

        def run(n):
            load(0)
            for i in range(n):
                if i + 1 < n:
                    load(i + 1)
                compute(i)
            comp.wait_event(read[(n - 1) % 2])

        e_steps = max(3, min(args.steps, 20))
        run(max(args.warmup, 2))
        torch.cuda.synchronize()
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(comp)
        h2d.wait_event(s)
        run(e_steps)
        e.record(comp)
        torch.cuda.synchronize()
        e_ms = max_over_ranks(s.elapsed_time(e) / e_steps, world)
        e2e = {"value": round(e_ms * 1e3, 3), "unit": "us/call",
               "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in (hx, hq, hs, hz)),
               "d2h_bytes_per_step": hy.numel() * hy.element_size(), "steps": e_steps,
               "path": ("ModelNew.forward" if world == 1 else
                        f"x row shards H2D + NCCL all-gather, {type(model).__name__}.forward"),
               "overlap": "step i+1's H2D copies overlap step i's compute and D2H (copy streams, "
                          "double-buffered inputs); compute on one stream"}
    return sweep, e2e, sampler.summary(), parity


def sharded_parity(model, inputs, world) -> bool:
    """One sharded call against this rank's shard computed by the plain
    single-GPU entry point (same kernel, same shard shape, hence the same
    split-K order), all shards gathered over NCCL: bit-identical on every rank."""
    from kernelbench_harbor_b200 import ops, parallel
    x, q, s_, z = inputs
    y = model(x, q, s_, z).clone()
    ref = parallel.gather_columns(ops.w4a16_gemm(x, q, s_, z, GROUP), world)
    ok = torch.tensor([1 if torch.equal(y, ref) else 0], device=x.device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    return bool(ok.item())


def run_siblings(device, steps, warmup, sampler):
    """The sibling configurations of the benchmark, each timed like the sweep
    (CUDA graph of `steps` calls over rotating input sets, CUDA events):
    W8A8 SmoothQuant M=16/512, MXFP8 M=128/4096, quantised top-2 MoE T=512."""
    from kernelbench_harbor_b200 import ops
    from kernelbench_harbor_b200.modules import QuantizedMoE
    from kernelbench_harbor_b200.mx import quantize_mxfp8
    from kernelbench_harbor_b200.quant import smoothquant_inputs
    peaks = load_peaks()
    out = {}
    K, N = K_DIM, N_DIM
    for M in (16, 512):
        sets = [[t.to(device) for t in smoothquant_inputs(M, K, N, seed=100 + i)[:4]] for i in range(4)]
        us = time_calls(lambda i: ops.w8a8_gemm(*sets[i]), 4, steps, warmup, 1, sampler, True) * 1e3
        b = M * K + K * N + 2 * M + 2 * N + 2 * M * N
        tops = 2 * M * N * K / us / 1e6
        out[f"w8a8_m{M}"] = {"us_per_call": round(us, 3), "GB_s": round(b / us / 1e3, 1),
                             "TOPS": round(tops, 1),
                             "hbm_frac": round(b / us / 1e3 / peaks["hbm_gbs"], 4),
                             "tensor_frac": round(tops / (2 * peaks["tflops"]), 4),
                             "tensor_peak": "2 x measured bf16 burst (dense int8 rate is twice bf16)"}
        del sets
    for M in (128, 4096):
        nset = 2 if M > 1024 else 4
        sets = []
        for i in range(nset):
            g = torch.Generator().manual_seed(200 + i)
            a = quantize_mxfp8(torch.randn(M, K, generator=g).half())
            bq = quantize_mxfp8((torch.randn(N, K, generator=g) * 0.02).half())
            sets.append([a[0].to(device), a[1].to(device), bq[0].to(device), bq[1].to(device)])
        us = time_calls(lambda i: ops.mxfp8_gemm(*sets[i]), nset, steps, warmup, 1, sampler, True) * 1e3
        b = M * K + N * K + (M + N) * (K // 32) + 2 * M * N
        tf = 2 * M * N * K / us / 1e6
        out[f"mxfp8_m{M}"] = {"us_per_call": round(us, 3), "GB_s": round(b / us / 1e3, 1),
                              "TFLOP_s": round(tf, 1),
                              "hbm_frac": round(b / us / 1e3 / peaks["hbm_gbs"], 4),
                              "tensor_frac": round(tf / (2 * peaks["tflops"]), 4),
                              "tensor_peak": "2 x measured bf16 burst (dense fp8 rate is twice bf16)"}
        del sets
    # MoE: Mixtral shape, one input set (its 8 experts x 3 W4A16 weights = 749 MB > L2)
    T, D, H, E = 512, 4096, 14336, 8
    g = torch.Generator(device=device).manual_seed(300)
    x = torch.randn(T, D, generator=g, device=device).half()
    logits = (x.float() @ (torch.randn(E, D, generator=g, device=device) * 0.02).t()).half()
    ws = []
    for (kk, nn) in ((D, H), (D, H), (H, D)):
        q, s_, z = [], [], []
        for e in range(E):
            qe, se, ze = make_weights(400 + 10 * e + len(ws), device, K=kk, N=nn)
            q.append(qe), s_.append(se), z.append(ze)
        ws += [torch.stack(q), torch.stack(s_), torch.stack(z)]
    moe = QuantizedMoE()
    msteps = max(3, min(steps, 20))
    us = time_calls(lambda i: moe(x, logits, *ws), 1, msteps, warmup, 1, sampler, True) * 1e3
    fl = T * 2 * 3 * 2 * D * H
    wb = E * 3 * (D * H // 2 + 2 * (D // GROUP) * H * 2)
    out["moe_top2_t512"] = {"us_per_call": round(us, 1), "TFLOP_s": round(fl / us / 1e6, 1),
                            "weight_GB_s": round(wb / us / 1e3, 1), "steps": msteps,
                            "timing": "CUDA graph: route, gather, fused gate/up/SiLU grouped GEMM, "
                                      "down grouped GEMM, combine (no host synchronisation)"}
    del ws
    torch.cuda.empty_cache()
    out.update(run_next_rows(device, steps, warmup, sampler))
    return out


def run_next_rows(device, steps, warmup, sampler):
    """The reference modules next to the W4A16 path, at one of their own
    configurations each (generate_tasks.py:351-355, 381-385, 427-431):
    FUSED_QMOE (mixtral, T=256, int8 weights packed on the GPU every call),
    FUSED_SILU fp8 (mixtral H=14336, T=512) and multi-LoRA (llama3-8B r16, T=64)."""
    from kernelbench_harbor_b200.modules import FusedQMoE, FusedSiluFp8, MultiLoRAW4
    out = {}
    g = torch.Generator(device=device).manual_seed(500)
    n = max(3, min(steps, 20))
    T, D, E, N = 256, 4096, 8, 14336
    x = torch.randn(T, D, generator=g, device=device).half()
    qw = torch.randint(-8, 8, (E, D, N), generator=g, device=device, dtype=torch.int8)
    sc = (torch.randn(E, D // 128, N, generator=g, device=device) * 0.01).half()
    lg = torch.randn(T, E, generator=g, device=device).half()
    mod = FusedQMoE()
    us = time_calls(lambda i: mod(x, qw, sc, lg), 1, n, warmup, 1, sampler, True) * 1e3
    wb = E * D * N + E * (D // 128) * N * 2
    out["fused_qmoe_mixtral_t256"] = {"us_per_call": round(us, 1), "weight_GB_s": round(wb / us / 1e3, 1),
                                      "note": "int8 weights read and packed on the GPU inside every call"}
    del qw
    T, H = 512, 14336
    y = torch.randn(T, 2 * H, generator=g, device=device).half()
    fs = FusedSiluFp8()
    us = time_calls(lambda i: fs(y), 1, n, warmup, 1, sampler, True) * 1e3
    b = T * 2 * H * 2 + T * H * 4
    out["silu_fp8_mixtral_t512"] = {"us_per_call": round(us, 2), "GB_s": round(b / us / 1e3, 1),
                                    "hbm_frac": round(b / us / 1e3 / load_peaks()["hbm_gbs"], 3)}
    T, D, N, r, L = 64, 4096, 4096, 16, 8
    x = torch.randn(T, D, generator=g, device=device).half()
    qw = torch.randint(-8, 8, (D, N), generator=g, device=device, dtype=torch.int8)
    sc = (torch.randn(D // 128, N, generator=g, device=device) * 0.01).half()
    A = (torch.randn(L, D, r, generator=g, device=device) * 0.02).half()
    B = (torch.randn(L, r, N, generator=g, device=device) * 0.02).half()
    ids = torch.randint(0, L, (T,), generator=g, device=device)
    lm = MultiLoRAW4()
    us = time_calls(lambda i: lm(x, qw, sc, A, B, ids), 1, n, warmup, 1, sampler, True) * 1e3
    out["multi_lora_llama3_8b_r16_t64"] = {"us_per_call": round(us, 1),
                                           "note": "int8 base weight packed on the GPU inside every call"}
    return out


def run_mxfp8_sharded(world, rank, device, steps, warmup, sampler):
    """MXFP8 M=4096 (K=14336, N=4096) with B column-sharded over the ranks and
    the all-gather fused into the GEMM epilogue (PeerGatherMXFP8); CUDA graph,
    CUDA events, max over ranks.  Parity: one call against the per-shard plain
    GEMMs gathered over NCCL, bit for bit."""
    from kernelbench_harbor_b200 import ops, parallel
    from kernelbench_harbor_b200.mx import quantize_mxfp8
    M, K, N = 4096, K_DIM, N_DIM
    n = N // world
    g = torch.Generator(device=device).manual_seed(200)
    sets = []
    for i in range(2):
        a = quantize_mxfp8(torch.randn(M, K, generator=g, device=device).half())
        b = quantize_mxfp8((torch.randn(N, K, generator=g, device=device) * 0.02).half())
        sets.append((a[0], a[1], b[0][rank * n:(rank + 1) * n].contiguous(),
                     b[1][rank * n:(rank + 1) * n].contiguous()))
    mod = parallel.PeerGatherMXFP8()
    us = time_calls(lambda i: mod(*sets[i]), 2, steps, warmup, world, sampler, True) * 1e3
    y = mod(*sets[0]).clone()
    ref = parallel.gather_columns(ops.mxfp8_gemm(*sets[0]), world)
    ok = torch.tensor([1 if torch.equal(y, ref) else 0], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    tf = 2 * M * N * K / us / 1e6
    return {"mxfp8_m4096_sharded": {"us_per_call": round(us, 2), "TFLOP_s": round(tf, 1),
                                    "tensor_frac": round(tf / (2 * load_peaks()["tflops"] * world), 4),
                                    "parity_vs_per_shard": bool(ok.item()),
                                    "parallelism": f"B N-sharded x{world}, gather fused in the epilogue"}}


def run_siblings_multi(world, rank, device, steps, warmup, sampler):
    """Expert-parallel MoE (Mixtral shape, T=512 tokens split evenly over the
    ranks, E/P experts per rank): route locally, NCCL all-to-all dispatch,
    grouped W4A16 experts, all-to-all return, gated combine.  The exchange
    uses fixed-capacity all-to-alls, so a call has no host synchronisation and
    is timed as a CUDA graph; CUDA events, max over ranks."""
    from kernelbench_harbor_b200 import parallel
    T, D, H, E = 512, 4096, 14336, 8
    tl, epr = T // world, E // world
    g = torch.Generator(device=device).manual_seed(300)
    x = torch.randn(T, D, generator=g, device=device).half()
    logits = (x.float() @ (torch.randn(E, D, generator=g, device=device) * 0.02).t()).half()
    x_all, logits_all = x, logits
    x, logits = x[rank * tl:(rank + 1) * tl].contiguous(), logits[rank * tl:(rank + 1) * tl].contiguous()
    ws = []
    for j, (kk, nn) in enumerate(((D, H), (D, H), (H, D))):
        q, s_, z = [], [], []
        for e in range(rank * epr, (rank + 1) * epr):
            qe, se, ze = make_weights(400 + 10 * e + 3 * j, device, K=kk, N=nn)
            q.append(qe), s_.append(se), z.append(ze)
        ws += [torch.stack(q), torch.stack(s_), torch.stack(z)]
    mod = parallel.ExpertParallelMoE(E)
    msteps = max(3, min(steps, 20))
    us = time_calls(lambda i: mod(x, logits, ws), 1, msteps, warmup, world, sampler, True) * 1e3
    fl = T * 2 * 3 * 2 * D * H
    # parity: this rank's tokens against the single-GPU module over all experts
    from kernelbench_harbor_b200.modules import QuantizedMoE
    y = mod(x, logits, ws).clone()
    del ws
    full = []
    for j, (kk, nn) in enumerate(((D, H), (D, H), (H, D))):
        q, s_, z = [], [], []
        for e in range(E):
            qe, se, ze = make_weights(400 + 10 * e + 3 * j, device, K=kk, N=nn)
            q.append(qe), s_.append(se), z.append(ze)
        full += [torch.stack(q), torch.stack(s_), torch.stack(z)]
    ref = QuantizedMoE()(x_all, logits_all, *full)[rank * tl:(rank + 1) * tl]
    # a rank holding few expert tiles splits K in the down projection where
    # the single-GPU module does not, so the fp32 sums may differ in order:
    # the check is the benchmark's tolerance, with the bit-identity reported
    # (outputs reach |y| ~ 800 at this shape, where fp16 steps by 0.5: the
    # absolute part of the tolerance scales with the output, as in the MoE tests)
    diff = (y.float() - ref.float()).abs().max()
    top = float(ref.float().abs().max())
    close = torch.allclose(y.float(), ref.float(), rtol=1e-2, atol=1e-2 * max(top, 1.0))
    flags = torch.tensor([1 if close else 0, 1 if torch.equal(y, ref) else 0], device=device)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    dist.all_reduce(diff, op=dist.ReduceOp.MAX)
    ok = flags[0]
    del full
    torch.cuda.empty_cache()
    return {"moe_ep_top2_t512": {"us_per_call": round(us, 1), "TFLOP_s": round(fl / us / 1e6, 1),
                                 "parity_vs_single_gpu": bool(ok.item()),
                                 "parity_check": "allclose(rtol=1e-2, atol=1e-2 x max|y|) against the "
                                                 "single-GPU module",
                                 "bit_identical": bool(flags[1].item()), "max_abs_diff": round(float(diff), 6),
                                 "experts_per_gpu": epr, "tokens_per_gpu": tl, "steps": msteps,
                                 "timing": "CUDA graph (fixed-capacity all-to-alls, no host "
                                           "synchronisation), CUDA events, max over ranks"}}


# ---------------------------------------------------------------------------- CPU legs
def cpu_reference_time(M, steps, warmup, budget_s=0.25):
    """Median seconds of one full call of the reference op sequence on the host
    cores, measured on a column sample (scaled by N / N_sample)."""
    from oracle.reference_port import w4a16_forward
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    q, s_, z = make_weights(1000, torch.device("cpu"))
    x = make_x(M, 2000, torch.device("cpu"))
    ns = N_DIM
    while True:  # shrink the column sample until one step fits the budget
        t0 = time.perf_counter()
        w4a16_forward(x, q[:, :ns // 8], s_[:, :ns], z[:, :ns], GROUP)
        if time.perf_counter() - t0 <= budget_s or ns <= 256:
            break
        ns = max(256, ns // 2)
    qs, ss, zs = q[:, :ns // 8].contiguous(), s_[:, :ns].contiguous(), z[:, :ns].contiguous()
    for _ in range(warmup):
        w4a16_forward(x, qs, ss, zs, GROUP)
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        w4a16_forward(x, qs, ss, zs, GROUP)
        ts.append(time.perf_counter() - t0)
    per_call = statistics.median(ts) * (N_DIM / ns)
    sample = (f"reference op sequence (torch CPU, fp16) on x[{M},{K_DIM}] x W[:, :{ns}] "
              f"({ns} of {N_DIM} columns), median of {steps} steps, scaled by {N_DIM // ns}")
    return per_call, cores, sample


def profile_case(args) -> int:
    """A few untimed calls of one seeded case on one GPU, for ncu:

        ncu --set full --clock-control none -k regex:w4a16 -s 1 -c 1 \\
            python bench.py --profile w4a16=4096 --calls 2
    """
    import kernelbench_harbor_b200 as pkg
    pkg.build()
    from kernelbench_harbor_b200 import ops
    kind, size = args.profile.split("=")
    size = int(size)
    device = torch.device("cuda", 0)
    if kind == "w4a16":
        q, s_, z = make_weights(1, device)
        x = make_x(size, 2, device)
        ops.set_weight_prefetch(args.prefetch)
        call = lambda: ops.w4a16_gemm(x, q, s_, z, GROUP)  # noqa: E731
    elif kind == "moe":
        from kernelbench_harbor_b200.modules import QuantizedMoE
        T, D, H, E = size, 4096, 14336, 8
        g = torch.Generator(device=device).manual_seed(3)
        x = torch.randn(T, D, generator=g, device=device).half()
        logits = (x.float() @ (torch.randn(E, D, generator=g, device=device) * 0.02).t()).half()
        ws = []
        for j, (kk, nn) in enumerate(((D, H), (D, H), (H, D))):
            parts = [make_weights(10 * e + j, device, K=kk, N=nn) for e in range(E)]
            ws += [torch.stack([p[i] for p in parts]) for i in range(3)]
        mod = QuantizedMoE()
        call = lambda: mod(x, logits, *ws)  # noqa: E731
    elif kind == "ep":
        # one rank of an expert-parallel MoE (a one-process NCCL group), SIZE
        # tokens, 4 local experts of the Mixtral shape: the exchange
        # bookkeeping and the grouped GEMMs as one rank runs them
        from kernelbench_harbor_b200 import parallel
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29541")
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=device)
        T, D, H, E = size, 4096, 14336, 4
        g = torch.Generator(device=device).manual_seed(3)
        x = torch.randn(T, D, generator=g, device=device).half()
        logits = (x.float() @ (torch.randn(E, D, generator=g, device=device) * 0.02).t()).half()
        ws = []
        for j, (kk, nn) in enumerate(((D, H), (D, H), (H, D))):
            parts = [make_weights(10 * e + j, device, K=kk, N=nn) for e in range(E)]
            ws += [torch.stack([p[i] for p in parts]) for i in range(3)]
        mod = parallel.ExpertParallelMoE(E)
        call = lambda: mod(x, logits, ws)  # noqa: E731
    elif kind == "w8a8":
        from kernelbench_harbor_b200.quant import smoothquant_inputs
        t = [v.to(device) for v in smoothquant_inputs(size, K_DIM, N_DIM, seed=1)[:4]]
        call = lambda: ops.w8a8_gemm(*t)  # noqa: E731
    elif kind == "mxfp8":
        from kernelbench_harbor_b200.mx import quantize_mxfp8
        g = torch.Generator().manual_seed(1)
        a = quantize_mxfp8(torch.randn(size, K_DIM, generator=g).half())
        b = quantize_mxfp8((torch.randn(N_DIM, K_DIM, generator=g) * 0.02).half())
        t = [a[0].to(device), a[1].to(device), b[0].to(device), b[1].to(device)]
        call = lambda: ops.mxfp8_gemm(*t)  # noqa: E731
    else:
        raise SystemExit(f"unknown profile kind {kind}")
    for _ in range(args.calls):
        call()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.destroy_process_group()
    print("ok")
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--m", type=int, default=HEADLINE_M)
    ap.add_argument("--sweep", type=lambda s: [int(v) for v in s.split(",") if v], default=list(SWEEP_M))
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-siblings", action="store_true")
    ap.add_argument("--profile", default=None,
                    help="KIND=SIZE: run `--calls` untimed calls of one case for a profiler and exit; "
                         "KIND is w4a16 (SIZE = M), moe (tokens), ep (tokens of one "
                         "expert-parallel rank), w8a8 (M), mxfp8 (M)")
    ap.add_argument("--calls", type=int, default=2)
    ap.add_argument("--prefetch", action="store_true", help="with --profile: weight prefetch on")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile:
        return profile_case(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    workload = f"W4A16 g{GROUP} M={args.m} K={K_DIM} N={N_DIM} fp16"

    if args.impl == "reference":
        if rank != 0:
            return 0
        per_call, cores, sample = cpu_reference_time(args.m, args.steps, args.warmup)
        us = per_call * 1e6
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": "us/call",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded, benchmark distributions)",
            "config": {"workload": workload, "device": "host CPU"},
            "cpu_baseline": {"value": round(us, 1), "unit": "us/call", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(us, 1), "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return 0

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    device = torch.device("cuda", torch.cuda.current_device())
    peaks = load_peaks()
    sweep, e2e, clocks, parity = run_ours(args, world, rank, device, peaks)
    siblings = None
    if world == 1 and not args.no_siblings:
        siblings = run_siblings(device, args.steps, args.warmup, ClockSampler(device.index))
    elif world > 1 and not args.no_siblings:
        siblings = run_siblings_multi(world, rank, device, args.steps, args.warmup, ClockSampler(device.index))
        siblings.update(run_mxfp8_sharded(world, rank, device, args.steps, args.warmup,
                                          ClockSampler(device.index)))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        per_call, cores, sample = cpu_reference_time(args.m, 3, 1)
        cpu = {"value": round(per_call * 1e6, 1), "unit": "us/call", "cores": cores, "kind": "port",
               "sample": sample}

    if rank == 0:
        M = args.m
        head = sweep[M]
        us = head["us_per_call"]
        # whole-job achieved rate against the whole job's peak (world x one GPU)
        if head["bound"] == "hbm":
            ach = algorithmic_bytes(M, N_DIM, K_DIM, GROUP) / (us * 1e-6) / 1e9
            pk = peaks["hbm_gbs"] * world
            roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": pk, "unit": "GB/s"}
        else:
            ach = flops(M, N_DIM, K_DIM) / (us * 1e-6) / 1e12
            pk = peaks["tflops"] * world
            roof = {"bound": "tensor", "achieved": round(ach, 1), "peak": pk, "unit": "TFLOP/s"}
        roof["frac"] = round(ach / pk, 4)
        if head["bound"] == "tensor":
            # the timed region is a loop of `steps` calls: long regions run
            # under the 1 kW power cap, so the sustained GEMM peak applies too
            roof["frac_of_sustained"] = round(ach / (peaks["tflops_sustained"] * world), 4)
        roof["peak_source"] = ("measured (MEASURED_PEAKS.json, burst)" if peaks["source"] == "measured"
                               else "fallback") + (f" x {world} GPUs" if world > 1 else "")
        # DRAM bytes (read + write) of one launch of the headline kernel, from
        # one ncu capture of `bench.py --profile w4a16=4096`; None for
        # workloads not captured
        roof["traffic"] = NCU_TRAFFIC.get(M)
        line = {"metric": METRIC, "value": us, "unit": "us/call", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(us / 1e3, 4), "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
                "data": "synthetic (seeded, benchmark distributions)",
                "config": {"workload": workload,
                           "parallelism": (f"N-sharded x{world} + "
                                           + ("all-gather fused in the GEMM epilogue (NVLink peer stores)"
                                              if args.gather == "peer" else "NCCL all-gather")
                                           if world > 1 else "single GPU"),
                           "l2": head["l2"]},
                "roofline": roof, "sweep": {str(k): v for k, v in sweep.items()}, "siblings": siblings,
                "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks,
                **({"parity": {"w4a16_gather": {str(k): v for k, v in parity.items()},
                               "ep_moe": (siblings or {}).get("moe_ep_top2_t512", {}).get(
                                   "parity_vs_single_gpu"),
                               "mxfp8_gather": (siblings or {}).get("mxfp8_m4096_sharded", {}).get(
                                   "parity_vs_per_shard")}} if world > 1 else {}),
                # our kernels per step: the GEMM (with the gather fused into it for --gather peer)
                "gpu_launches": args.steps}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
