#!/usr/bin/env python
"""bench.py — the headline measurement: one DiffusionGemma W4A16 MoE layer on a 256-token canvas
(configs[1]: fused RMSNorm -> router with the Zipf bias -> 128-expert top-8 MoE) in microseconds
and HBM GB/s, plus the configs[2] sampler step in microseconds.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line on rank 0.  `value` is microseconds per canvas-layer for the whole job (lower
is better); for N > 1 the 128 experts are sharded over the ranks (128/N each, device-initiated
exchange over NVLink) and every rank brings its own canvas, so value = max-over-ranks time /
(N * K).  Inputs are synthetic (workloads.py) with the BASELINE
shapes and distributions; four distinct weight sets (4 x 416 MB) rotate between steps so every
step streams its weights from HBM, not L2.

--impl reference times the reference algorithm's CPU implementation (the oracle restatement of the
reference's torch path) on the host cores, rank 0 only, on a bounded sample of the same workload.
"""
import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

REPO = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "knivesysl-diffusion-xe_b200" / "kernels"))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

METRIC = json.loads((REPO / "BASELINE.json").read_text())["metric"]
T, H, I, E, TOPK = 256, 2816, 704, 128, 8
V_SAMPLER = 262144
NSETS = 4
# The dominant kernel per GEMM engine, and its DRAM bytes per launch (dram__bytes_read.sum +
# dram__bytes_write.sum) from one ncu capture of the configs[1] layer, summarised under profiles/;
# None where no capture of the current kernel exists.
GEMM1_KERNEL = {"tc": "tcp_gemm_kernel<1,0> (gate_up + GELU)",
                "ws": "hw_gemm_kernel<1,0,4> (gate_up + GELU)",
                "mma": "gateup_gelu_kernel"}
GEMM1_NCU_TRAFFIC = {"tc": None, "ws": 302.726912e6 + 4.080384e6}


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Dense f16/bf16 tensor peak (TFLOP/s) for a kernel timed inside a multi-millisecond step:
    the sustained cuBLAS figure of MEASURED_PEAKS.json, else the recipe's fallback."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured sustained"
    return 1400.0, "fallback sustained"


# --------------------------------------------------------------------------------- clocks
class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        rows = [ln.split(",") for ln in open(self.f.name).read().splitlines() if ln.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------------- workloads
def build_layer(dev):
    import workloads
    sets = []
    for i in range(NSETS):
        sets.append(workloads.moe_weights(E, H, I, seed=100 + i, device=dev))
    inp = workloads.moe_inputs(T, H, E, seed=0, device=dev)
    return sets, inp


def layer_step(W, inp, xn, xp):
    """configs[1] step: fused RMSNorm (also writes the MoE K-interleave copy) -> router -> MoE."""
    import fused_moe_w4_v2
    import moe_router
    y_norm, ids, w, _ = moe_router.rmsnorm_route_topk(inp["hidden"], inp["norm_w"], 1e-6,
                                                      inp["router_w"], TOPK, bias=inp["bias"],
                                                      xperm=xp, want_logits=False)
    return fused_moe_w4_v2.moe_forward(y_norm, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"],
                                       W["dn_s"], W["dn_z"], ids, w, hidden_perm=xp), ids


LAUNCHES_PER_LAYER = 5  # RMSNorm + router (one clustered kernel), align, gate_up, down, combine


def time_layer(dev, steps, warmup, dist):
    import _knx
    sets, inp = build_layer(dev)
    xp = torch.empty(T, H, dtype=torch.float16, device=dev)
    for i in range(warmup):
        layer_step(sets[i % NSETS], inp, None, xp)
    torch.cuda.synchronize(dev)
    _, ids = layer_step(sets[0], inp, None, xp)
    counts = torch.bincount(ids.flatten().long(), minlength=E).cpu()
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    clk = Clocks(dev.index)
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(steps):
        layer_step(sets[i % NSETS], inp, None, xp)
    ev1.record()
    torch.cuda.synchronize(dev)
    clocks = clk.stop()
    ms = ev0.elapsed_time(ev1)
    # stage breakdown in a second pass: its event records between the stages would stop the
    # kernels from launching ahead of their predecessors (programmatic dependent launch)
    _knx.prof_start(steps)
    for i in range(steps):
        layer_step(sets[i % NSETS], inp, None, xp)
    torch.cuda.synchronize(dev)
    stages, ncalls = _knx.prof_stop()
    if dist:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    return ms, {k: v / max(ncalls, 1) for k, v in stages.items()}, counts, clocks


def pipelined_e2e(dev, step_fn, host_src, steps, warmup, sync=None):
    """End to end as a serving loop runs it: every step copies its input host->device from
    pinned memory, runs step_fn(i, dev_input) -> output, and copies the output device->host.
    The copies run on a second stream with two buffers each way, so step i+1's upload and step
    i's download overlap the neighbouring steps' compute.  The timed region covers every copy of
    every step.  -> (ms, h2d bytes per step, d2h bytes per step)."""
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    host_in = [host_src.clone().pin_memory() for _ in range(2)]
    dev_in = [torch.empty(host_src.shape, dtype=host_src.dtype, device=dev) for _ in range(2)]
    host_out = [None, None]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    out_bytes = [0]

    def upload(i):
        b = i % 2
        with torch.cuda.stream(copy):
            copy.wait_event(in_free[b])  # the step that read this buffer two steps ago is done
            dev_in[b].copy_(host_in[b], non_blocking=True)
            in_ready[b].record(copy)

    def run(i):
        b = i % 2
        comp.wait_event(in_ready[b])
        y = step_fn(i, dev_in[b])
        in_free[b].record(comp)
        out_ready[b].record(comp)
        if host_out[b] is None:
            host_out[b] = torch.empty(y.shape, dtype=y.dtype).pin_memory()
        out_bytes[0] = y.numel() * y.element_size()
        with torch.cuda.stream(copy):
            copy.wait_event(out_ready[b])
            y.record_stream(copy)
            host_out[b].copy_(y, non_blocking=True)

    def loop(i0, n):
        upload(i0)
        for i in range(i0, i0 + n):
            if i + 1 < i0 + n:
                upload(i + 1)
            run(i)
        comp.wait_stream(copy)

    loop(0, warmup)
    torch.cuda.synchronize(dev)
    if sync is not None:
        sync()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(comp)
    loop(warmup, steps)
    ev1.record(comp)
    torch.cuda.synchronize(dev)
    return ev0.elapsed_time(ev1), host_src.numel() * host_src.element_size(), out_bytes[0]


def time_layer_e2e(dev, steps, warmup):
    """Through the public API with host buffers: H2D of the canvas hidden states from pinned
    memory, the layer, D2H of the layer output, every step (copies overlapped on a second
    stream, see pipelined_e2e)."""
    sets, inp = build_layer(dev)
    xp = torch.empty(T, H, dtype=torch.float16, device=dev)

    def step(i, x):
        y, _ = layer_step(sets[i % NSETS], dict(inp, hidden=x), None, xp)
        return y
    return pipelined_e2e(dev, step, inp["hidden"].cpu(), steps, warmup)


def balanced_owners(Tr, seeds, world, tpe, dev):
    """Expert labels that balance the ranks' grouped-GEMM work (ep_moe.balanced_relabel) for
    the job's routing: every rank routes every rank's synthetic tokens (the same counts on all
    ranks, no communication).  Tasks of the engine the layer will pick (32 tokens for ws, 128
    for tc).  -> (relabel, order)."""
    import ep_moe
    import moe_router
    import workloads
    counts = torch.zeros(E, dtype=torch.int64)
    for sd in seeds:
        inp = workloads.moe_inputs(Tr, H, E, seed=sd, device=dev)
        xp = torch.empty(Tr, H, dtype=torch.float16, device=dev)
        _, ids, _, _ = moe_router.rmsnorm_route_topk(inp["hidden"], inp["norm_w"], 1e-6,
                                                     inp["router_w"], TOPK, bias=inp["bias"],
                                                     xperm=xp, want_logits=False)
        counts += torch.bincount(ids.flatten().long(), minlength=E).cpu()
    return ep_moe.balanced_relabel(counts.tolist(), world, 32 if tpe <= 36 else 128)


class EpLayer:
    """N > 1: the same configs[1] layer with the 128 experts sharded over the ranks (expert
    parallelism; dispatch and return by device-initiated stores over NVLink; owners balanced by
    the job's routing); each rank runs its own 256-token canvas."""

    def __init__(self, dev, rank, world):
        import ep_moe
        import workloads
        self.tpe = T * TOPK * world // E  # job-wide pairs per expert (engine choice)
        relabel, order = balanced_owners(T, range(world), world, self.tpe, dev)
        self.layers = []
        for i in range(NSETS):
            Wf = workloads.moe_weights(E, H, I, seed=100 + i, device=dev)
            local = ep_moe.shard_experts(Wf["gu_q"], Wf["gu_s"], Wf["gu_z"], Wf["dn_q"],
                                         Wf["dn_s"], Wf["dn_z"], rank, world, interleaved=True,
                                         order=order)
            del Wf
            # the exchange runs on the device over NVLink (no host sync per layer)
            self.layers.append(ep_moe.P2PExpertParallelMoE(*local, E_total=E, int_zeros=False,
                                                           max_tokens=T, topk=TOPK,
                                                           relabel=relabel))
        torch.cuda.empty_cache()
        self.inp = workloads.moe_inputs(T, H, E, seed=rank, device=dev)  # this rank's canvas
        self.xp = torch.empty(T, H, dtype=torch.float16, device=dev)

    def step(self, i, hidden=None):
        import moe_router
        inp = self.inp
        x = inp["hidden"] if hidden is None else hidden
        _, ids, w, _ = moe_router.rmsnorm_route_topk(x, inp["norm_w"], 1e-6, inp["router_w"], TOPK,
                                                     bias=inp["bias"], xperm=self.xp,
                                                     want_logits=False)
        return self.layers[i % NSETS](self.xp, ids, w, out_dtype=torch.float16,
                                      tokens_per_expert=self.tpe), ids


EP_LAUNCHES_PER_LAYER = 9  # RMSNorm + router, align, counts exchange + plan, dispatch + barrier,
                           # task list, gate_up, down, return + barrier, combine (NVLink exchange)


def time_layer_ep(dev, steps, warmup, rank, world):
    ep = EpLayer(dev, rank, world)
    for i in range(warmup):
        ep.step(i)
    torch.cuda.synchronize(dev)
    _, ids = ep.step(0)
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    torch.distributed.all_reduce(counts)
    counts = counts.cpu()
    torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    clk = Clocks(dev.index)
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(steps):
        ep.step(i)
    ev1.record()
    torch.cuda.synchronize(dev)
    torch.distributed.barrier()
    clocks = clk.stop()
    t = torch.tensor([ev0.elapsed_time(ev1)], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    # end to end: the canvas from pinned host memory, the layer output back, every step
    def step(i, x):
        y, _ = ep.step(i, x)
        return y
    e2e_ms, h2d, d2h = pipelined_e2e(dev, step, ep.inp["hidden"].cpu(), steps, warmup,
                                     sync=torch.distributed.barrier)
    t = torch.tensor([e2e_ms], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    e2e_ms = float(t.item())
    stages = ep_stage_times(ep, dev, steps)
    return ms, counts, clocks, e2e_ms, h2d, d2h, stages


def ep_stage_times(ep, dev, steps):
    """A second pass of `steps` layers with CUDA events between the stages of the NVLink layer
    (the events stop the kernels from overlapping, so the stages add up to more than a step of
    the timed pass): per stage the mean device time in us, max over ranks.  The barrier stages
    hold the wait for the slowest rank."""
    for layer in ep.layers:
        layer.stage_events = []
    torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    for i in range(steps):
        ep.step(i)
    torch.cuda.synchronize(dev)
    sums = {}
    for layer in ep.layers:
        marks, layer.stage_events = layer.stage_events, None
        for (_, a), (name, b) in zip(marks, marks[1:]):
            if name != "start":
                sums[name] = sums.get(name, 0.0) + a.elapsed_time(b)
    names = sorted(sums)
    t = torch.tensor([sums[n] for n in names], device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return {n: float(v) * 1000.0 / steps for n, v in zip(names, t.tolist())}


def time_stack(dev, steps=48):
    """one denoising-step forward of a 60-block stack (30 encoder + 30 decoder) of
    RMSNorm -> W4A16 MoE -> residual on a 256-token canvas, then the configs[2] sampler step;
    decoder block b reuses encoder block b's expert weights (the checkpoint's aliasing,
    load_w4_checkpoint.py:56-59), so 30 weight sets (12.5 GB) stream per step.  Steps/s over
    `steps` steps with the temperature schedule."""
    import fused_moe_w4_v2
    import fused_sampler_ops
    import moe_router
    import workloads
    sets = [workloads.moe_weights(E, H, I, seed=200 + i, device=dev) for i in range(30)]
    blocks = [workloads.moe_inputs(T, H, E, seed=300 + b, device=dev) for b in range(60)]
    h0 = blocks[0]["hidden"]
    logits = workloads.sampler_logits(256, V_SAMPLER, seed=5, device=dev)
    xp = torch.empty(T, H, dtype=torch.float16, device=dev)

    def step(k):
        h = h0
        for b in range(60):
            W, inp = sets[b % 30], blocks[b]
            yn, ids, w, _ = moe_router.rmsnorm_route_topk(h, inp["norm_w"], 1e-6, inp["router_w"],
                                                          TOPK, bias=inp["bias"], xperm=xp,
                                                          want_logits=False)
            h = h + fused_moe_w4_v2.moe_forward(yn, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"],
                                                W["dn_s"], W["dn_z"], ids, w, hidden_perm=xp,
                                                int_zeros=False)
        return fused_sampler_ops.sample_step(logits, workloads.step_seed(1234, k),
                                             workloads.temperature(k))
    step(0)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for k in range(steps):
        step(k)
    ev1.record()
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    del sets
    torch.cuda.empty_cache()
    return {"steps_per_s": steps / (ms * 1e-3), "ms_per_step": ms / steps, "steps": steps,
            "blocks": 60, "weight_sets": 30, "canvas_tokens": T,
            "data": "synthetic (random-init weights of configs[0] shapes; sampler logits N(0,3))"}


PREFILL_TOKENS = 2048 + 16384  # configs[4]: 8 canvases + one 16384-token prefill chunk


def time_prefill(dev, steps, rank, world):
    """18432 tokens (8 canvases + a 16384-token prefill chunk), Zipf routing, through
    RMSNorm -> router -> MoE; with N > 1 each rank holds 128/N experts and 18432/N tokens
    (expert parallelism).  Job-wide tokens/s and per-GPU HBM GB/s."""
    import fused_moe_w4_v2
    import moe_router
    import workloads
    Tr = PREFILL_TOKENS // world
    Wf = workloads.moe_weights(E, H, I, seed=400, device=dev)
    inp = workloads.moe_inputs(Tr, H, E, seed=500 + rank, device=dev)
    xp = torch.empty(Tr, H, dtype=torch.float16, device=dev)
    tpe = PREFILL_TOKENS * TOPK // E
    if world > 1:
        import ep_moe
        relabel, order = balanced_owners(Tr, [500 + r for r in range(world)], world, tpe, dev)
        layer = ep_moe.P2PExpertParallelMoE(*ep_moe.shard_experts(Wf["gu_q"], Wf["gu_s"],
                                                                    Wf["gu_z"], Wf["dn_q"],
                                                                    Wf["dn_s"], Wf["dn_z"], rank,
                                                                    world, interleaved=True,
                                                                    order=order),
                                            E_total=E, int_zeros=False, max_tokens=Tr, topk=TOPK,
                                            relabel=relabel)
        del Wf

    def step():
        yn, ids, w, _ = moe_router.rmsnorm_route_topk(inp["hidden"], inp["norm_w"], 1e-6,
                                                      inp["router_w"], TOPK, bias=inp["bias"],
                                                      xperm=xp, want_logits=False)
        if world > 1:
            return layer(xp, ids, w, out_dtype=torch.float16, tokens_per_expert=tpe), ids
        return fused_moe_w4_v2.moe_forward(yn, Wf["gu_q"], Wf["gu_s"], Wf["gu_z"], Wf["dn_q"],
                                           Wf["dn_s"], Wf["dn_z"], ids, w, hidden_perm=xp,
                                           int_zeros=False), ids
    for _ in range(3):
        _, ids = step()
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    if world > 1:
        torch.distributed.all_reduce(counts)
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    # per-step events (their median shows whether one step stalled) inside the bracketing pair
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    clk = Clocks(dev.index if dev.index is not None else 0) if rank == 0 else None
    evs[0].record()
    for i in range(steps):
        step()
        evs[i + 1].record()
    torch.cuda.synchronize(dev)
    clocks = clk.stop() if clk is not None else None
    per_step = sorted(evs[i].elapsed_time(evs[i + 1]) for i in range(steps))
    t = torch.tensor([evs[0].elapsed_time(evs[-1])], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item()) / steps
    layer_bytes = workloads.moe_layer_bytes(counts.cpu().numpy(), T=PREFILL_TOKENS)
    # tensor-bound at ~1150 pairs per expert: the expert GEMMs' FLOPs per GPU over the step time
    tpeak, tkind = tensor_peak()
    tflops = workloads.moe_layer_flops(PREFILL_TOKENS * TOPK) / world / (ms * 1e-3) / 1e12
    return {"tokens_per_s": PREFILL_TOKENS / (ms * 1e-3), "ms_per_step": ms, "steps": steps,
            "ms_median_step_rank0": per_step[len(per_step) // 2], "ms_max_step_rank0": per_step[-1],
            "clocks": clocks,
            "tokens": PREFILL_TOKENS, "n_gpus": world,
            "per_gpu_tflops": tflops, "tensor_frac": tflops / tpeak, "tensor_peak_tflops": tpeak,
            "tensor_peak_kind": tkind,
            "per_gpu_hbm_gbs": layer_bytes / world / (ms * 1e-3) / 1e9,
            "max_tokens_per_expert": int(counts.max()),
            "engine": "tc" if tpe > 36 else "ws"}


def time_sampler(dev, reps=1):
    """48 denoising steps with the temperature schedule; per step one fused pass
    (entropy + Gumbel-max + argmax) and one acceptance/stop launch."""
    import accept_ops
    import fused_sampler_ops
    import workloads
    xs = [workloads.sampler_logits(256, V_SAMPLER, seed=s, device=dev) for s in (0, 1)]
    canvas = torch.zeros(1, 256, dtype=torch.int64, device=dev)
    hist = torch.full((2, 1, 256), -1, dtype=torch.int64, device=dev)

    def run(step, x):
        Tm = workloads.temperature(step)
        h, s, a = fused_sampler_ops.sample_step(x, workloads.step_seed(1234, step), Tm)
        accept_ops.accept_and_stop(h.view(1, 256), canvas, s.view(1, 256), 0.1, a.view(1, 256),
                                   hist, 0.005)
    for i in range(3):
        run(i, xs[i % 2])
    torch.cuda.synchronize(dev)
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kern_ms = 0.0
    e0.record()
    n = 0
    for _ in range(reps):
        for step in range(48):
            x = xs[step % 2]
            k0.record()
            fused_sampler_ops.sample_step(x, workloads.step_seed(1234, step),
                                          workloads.temperature(step))
            k1.record()
            torch.cuda.synchronize(dev)
            kern_ms += k0.elapsed_time(k1)
            n += 1
    e1.record()
    torch.cuda.synchronize(dev)
    # full step (fused pass + acceptance/stop), back to back
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for step in range(48):
        run(step, xs[step % 2])
    f1.record()
    torch.cuda.synchronize(dev)
    return f0.elapsed_time(f1) / 48.0, kern_ms / n


# --------------------------------------------------------------------------------- CPU arms
def time_selfcond(dev, reps=20, T=0.6):
    """The denoising step's self-conditioning copy (bf16 of the processed logits): the sampler
    pass with the copy written by the pass itself, against the pass alone and against torch's
    separate cast of the fp32 logits (the reference step's .to(bfloat16), fast_sampler.py:109)."""
    import fused_sampler_ops
    import workloads
    x = workloads.sampler_logits(256, V_SAMPLER, seed=0, device=dev).view(1, 256, V_SAMPLER)
    prev = torch.zeros(x.shape, dtype=torch.bfloat16, device=dev)
    fin = torch.zeros(1, dtype=torch.bool, device=dev)

    def t(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1000.0 / reps
    base = t(lambda: fused_sampler_ops.sample_step(x, 1234, T))
    fused = t(lambda: fused_sampler_ops.sample_step_selfcond(x, 1234, T, prev, fin))
    cast = t(lambda: x.to(torch.bfloat16))
    return {"temperature": T, "sample_step_us": base, "sample_step_with_copy_us": fused,
            "separate_cast_us": cast, "copy_bytes": x.numel() * 2}


def cpu_layer(nthreads):
    """One configs[1] layer of the reference algorithm on the host, all 128 experts: the oracle
    restatement of the reference's torch path (RMSNorm, router, per-expert F.linear on
    dequant_w4 weights, tanh-GELU, fixed-order combine), with the dequantisation inside the
    timed region.  Returns microseconds."""
    from oracle import ref
    torch.set_num_threads(nthreads)
    W, inp = _cpu_inputs()
    t0 = time.perf_counter()
    xn = ref.rmsnorm(inp["hidden"], inp["norm_w"], 1e-6)
    ids, w, _ = ref.router_topk(xn, inp["router_w"], inp["bias"], TOPK)
    ref.moe_layer(xn, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"], W["dn_z"], ids, w)
    return (time.perf_counter() - t0) * 1e6


_CPU_CACHE = {}


def _cpu_inputs():
    """The CPU layer's packed weights and inputs (built once)."""
    import workloads
    if "W" not in _CPU_CACHE:
        _CPU_CACHE["W"] = workloads.moe_weights(E, H, I, seed=100)
        _CPU_CACHE["inp"] = workloads.moe_inputs(T, H, E, seed=0)
    return _CPU_CACHE["W"], _CPU_CACHE["inp"]


CPU_SAMPLE = ("the full configs[1] layer (RMSNorm + router + all 128 experts, dequant inside the "
              "timed region) per step")


def cpu_layer_predequant(nthreads):
    """The same CPU layer with every expert's weights dequantised to fp32 before the timed region
    (the second way the reference's torch path can run).  Returns microseconds."""
    from oracle import ref
    torch.set_num_threads(nthreads)
    W, inp = _cpu_inputs()
    dense = _CPU_CACHE.get("dense")
    if dense is None:
        dense = _CPU_CACHE["dense"] = ref.dense_experts(W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"],
                                                        W["dn_s"], W["dn_z"])
    t0 = time.perf_counter()
    xn = ref.rmsnorm(inp["hidden"], inp["norm_w"], 1e-6)
    ids, w, _ = ref.router_topk(xn, inp["router_w"], inp["bias"], TOPK)
    ref.moe_layer(xn, W["gu_q"], W["gu_s"], W["gu_z"], W["dn_q"], W["dn_s"], W["dn_z"], ids, w,
                  dense=dense)
    return (time.perf_counter() - t0) * 1e6


def cpu_sampler_step(nthreads):
    """One configs[2] sampler step of the reference algorithm on the host (temperature of step
    24): Categorical entropy of the processed logits, the Philox Gumbel-max sample and argmax
    (the oracle's C restatement on `nthreads` threads) and the entropy-bound acceptance.
    Returns microseconds."""
    import workloads
    from oracle import ref
    torch.set_num_threads(nthreads)
    x = _CPU_CACHE.get("logits")
    if x is None:
        x = _CPU_CACHE["logits"] = workloads.sampler_logits(256, V_SAMPLER, seed=0)
    cur = torch.zeros(1, 256, dtype=torch.int64)
    step = 24
    Tm = workloads.temperature(step)
    t0 = time.perf_counter()
    h = ref.entropy(x / Tm)
    s, _ = ref.gumbel_argmax(x, workloads.step_seed(1234, step), temperature=Tm, nthreads=nthreads)
    ref.accept_canvas(h.view(1, 256), cur, s.view(1, 256), 0.1)
    return (time.perf_counter() - t0) * 1e6


def cpu_baseline(nthreads, runs=5, warmup=1):
    """Median of `runs` full CPU layers after `warmup`, with their spread."""
    vals = [cpu_layer(nthreads) for _ in range(warmup + runs)][warmup:]
    med = statistics.median(vals)
    return med, (max(vals) - min(vals)) / med


def reference_arm(args, rank):
    if rank != 0:
        return
    ncores = len(os.sched_getaffinity(0))
    vals = [cpu_layer(ncores) for _ in range(args.warmup + args.steps)][args.warmup:]
    v = statistics.median(vals)
    line = {"metric": METRIC, "value": v, "unit": "us", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": v / 1000.0, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "configs[1]: RMSNorm -> router (Zipf bias) -> W4A16 MoE layer, "
                                   "T=256 H=2816 I=704 E=128 top-8", "device": "cpu"},
            "cpu_baseline": {"value": v, "unit": "us", "cores": ncores, "kind": "port",
                             "sample": CPU_SAMPLE,
                             "spread": (max(vals) - min(vals)) / v},
            "e2e": {"value": v, "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the configs[3] stack and configs[4] prefill measurements")
    ap.add_argument("--only", choices=("layer", "sampler", "prefill", "stack"), default=None,
                    help="run just one workload (used for profiling captures); prints its timing")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    dist = world > 1
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.only == "layer":
        ms, stages, counts, _ = time_layer(dev, args.steps, args.warmup, False)
        print(json.dumps({"only": "layer", "us_per_layer": ms * 1000.0 / args.steps,
                          "stages_us": {k: v * 1000.0 for k, v in stages.items()}}), flush=True)
        return
    if args.only == "sampler":
        step_ms, kern_ms = time_sampler(dev)
        print(json.dumps({"only": "sampler", "step_us": step_ms * 1000.0,
                          "kernel_us": kern_ms * 1000.0}), flush=True)
        return
    if args.only == "prefill":
        print(json.dumps({"only": "prefill", **time_prefill(dev, max(10, 2 * args.steps), 0, 1)}),
              flush=True)
        return
    if args.only == "stack":
        print(json.dumps({"only": "stack", **time_stack(dev)}), flush=True)
        return
    if dist:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    if dist:
        ms, counts, clocks, e2e_ms, h2d, d2h, ep_stages = time_layer_ep(dev, args.steps,
                                                                        args.warmup, rank, world)
        stages = {}
    else:
        ms, stages, counts, clocks = time_layer(dev, args.steps, args.warmup, dist)
    ms_step = ms / args.steps
    value = ms * 1000.0 / (args.steps * world)
    import workloads
    peak, peak_kind = peaks()
    touched = int((counts > 0).sum())
    bytes_layer = workloads.moe_layer_bytes(counts.numpy())
    gemm1_bytes = touched * (2 * I * H // 2 + 2 * I * (H // 128) * 4) + T * H * 2
    gemm1_ms = stages.get("gate_up_gelu")
    if not dist:
        e2e_ms, h2d, d2h = time_layer_e2e(dev, args.steps, args.warmup)
    samp_step_ms, samp_kern_ms = time_sampler(dev)
    cfg4 = None if args.no_extra else time_prefill(dev, max(10, 2 * args.steps), rank, world)
    selfcond = None if (args.no_extra or rank != 0) else time_selfcond(dev)
    cfg3 = None if (args.no_extra or dist) else time_stack(dev)
    if dist:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    cpu = cpu_extra = None
    if not args.no_cpu_baseline and not dist:  # rank 0 at N = 1 only
        ncores = len(os.sched_getaffinity(0))
        us, spread = cpu_baseline(ncores)
        cpu = {"value": us, "unit": "us", "cores": ncores, "kind": "port",
               "sample": CPU_SAMPLE + ", median of 5 after 1 warm-up", "spread": spread}
        pre = [cpu_layer_predequant(ncores) for _ in range(4)][1:]
        samp = [cpu_sampler_step(ncores) for _ in range(4)][1:]
        cpu_extra = {
            "layer_predequantised": {"value": statistics.median(pre), "unit": "us",
                                     "cores": ncores, "kind": "port",
                                     "sample": "the same layer with every expert's weights "
                                               "dequantised to fp32 before the timed region, "
                                               "median of 3 after 1 warm-up"},
            "sampler_step": {"value": statistics.median(samp), "unit": "us", "cores": ncores,
                             "kind": "port",
                             "sample": "one configs[2] step at step 24's temperature (entropy, "
                                       "Philox Gumbel-max and argmax, acceptance) over all 256 "
                                       "rows, median of 3 after 1 warm-up"}}
    # the kernel roofline is the single-GPU layer's (per-stage events exist only there)
    achieved = gemm1_bytes / (gemm1_ms * 1e-3) / 1e9 if gemm1_ms else None
    engine = os.environ.get("KNX_ENGINE", "auto")
    if engine == "auto":  # the library's rule on job-wide pairs per expert: ws up to 36, else tc
        engine = "ws" if T * TOPK * world // E <= 36 else "tc"
    line = {
        "metric": METRIC, "value": value, "unit": "us", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "configs[1]: RMSNorm -> router (Zipf bias) -> W4A16 MoE layer, "
                               "T=256 H=2816 I=704 E=128 top-8, gate_up gs128 / down gs64",
                   "l2": f"{NSETS} rotating weight sets ({NSETS} x 416 MB) > 126 MB L2",
                   "parallelism": (f"expert-parallel x{world} (128/{world} experts per GPU, "
                                   f"owners balanced by the job's routing, one 256-token canvas "
                                   f"per GPU, device-initiated NVLink exchange through symmetric "
                                   f"memory)" if world > 1 else "single GPU"),
                   "touched_experts": touched,
                   "max_tokens_per_expert": int(counts.max())},
        "layer_hbm_gbs": bytes_layer / (ms_step * 1e-3) / 1e9,
        # each step streams every touched expert once, split over the ranks: per-GPU fraction
        "layer_hbm_frac": bytes_layer / (ms_step * 1e-3) / 1e9 / (peak * world),
        "layer_bytes": bytes_layer,
        "stages_us": ({k: v * 1000.0 for k, v in stages.items()} if not dist else
                      {"note": "per rank, with events between stages (no overlap), max over ranks",
                       **ep_stages}),
        "roofline": {"kernel": GEMM1_KERNEL[engine], "bound": "hbm", "achieved": achieved,
                     "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak if achieved else None,
                     "peak_kind": peak_kind, "traffic": GEMM1_NCU_TRAFFIC.get(engine),
                     "algorithmic_bytes": gemm1_bytes,
                     **({} if achieved else {"note": "per-kernel events are taken on the "
                                                     "single-GPU layer only; layer_hbm_frac is "
                                                     "the per-GPU fraction of this run"})},
        "sampler_step_us": samp_step_ms * 1000.0,
        "sampler_roofline": {"kernel": "sampler_stream_kernel + row_merge_kernel", "bound": "hbm",
                             "achieved": 256 * V_SAMPLER * 4 / (samp_kern_ms * 1e-3) / 1e9,
                             "peak": peak, "unit": "GB/s",
                             "frac": 256 * V_SAMPLER * 4 / (samp_kern_ms * 1e-3) / 1e9 / peak,
                             "kernel_us": samp_kern_ms * 1000.0},
        "e2e": {"value": e2e_ms * 1000.0 / (args.steps * world), "unit": "us",
                "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world},
        "gpu_launches": (EP_LAUNCHES_PER_LAYER if dist else LAUNCHES_PER_LAYER) * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
        "cpu_baselines_extra": cpu_extra,
        "configs3_stack": cfg3,
        "configs4_prefill": cfg4,
        "sampler_selfcond": selfcond,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
