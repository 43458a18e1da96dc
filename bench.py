#!/usr/bin/env python
"""Benchmark of the DiT hot path: seconds per 30-layer DiT denoise step of Wan2.2-TI2V-5B at
7854 tokens (latent grid 21x17x22, 704x544x81 video) with CFG (cond + uncond), on N B200s of
one node.  N = 1 runs the whole step (batch 2) on one GPU; N > 1 uses --layout (default: CFG
groups of N/2 GPUs with Q-local sequence parallelism inside, see wanb200.parallel).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--layout L]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Prints one JSON line on rank 0.  `value` is device time per step (CUDA events, inputs resident
in HBM, max over ranks, no per-launch instrumentation); `kernels` and `roofline` come from a
second pass over the same steps with a CUDA-event pair around every launch; `e2e` is the same
step through the public `FastWanDiT.__call__` with the latent copied from pinned host memory
and the noise prediction copied back every step.
Weights are seeded N(0, 0.02) bf16 with the TI2V-5B shapes, the text context is seeded, so
`data` is synthetic.  `device_error` is the kernels' error word after all the timed steps (max
over ranks); `parity` is the rel-RMS of the step-0 prediction against the fp32 CPU oracle over
all the layers (N = 1; that oracle run is also the `cpu_baseline`) or against a single-GPU run of
the same model (N > 1).  `graph` (N = 1) is the device time per replay of the same step
captured as one CUDA graph (`FastWanDiT.capture`) and whether its prediction equals the eager
step's.  A non-zero error word or a parity miss ends the run with a non-zero
status after the line is printed.  `--impl reference` times the CPU oracle (the reference's fp32
block math, ref_fp32.main restated in oracle/dit_ref.py): one whole step on this host's cores.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "wan2-ti2v-5b_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "DiT s/step @7854 tok CFG=2 at 1/2/4/8 B200; self-attn TFLOP/s vs bf16 peak"
GRID = (21, 17, 22)
LATENT = (48, 21, 34, 44)
GUIDE = 5.0
T_STEP = 999.0
CFG_BATCH = 2
CTX_LEN, TEXT_DIM = 512, 4096

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per launch at config 2, by kernel
# role, from ncu captures summarised in profiles/ (command lines there).
NCU_TRAFFIC_PER_LAUNCH = {
    "attn_self": (364_468_992, "ncu dram__bytes_read.sum + dram__bytes_write.sum of the self-attention launch "
                               "inside a 2-layer config-2 step (profiles/attn_persistent_self_b2h24_l7854.txt); "
                               "algorithmic bytes q+k+v+o = 386 MB"),
}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """SM clock, max clock and clock-event (throttle) reasons of this rank's GPU, read through
    NVML every 20 ms from a background thread while the timed region runs (read-only queries)."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, torch_device_index):
        self.idx = torch_device_index
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.error = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                nvml_idx = torch.cuda._get_nvml_device_index(self.idx)
            except Exception:
                nvml_idx = self.idx
            self._h = pynvml.nvmlDeviceGetHandleByIndex(nvml_idx)
            self._nv = pynvml
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
            self._bits = [(n, getattr(pynvml, c)) for n, c in self.REASONS]
        except Exception as ex:  # no NVML: report no samples
            self.error = repr(ex)
            return
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for n, bit in self._bits:
                    if r & bit:
                        self.reasons.add(n)
            except Exception as ex:
                self.error = repr(ex)
                return
            time.sleep(0.02)

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
               "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml, 20 ms"}
        if self.error:
            out["error"] = self.error
        return out


def init_dist(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 under torchrun")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


STEP_TOL = 5e-2  # north star: rel-RMS of the step-0 noise prediction


def rel_rms(a, b) -> float:
    """||a - b|| / ||b|| (the reference's error score, ref_fp32.py:108)."""
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


ORACLE_CFG = {"num_heads": 24, "num_layers": 30, "freq_dim": 256, "patch": (1, 2, 2), "out_dim": 48}


def oracle_step(sd, ctx, ctx_null, latent, layers, threads=None):
    """Step-0 CFG noise prediction of config 2 through the fp32 CPU oracle (the reference's
    scripts/validate/ref_fp32.py:62-99, restated in oracle/dit_ref.py) on this host's cores.
    sd may live on the GPU in bf16: the oracle copies one block at a time to fp32 host tensors.
    Returns (prediction [48, F, H, W] fp32, seconds)."""
    from oracle import dit_ref as R
    torch.set_num_threads(threads or os.cpu_count() or 1)
    cfg = dict(ORACLE_CFG, num_layers=layers)
    with torch.no_grad():
        t0 = time.perf_counter()
        pred = R.step(sd, cfg, latent, T_STEP, ctx, ctx_null, GUIDE)
        return pred, time.perf_counter() - t0


def cpu_info():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args):
    """Reference arm: the reference's own CPU implementation of the path (its fp32 block math,
    ref_fp32.block_fwd / main, restated in oracle/dit_ref.py) on all host cores, rank 0 only: one
    whole 30-layer config-2 step (B=2, L=7854, dim 3072) timed end to end, nothing extrapolated.
    The 30 layers share one seeded block's fp32 weights (CPU time does not depend on the values;
    generating 30 distinct blocks on the host would take longer than the step)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_grad_enabled(False)
    from wanb200.weights import TI2V_5B, random_block_state, random_model_state
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    spec = TI2V_5B
    emb = {k: v.float() for k, v in random_model_state(spec, seed=0, num_layers=0).items()}
    blk = {k: v.float() for k, v in random_block_state(spec, 0).items()}
    sd = dict(emb)
    for i in range(args.layers):
        sd.update({f"blocks.{i}.{k}": v for k, v in blk.items()})
    g = torch.Generator().manual_seed(123)
    ctx, ctx_null = torch.randn(CTX_LEN, TEXT_DIM, generator=g), torch.randn(CTX_LEN, TEXT_DIM, generator=g)
    latent = torch.randn(LATENT, generator=torch.Generator().manual_seed(7))
    pred, secs = oracle_step(sd, ctx, ctx_null, latent, args.layers, threads)
    assert torch.isfinite(pred).all()
    sample = (f"one whole {args.layers}-layer config-2 step-0 (B=2, L=7854, dim 3072, CFG) through the fp32 oracle "
              f"(ref_fp32.main restated), timed once; --steps/--warmup not used (one step is ~{secs:.0f} s); "
              f"host: {cpu_info()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": secs, "unit": "s/step", "n_gpus": world,
        "steps": 1, "warmup": 0, "requested_steps": args.steps, "requested_warmup": args.warmup,
        "layers_timed": args.layers, "extrapolated": False, "ms_per_step": secs * 1e3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config2: {args.layers}-layer Wan2.2-TI2V-5B DiT step, 7854 tokens (21x17x22), "
                               "CFG batch 2", "global_batch": CFG_BATCH, "seq_len": GRID[0] * GRID[1] * GRID[2],
                   "parallelism": "cpu", "inputs_larger_than_l2": True},
        "cpu_baseline": {"value": secs, "unit": "s/step", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": secs, "unit": "s/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    world, rank, local = init_dist(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    torch.set_grad_enabled(False)
    from wanb200 import FastWanDiT, TI2V_5B, random_model_state
    from wanb200 import ops
    from wanb200.dit import block_flops

    spec = TI2V_5B
    layers = args.layers
    sd = random_model_state(spec, seed=0, device=device, num_layers=layers)
    from wanb200.parallel import make_layout
    lay = make_layout(args.layout)
    fast = FastWanDiT((spec, sd), GRID, GUIDE, device, cfg_group=lay.cfg_group, pair_group=lay.pair_group,
                      tp_group=lay.tp_group, num_layers=layers, comm=args.comm, sp_group=lay.sp_group)
    # sd stays: the parity check below runs the same seeded weights through the oracle (N = 1) or
    # through a single-GPU model on rank 0 (N > 1)
    g = torch.Generator(device=device).manual_seed(123)
    ctx = torch.randn(CTX_LEN, TEXT_DIM, generator=g, device=device)
    ctx_null = torch.randn(CTX_LEN, TEXT_DIM, generator=g, device=device)
    fast.set_context(ctx, ctx_null)
    latent_host = torch.randn(LATENT, generator=torch.Generator().manual_seed(7)).pin_memory()
    latent_dev = latent_host.to(device)
    out_host = torch.empty(LATENT, dtype=torch.bfloat16).pin_memory()  # the prediction is bf16, as the reference's
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(device)

    for _ in range(args.warmup):
        fast(latent_dev, T_STEP)
    barrier()

    # ---- device-timed steps (inputs resident), no per-launch events in this region
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = ops.launch_count
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        out = fast(latent_dev, T_STEP)
    t1.record(stream)
    barrier()
    launches = ops.launch_count - launches0
    step_s = max_over_ranks(t0.elapsed_time(t1) / 1e3 / args.steps, world, device)
    clk = clocks.stop()

    # ---- the same steps again with a CUDA-event pair around every launch (on its stream): the
    # per-kernel times of the roofline and the breakdown
    timer = ops.KernelTimer()
    ops.set_timer(timer)
    barrier()
    for _ in range(args.steps):
        out = fast(latent_dev, T_STEP)
    barrier()
    ops.set_timer(None)
    kern = timer.summary()

    # ---- end to end through the public call: pinned H2D of the latent, D2H of the prediction
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        lat = latent_host.to(device, non_blocking=True)
        out = fast(lat, T_STEP)
        out_host.copy_(out, non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_s = max_over_ranks(e0.elapsed_time(e1) / 1e3 / args.steps, world, device)
    assert torch.isfinite(out_host).all()

    # ---- the same step captured as one CUDA graph (FastWanDiT.capture; single GPU only): device
    # time per replay and whether its prediction equals the eager step's bit for bit
    graph = None
    if world == 1 and not args.no_graph:
        try:
            step = fast.capture(latent_dev)
            for _ in range(args.warmup):
                step(latent_dev, T_STEP)
            barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            for _ in range(args.steps):
                out_g = step(latent_dev, T_STEP)
            g1.record(stream)
            barrier()
            graph = {"value": g0.elapsed_time(g1) / 1e3 / args.steps, "unit": "s/step", "steps": args.steps,
                     "equal_to_eager": bool(torch.equal(out_g, fast(latent_dev, T_STEP))),
                     "what": "FastWanDiT.capture: the whole step as one CUDA graph, replayed with the same inputs"}
            del step, out_g
        except RuntimeError as exc:  # reported, not fatal: the headline is the eager step above
            graph = {"error": str(exc).splitlines()[0][:200]}

    # ---- device error word: every bounded wait inside the kernels of all the steps above
    derr = int(max_over_ranks(float(fast.check_device_errors(raise_error=False)), world, device))

    # ---- parity of the step-0 prediction: N = 1 against the fp32 CPU oracle over all the
    # layers (the reference's own score, ref_fp32.py:62-109; its time is the cpu_baseline); N > 1
    # against a single-GPU run of the same seeded model on rank 0
    pred = fast(latent_dev, T_STEP).float()
    parity, oracle_s = None, None
    if world == 1:
        if not args.no_cpu_baseline:
            ref, oracle_s = oracle_step(sd, ctx, ctx_null, latent_host, layers)
            parity = {"rel_rms": rel_rms(pred, ref), "tol": STEP_TOL,
                      "against": f"fp32 CPU oracle, whole {layers}-layer step-0 (ref_fp32.main restated)"}
    else:
        if rank == 0:
            single = FastWanDiT((spec, sd), GRID, GUIDE, device, num_layers=layers)
            single.set_context(ctx, ctx_null)
            ref = single(latent_dev, T_STEP).float()
            parity = {"rel_rms": rel_rms(pred, ref), "tol": STEP_TOL,
                      "against": "single-GPU step-0 of the same seeded model (rank 0; itself checked against the "
                                 "CPU oracle at N = 1)"}
            del single, ref
        barrier()
    if parity is not None:
        parity["ok"] = parity["rel_rms"] <= parity["tol"]
    del sd

    if rank != 0:
        if world > 1:
            dist.barrier(device_ids=[local])
            dist.destroy_process_group()
        return

    peaks = measured_peaks()
    hbm_kinds = {"layernorm", "qk_norm_rope", "bias_gate_residual", "kv_gather", "peer_barrier",
                 "tp_allreduce_exposed", "patchify", "unpatchify", "sumsq_reduce"}
    total_ms = sum(x[1] for x in kern.values())
    per_kernel = {k: {"launches": v[0], "ms": v[1], "share": v[1] / total_ms,
                      ("tflops" if k not in hbm_kinds else "gbs"):
                          (v[2] / (v[1] / 1e3) / (1e12 if k not in hbm_kinds else 1e9))} for k, v in kern.items()}
    g_all = [v for k, v in kern.items() if k.startswith("gemm")]
    if g_all:
        gms, gw = sum(v[1] for v in g_all), sum(v[2] for v in g_all)
        per_kernel["gemm_all"] = {"launches": sum(v[0] for v in g_all), "ms": gms, "share": gms / total_ms,
                                  "tflops": gw / (gms / 1e3) / 1e12}
    # the dominant kernel: the single kernel (by role) with the largest device time
    dom = max(kern, key=lambda k: kern[k][1])
    n, ms, work = kern[dom]
    if dom in hbm_kinds:
        achieved = work / n / (ms / n / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s"}
    else:
        achieved = work / n / (ms / n / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["kernel"] = ("attn_persistent_kernel (" + dom[5:] + ")") if dom.startswith("attn") else (
        "gemm_bf16_kernel (" + dom[5:] + ")" if dom.startswith("gemm") else dom)
    roof["peak_kind"] = f"{peaks['source']} {'sustained bf16' if roof['bound'] == 'tensor' else 'HBM copy'}"
    if roof["bound"] == "tensor":
        roof["frac_of_burst_peak"] = roof["achieved"] / peaks["bf16_tflops"]
    roof["launches"] = n
    roof["ms_per_launch"] = ms / n
    roof["work_per_launch"] = work / n
    tr = NCU_TRAFFIC_PER_LAUNCH.get(dom) if world == 1 else None  # captured on the 1-GPU launch shapes
    roof["traffic"] = tr[0] if tr else None
    if tr:
        roof["traffic_note"] = tr[1]
    sa = kern.get("attn_self")
    self_attn = None
    if sa:
        tf = sa[2] / (sa[1] / 1e3) / 1e12
        self_attn = {"tflops": tf, "frac_of_burst_peak": tf / peaks["bf16_tflops"],
                     "frac_of_sustained_peak": tf / peaks["bf16_tflops_sustained"], "ms_per_launch": sa[1] / sa[0]}

    fl = block_flops(CFG_BATCH * GRID[0] * GRID[1] * GRID[2], GRID[0] * GRID[1] * GRID[2])
    step_flops = layers * sum(fl.values())
    line = {
        "metric": METRIC, "value": step_s, "unit": "s/step", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) bf16 weights, seeded context/latent)",
        "config": {"workload": f"config2: {layers}-layer Wan2.2-TI2V-5B DiT step, 7854 tokens (21x17x22), CFG batch 2",
                   "global_batch": CFG_BATCH, "seq_len": GRID[0] * GRID[1] * GRID[2],
                   "parallelism": lay.describe(world) + (f", {args.comm} collectives"
                                                          if (fast.sp or fast.kv_gather is not None) else ""),
                   "layers": layers, "inputs_larger_than_l2": True,
                   "l2_note": "each step streams ~9.8 GB of weights, far above the 126 MB L2"},
        "e2e": {"value": e2e_s, "unit": "s/step",
                # the latent, and the timestep's per-frame sinusoid (computed on the host, as the
                # reference's _time_embed does)
                "h2d_bytes_per_step": latent_host.numel() * 4 + GRID[0] * 256 * 2,
                "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
        "gpu_launches": launches,
        "roofline": roof,
        "self_attn": self_attn,
        "step_tflops": step_flops / step_s / 1e12,
        "kernels": per_kernel,
        "clocks": clk,
        "device_error": derr,
        "parity": parity,
        "graph": graph,
    }
    if oracle_s is not None:
        line["cpu_baseline"] = {"value": oracle_s, "unit": "s/step", "cores": torch.get_num_threads(),
                                "kind": "port",
                                "sample": f"one whole {layers}-layer step-0 (B=2, L=7854, dim 3072, CFG) through the "
                                          f"fp32 oracle, timed once (the run the parity key compares with); "
                                          f"host: {cpu_info()}"}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if derr or (parity is not None and not parity["ok"]):
        raise SystemExit(f"invalid run: device error word {derr}, parity {parity}")


GRID4, LATENT4, STEPS4, SHIFT4 = (31, 22, 40), (48, 31, 44, 80), 10, 1.0


def run_config4(args):
    """The long-video workload: the 10-step UniPC denoise loop at 1280x704, 121 frames (27280 tokens),
    CFG, image frame pinned to a seeded image latent, timesteps linear from 999 (shift 1), on N
    GPUs in --layout.  One JSON line: seconds per loop (device time, max over ranks), e2e with
    the latent copied in and the result copied out."""
    world, rank, local = init_dist(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    torch.set_grad_enabled(False)
    from wanb200 import FastWanDiT, TI2V_5B, random_model_state
    from wanb200 import ops
    from wanb200.parallel import make_layout
    from wanb200.unipc import denoise
    from wanb200.dit import block_flops

    spec = TI2V_5B
    sd = random_model_state(spec, seed=0, device=device, num_layers=args.layers)
    lay = make_layout(args.layout)
    fast = FastWanDiT((spec, sd), GRID4, GUIDE, device, cfg_group=lay.cfg_group, pair_group=lay.pair_group,
                      tp_group=lay.tp_group, num_layers=args.layers, comm=args.comm, sp_group=lay.sp_group)
    del sd
    g = torch.Generator(device=device).manual_seed(123)
    fast.set_context(torch.randn(CTX_LEN, TEXT_DIM, generator=g, device=device),
                     torch.randn(CTX_LEN, TEXT_DIM, generator=g, device=device))
    gh = torch.Generator().manual_seed(0)
    latent_host = torch.randn(LATENT4, generator=gh).pin_memory()
    image_host = torch.randn((LATENT4[0], 1) + LATENT4[2:], generator=gh).pin_memory()
    latent_dev, image_dev = latent_host.to(device), image_host.to(device)
    out_host = torch.empty(LATENT4, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(device)

    for _ in range(args.warmup):
        fast(latent_dev, 999.0)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    launches0 = ops.launch_count
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.loops):
        out = denoise(fast, latent_dev, STEPS4, SHIFT4, image_dev)
    t1.record(stream)
    barrier()
    launches = ops.launch_count - launches0
    loop_s = max_over_ranks(t0.elapsed_time(t1) / 1e3 / args.loops, world, device)
    clk = clocks.stop()
    assert torch.isfinite(out).all()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    lat = latent_host.to(device, non_blocking=True)
    img = image_host.to(device, non_blocking=True)
    out = denoise(fast, lat, STEPS4, SHIFT4, img)
    out_host.copy_(out, non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_s = max_over_ranks(e0.elapsed_time(e1) / 1e3, world, device)
    derr = int(max_over_ranks(float(fast.check_device_errors(raise_error=False)), world, device))
    if rank == 0:
        L4 = GRID4[0] * GRID4[1] * GRID4[2]
        fl = block_flops(CFG_BATCH * L4, L4)
        loop_flops = STEPS4 * args.layers * sum(fl.values())
        print(json.dumps({
            "metric": "s per 10-step UniPC denoise loop @27280 tok CFG=2 (config 4)", "value": loop_s,
            "unit": "s/loop", "s_per_step": loop_s / STEPS4, "n_gpus": world, "loops": args.loops,
            "warmup": args.warmup, "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) bf16 weights, seeded latent / image latent / context)",
            "config": {"workload": f"config4: {args.layers}-layer Wan2.2-TI2V-5B DiT, 27280 tokens (31x22x40), CFG, "
                                   f"{STEPS4}-step UniPC (shift {SHIFT4}), image frame pinned",
                       "parallelism": lay.describe(world), "seq_len": L4, "layers": args.layers},
            "e2e": {"value": e2e_s, "unit": "s/loop", "h2d_bytes_per_loop": (latent_host.numel() + image_host.numel()) * 4,
                    "d2h_bytes_per_loop": out_host.numel() * 4},
            "gpu_launches": launches, "loop_tflops": loop_flops / loop_s / 1e12, "clocks": clk,
            "device_error": derr}), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if derr:
        raise SystemExit(f"invalid run: device error word {derr}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--comm", default="peer", choices=["peer", "nccl"],
                    help="sequence-parallel collectives: fused into the kernels over NVLink peer memory, or NCCL")
    ap.add_argument("--layout", default="auto", choices=["auto", "tp", "cfg", "sp", "cfgsp", "cfgsptp"],
                    help="N>1: tp = TP over all N ranks (batched CFG); cfg = CFG-parallel groups of N/2 "
                         "(token-sharded TP inside each); sp = Q-local sequence parallelism over all N ranks "
                         "(batched CFG, K/V all-gather); cfgsp = CFG-parallel groups of N/2 with Q-local SP "
                         "inside; cfgsptp = CFG-parallel groups of SP2 x TP(N/4); auto = cfgsp for even N, else sp")
    ap.add_argument("--layers", type=int, default=30, help="blocks per step (30 for the bench line)")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU oracle step (the N = 1 cpu_baseline and parity keys)")
    ap.add_argument("--no-graph", action="store_true",
                    help="skip the N = 1 CUDA-graph replay of the step (the graph key)")
    ap.add_argument("--workload", default="config2", choices=["config2", "config4"],
                    help="config2: the bench line (s/step at 7854 tokens); config4: one line for the "
                         "10-step UniPC loop at 27280 tokens (--loops loops timed)")
    ap.add_argument("--loops", type=int, default=1, help="config4: denoise loops in the timed region")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "config4":
        run_config4(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
