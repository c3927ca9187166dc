#!/usr/bin/env python3
"""Headline benchmark: SigLIP-base encoder images/s on B200 through libsh_ops_cuda.so.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload encoder|layer|gemm512|gemm|attention|rowops|summa]

Workload: 12 pre-LN SigLIP-base layers (S=256, D=768, 12 heads x 64, FFN 3072, tanh-GELU,
scale 1/8, eps 1e-6), a global batch of 512 sequences sharded data-parallel over the N ranks (B = 512 / N per GPU,
weights replicated: every rank generates the same per-layer N(0, 0.02) weights from the same LCG seeds; x ~ N(0,1)).
One step = one forward pass over the rank's shard, 84 library launches replayed from a CUDA graph (--ln-fold: 61, the
input's row statistics, then per layer 5 launches with both LayerNorms folded into the GEMMs). The activations
(201 MB per tensor at B=512) are larger than the 126 MB L2, so no flush is needed between steps.

One JSON line on rank 0 (the contract of this repository's driver): `value` is the whole-job images/s with the
inputs resident in HBM, timed with CUDA events over K steps between barriers, max over ranks; `e2e` is the same
metric through the public API with the input batch copied from pinned host memory and the result copied back
inside every timed step; `roofline` describes the dominant kernel (the tcgen05 GEMM), `kernels` the per-kernel
breakdown measured with CUDA events around each launch; `cpu_baseline` times the numpy oracle of the same layer on
the host cores (rank 0, N=1 only). `--impl reference` times that CPU implementation alone (there is no GPU
implementation in the reference: it targets a simulated RISC-V accelerator).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "softhier-mlir_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

S, D, F, H, NLAYERS = 256, 768, 3072, 12, 12
GLOBAL_BATCH = 512
EPS, SCALE = 1e-6, 0.125
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---- environment -------------------------------------------------------------------------------------------------
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def init_dist(world: int, local: int):
    import torch
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    """The largest `v` over all ranks (an all-reduce on the process group's device: CUDA for NCCL, CPU for gloo)."""
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def encoder_shard(world: int, rank: int) -> tuple[int, int]:
    """(sequences on this rank, the seed of its input shard): the global batch splits evenly over the ranks; every
    rank generates the same weights and its own input shard, so no data moves between GPUs inside a step."""
    if GLOBAL_BATCH % world:
        raise SystemExit(f"global batch {GLOBAL_BATCH} does not split over {world} ranks")
    from softhier_cuda import encoder
    return GLOBAL_BATCH // world, encoder.INPUT_SEED0 + rank


def job_rate(ms_local: float, steps: int, world: int) -> tuple[float, float]:
    """(ms of the slowest rank, whole-job images/s): the timed region ends when the last rank's last step ends."""
    ms = max_over_ranks(ms_local, world)
    return ms, GLOBAL_BATCH * steps / (ms / 1e3)


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except ValueError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(kernel: str) -> float | None:
    """DRAM bytes per launch of `kernel` at the bench shape, from the committed ncu summary in profiles/
    (a line `traffic_bytes_per_launch <kernel> <bytes>`), or None."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        for m in re.finditer(r"traffic_bytes_per_launch\s+(\S+)\s+([0-9.eE+]+)", f.read_text()):
            if m.group(1) == kernel:
                return float(m.group(2))
    return None


class ClockSampler:
    """SM clock, power and clock-event reasons of this rank's GPU, sampled while the timed region runs.

    NVML (read-only queries) polled every 2 ms from a thread, so even a timed region of a few milliseconds gets
    samples; the GPU is matched by UUID. Without NVML: nvidia-smi every 20 ms. start() returns once the first sample
    exists; mark() is called where the timed region begins and earlier samples are dropped."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, local: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.local = local
        self.index = vis.split(",")[local] if vis else str(local)
        self.proc = None
        self.nvml = None
        self.samples: list[tuple[float, float, int]] = []    # (sm MHz, max MHz, reason bits)
        self.lines: list[str] = []
        self.first = 0
        self.stop_flag = threading.Event()

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.local).uuid)
        for key in (uuid, "GPU-" + uuid):
            try:
                return pynvml, pynvml.nvmlDeviceGetHandleByUUID(key)
            except pynvml.NVMLError:
                continue
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(int(self.index))

    def start(self):
        try:
            nv, h = self._nvml_handle()
            reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons",
                              getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
            mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))

            def poll():
                while not self.stop_flag.is_set():
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), mx,
                                             int(reasons(h)) if reasons else 0))
                    except nv.NVMLError:
                        pass
                    time.sleep(0.002)
            self.nvml = nv
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 2.0:
                time.sleep(0.001)
            return
        except Exception:   # no NVML here: nvidia-smi below
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", self.index, "-lms", "20"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
            return
        t0 = time.time()
        while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)

    def mark(self):
        """The timed region starts now."""
        self.first = len(self.samples) if self.nvml else len(self.lines)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.nvml:
            self.stop_flag.set()
            self.thread.join(timeout=2)
            got = self.samples[self.first:]
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
            reasons = sorted({nm for _, _, bits in got for nm, b in self.REASONS if bits & b})
            return {"sm_mhz": statistics.median(c for c, _, _ in got) if got else None,
                    "sm_max_mhz": got[0][1] if got else None, "samples": len(got), "reasons": reasons,
                    "source": "nvml, 2 ms"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines[self.first:]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons), "source": "nvidia-smi, 20 ms"}


# ---- the GPU arm -----------------------------------------------------------------------------------------------------
def setup_encoder(rt, B: int, input_seed: int, nlayers: int = NLAYERS):
    """Device weights (identical on every rank) and activations for a shard of B sequences: the library's synthetic
    encoder (softhier_cuda.encoder.synthetic_encoder)."""
    from softhier_cuda import encoder
    return encoder.synthetic_encoder(rt, B, S, D, F, nlayers, input_seed)


def schedule_maker(rt, act, layers, M: int, fold: str):
    """(x_in, x_out) -> (calls of one forward pass, result address). By default the 7-launch layer (separate
    LayerNorm kernels); with --ln-fold both LayerNorms of every layer are folded into the GEMMs that consume them
    (sh_cuda_gemm_ln: 1 + 5 launches per layer after a one-time weight transform). The folded form measured ~1 %
    slower at B = 512: the GEMM epilogues, already as long as the main loops, absorb more than the LayerNorm kernels
    cost."""
    from softhier_cuda import encoder
    lib = rt.lib
    if fold == "none":
        return lambda xi, xo: encoder.encoder_schedule(lib, act, layers, H, EPS, SCALE, xi, xo)
    if fold == "ln1":
        folded1 = [encoder.fold_layer_norm1(rt, w, D) for w in layers]
        stats_x = encoder.alloc_row_stats(rt, M, D)[0]
        return lambda xi, xo: encoder.encoder_schedule_ln1_folded(lib, act, folded1, stats_x, H, EPS, SCALE, xi, xo)
    folded = [encoder.fold_layer_norms(rt, w, D, F) for w in layers]
    stats = encoder.alloc_row_stats(rt, M, D)
    return lambda xi, xo: encoder.encoder_schedule_folded(lib, act, folded, stats, H, EPS, SCALE, xi, xo)


def run_ours(args, rank: int, world: int, local: int) -> dict | None:
    import torch
    from softhier_cuda import encoder
    from softhier_cuda.runtime import Runtime

    init_dist(world, local)
    B, input_seed = encoder_shard(world, rank)
    M = B * S
    arena = ((17 * M * D + (M * F - M * D) + NLAYERS * (7 * D * D + 3 * D * F + 16 * F)) * 2 + 2 * M * (D // 64) * 8
             + (256 << 20))
    rt = Runtime.open(local, arena_bytes=arena)
    lib = rt.lib
    layers, act, x_in = setup_encoder(rt, B, input_seed)
    make_schedule = schedule_maker(rt, act, layers, B * S, args.ln_fold)
    rt.check()
    sched, res = make_schedule(x_in, None)
    stream = torch.cuda.Stream(device=local)
    rt.activate(stream)

    def enqueue():
        for kind, fn in sched:
            rc = fn()
            if rc:
                raise RuntimeError(f"{kind} returned {rc}")

    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            enqueue()
    stream.synchronize()
    rt.check()

    # ---- per-kernel breakdown: CUDA events around every launch of 2 eager steps --------------------------------
    if args.debug:
        log("library stream", lib.sh_cuda_get_stream(), "bench stream", stream.cuda_stream)
    kinds = [k for k, _ in sched]
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(sched) + 1)]
    per_kind: dict[str, list[float]] = {}
    with torch.cuda.stream(stream):
        for _ in range(2):
            evs[0].record(stream)
            for i, (_, fn) in enumerate(sched):
                fn()
                evs[i + 1].record(stream)
            stream.synchronize()
            for i, k in enumerate(kinds):
                per_kind.setdefault(k, []).append(evs[i].elapsed_time(evs[i + 1]))
    rt.check()
    if args.debug:
        log("breakdown ms per kind:", {k: round(sum(v), 3) for k, v in per_kind.items()})

    # ---- CUDA graph of one step ------------------------------------------------------------------------------------
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            lib.sh_cuda_set_stream(torch.cuda.current_stream().cuda_stream)
            enqueue()
        lib.sh_cuda_set_stream(stream.cuda_stream)

    def step():
        with torch.cuda.stream(stream):   # graph replays and eager launches both go to `stream`
            if graph is not None:
                graph.replay()
            else:
                enqueue()

    for _ in range(max(3, args.warmup)):
        step()
    stream.synchronize()
    rt.check()

    # ---- timed region: inputs resident in HBM --------------------------------------------------------------------------
    clocks = ClockSampler(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    clocks.mark()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    clock_info = clocks.stop()
    barrier(world)
    ms, value = job_rate(e0.elapsed_time(e1), args.steps, world)
    rt.check()

    # ---- e2e: host input -> device -> encoder -> host output every step ----------------------------------------------
    # Every step copies its input batch from pinned host memory and its result back. The copies of neighbouring
    # steps overlap the encoder (H2D of step k+1 and D2H of step k-1 run on their own streams while step k computes),
    # with two device input / output slots and one captured graph per slot; the timed region spans all copies.
    host_in = torch.empty((M, D), dtype=torch.float16, pin_memory=True)
    host_out = torch.empty((M, D), dtype=torch.float16, pin_memory=True)
    host_in.copy_(rt.view(x_in, M, D).cpu())
    slots_in = [x_in, rt.alloc(M, D)]
    slots_out = [rt.alloc(M, D), rt.alloc(M, D)]
    slot_step = []
    for sl in range(2):
        sched_s, _ = make_schedule(slots_in[sl], slots_out[sl])

        def enqueue_s(sched_s=sched_s):
            for kind, fn in sched_s:
                rc = fn()
                if rc:
                    raise RuntimeError(f"{kind} returned {rc}")
        if graph is not None:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                lib.sh_cuda_set_stream(torch.cuda.current_stream().cuda_stream)
                enqueue_s()
            lib.sh_cuda_set_stream(stream.cuda_stream)
            slot_step.append((g, g.replay))
        else:
            slot_step.append((None, enqueue_s))
    h2d, d2h = torch.cuda.Stream(device=local), torch.cuda.Stream(device=local)
    e2e_steps = args.steps                   # the same step count as the device-resident leg
    in_ready = [torch.cuda.Event(), torch.cuda.Event()]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    out_read = [torch.cuda.Event(), torch.cuda.Event()]

    def e2e_run(n):
        h2d.wait_stream(stream)                  # copies start inside the timed region
        d2h.wait_stream(stream)
        for k in range(n):
            sl = k % 2
            dev_in, dev_out = rt.view(slots_in[sl], M, D), rt.view(slots_out[sl], M, D)
            if k >= 2:
                h2d.wait_event(done[sl])            # step k-2 has consumed this input slot
            with torch.cuda.stream(h2d):
                dev_in.copy_(host_in, non_blocking=True)
                in_ready[sl].record(h2d)
            stream.wait_event(in_ready[sl])
            if k >= 2:
                stream.wait_event(out_read[sl])     # step k-2's result has left this output slot
            with torch.cuda.stream(stream):
                slot_step[sl][1]()
                done[sl].record(stream)
            d2h.wait_event(done[sl])
            with torch.cuda.stream(d2h):
                host_out.copy_(dev_out, non_blocking=True)
                out_read[sl].record(d2h)
        stream.wait_stream(d2h)

    e2e_run(2)                                   # warm the copy paths
    stream.synchronize()

    def timed(fn) -> float:
        """ms of one timed region of K steps (barrier + synchronize on both sides, max over ranks)"""
        barrier(world)
        torch.cuda.synchronize()
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        barrier(world)
        return max_over_ranks(e0.elapsed_time(e1), world)

    def steps_resident():
        for _ in range(args.steps):
            step()

    e2e_ms = timed(lambda: e2e_run(e2e_steps))
    e2e_value = GLOBAL_BATCH * e2e_steps / (e2e_ms / 1e3)
    # two more regions of each leg, alternating, so that both legs are compared at the same clocks
    rep_value, rep_e2e = [ms], [e2e_ms]
    for _ in range(2):
        rep_value.append(timed(steps_resident))
        rep_e2e.append(timed(lambda: e2e_run(e2e_steps)))
    rt.check()
    step()                                       # the device-resident step on the same input batch ...
    stream.synchronize()
    if not torch.equal(host_out, rt.view(res, M, D).cpu()):   # ... must give the same encoder output
        raise RuntimeError("end-to-end output differs from the device-resident run")
    del slot_step

    # ---- roofline of the dominant kernel and the per-kernel table -------------------------------------------------------
    pk, src = peaks()
    kernels = {}
    for k, times in per_kind.items():
        n_per_step = kinds.count(k)
        t_launch = sum(times) / len(times) * 1e-3   # s per launch (one entry per launch)
        flops, nbytes = encoder.op_work(k, B, S, D, F, H)
        kernels[k] = {"launches_per_step": n_per_step, "ms_per_launch": round(t_launch * 1e3, 4),
                      "tflops": round(flops / t_launch / 1e12, 1), "gbs": round(nbytes / t_launch / 1e9, 1)}
    gemm_kinds = [k for k in kernels if k.startswith("gemm")]
    gemm_flops = sum(encoder.op_work(k, B, S, D, F, H)[0] * kernels[k]["launches_per_step"] for k in gemm_kinds)
    gemm_time = sum(kernels[k]["ms_per_launch"] * 1e-3 * kernels[k]["launches_per_step"] for k in gemm_kinds)
    gemm_all = gemm_flops / gemm_time / 1e12
    # the roofline line describes the single largest launch: the FC1 GEMM (131072 x 3072 x 768 at B = 512 on one GPU)
    fc1 = kernels["gemm_fc1"]
    fc1_flops = encoder.op_work("gemm_fc1", B, S, D, F, H)[0]
    achieved = fc1_flops / (fc1["ms_per_launch"] * 1e-3) / 1e12
    peak = pk.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    traffic = profile_traffic(f"gemm_fc1_m{B * S}") if world == 1 else None
    roofline = {"kernel": f"k_gemm_tc2 (tcgen05 2-CTA GEMM) on FC1 {B * S}x{F}x{D}, bias + GELU epilogue",
                "bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 3), "peak_source": f"{src} bf16 sustained (kernel timed inside a long step)",
                "flops_per_launch": round(fc1_flops), "traffic": traffic,
                "algorithmic_bytes_per_launch": round(encoder.op_work("gemm_fc1", B, S, D, F, H)[1])}
    ln = kernels.get("layernorm")
    hbm = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    attn = kernels.get("attention")
    out = {
        "metric": "encoder images/s", "value": round(value, 1), "unit": "images/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded LCG: x N(0,1), weights N(0,0.02), zero biases, gamma 1, beta 0)",
        "config": {"workload": "SigLIP-base 12-layer encoder forward (BASELINE config 5)", "global_batch": GLOBAL_BATCH,
                   "per_gpu_batch": B, "seq_len": S, "d_model": D, "ffn": F, "heads": H, "layers": NLAYERS,
                   "parallelism": f"dp{world}", "cuda_graph": graph is not None, "ln_fold": args.ln_fold,
                   "l2": "inputs larger than L2 (201 MB per activation tensor at B=512), no flush"},
        "e2e": {"value": round(e2e_value, 1), "unit": "images/s", "h2d_bytes_per_step": M * D * 2,
                "d2h_bytes_per_step": M * D * 2, "steps": e2e_steps},
        "repeats": {"what": "value / e2e legs timed three times each (alternating, K steps per region); value and "
                            "e2e above are the first region of each",
                    "value_images_per_s": [round(GLOBAL_BATCH * args.steps / (t / 1e3), 1) for t in rep_value],
                    "e2e_images_per_s": [round(GLOBAL_BATCH * e2e_steps / (t / 1e3), 1) for t in rep_e2e],
                    "median_value": round(GLOBAL_BATCH * args.steps / (statistics.median(rep_value) / 1e3), 1),
                    "median_e2e": round(GLOBAL_BATCH * e2e_steps / (statistics.median(rep_e2e) / 1e3), 1)},
        "gpu_launches": args.steps * len(sched),
        "roofline": roofline,
        "kernels": kernels,
        "gemm_tflops": round(gemm_all, 1),   # all four GEMMs of a layer together
        "attention_tflops": attn["tflops"] if attn else None,
        "rowop_gbs": ln["gbs"] if ln else None,
        "rowop_frac_hbm": round(ln["gbs"] / hbm, 3) if ln else None,
        "clocks": clock_info,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args.cpu_images)
    if world > 1:
        import torch.distributed as dist
        del graph
        dist.destroy_process_group()
    return out if rank == 0 else None


# ---- the CPU leg: the reference's numpy layer (oracle port) ------------------------------------------------------------
def host_blas() -> str:
    """The BLAS numpy runs the CPU baselines on (name, version and build configuration)."""
    try:
        import numpy as np
        b = np.__config__.CONFIG["Build Dependencies"]["blas"]
        return f"{b.get('name', '?')} {b.get('version', '?')} ({b.get('openblas configuration', '').strip()})"
    except Exception:   # a numpy without the build-config table
        return "unknown"


def cpu_layer_setup(seed: int = 3):
    import numpy as np
    from oracle import lcg, siglip
    x = lcg.normal_fp16(S, D, seed)
    p = siglip.baseline_layer_params(D, F, 1)
    return np, siglip, x, p


def cpu_baseline(images: int) -> dict:
    np, siglip, x, p = cpu_layer_setup()
    siglip.layer_reference_arrays(x, p, H)          # warm BLAS
    t0 = time.perf_counter()
    for _ in range(images):
        cur = x
        for _ in range(NLAYERS):
            cur = siglip.layer_reference_arrays(cur, p, H)["OUT"]
    dt = time.perf_counter() - t0
    return {"value": round(images / dt, 4), "unit": "images/s", "cores": os.cpu_count(), "blas": host_blas(), "kind": "port",
            "sample": f"{images} image(s) x {NLAYERS} layers (S={S}, D={D}) of the 512-image batch through the numpy "
                      f"oracle of siglip_ref.layer_reference (fp32 BLAS, all host threads); {dt:.1f} s"}


def run_reference(args, rank: int, world: int) -> dict | None:
    if rank != 0:
        return None
    np, siglip, x, p = cpu_layer_setup()
    for _ in range(max(0, args.warmup)):
        siglip.layer_reference_arrays(x, p, H)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        siglip.layer_reference_arrays(x, p, H)
        times.append(time.perf_counter() - t0)
    t_layer = statistics.mean(times)
    value = 1.0 / (NLAYERS * t_layer)
    sample = (f"each step: 1 image through 1 of the {NLAYERS} layers (numpy fp32 oracle of siglip_ref, all host "
              f"threads); images/s = 1 / ({NLAYERS} x mean layer time)")
    return {"metric": "encoder images/s", "value": round(value, 4), "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_layer * 1e3, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded LCG)", "impl": "reference",
            "config": {"workload": "SigLIP-base 12-layer encoder forward (BASELINE config 5)",
                       "global_batch": GLOBAL_BATCH, "seq_len": S, "parallelism": "cpu"},
            "cpu_baseline": {"value": round(value, 4), "unit": "images/s", "cores": os.cpu_count(), "blas": host_blas(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---- secondary workloads (BASELINE configs 1 and 2): their own JSON lines, not the headline ------------------------
def _event_time(torch, stream, fn, steps: int) -> float:
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


def run_gemm512(args, local: int) -> dict:
    """Config 1: Z = X W, 512^3, X / W uniform [-1, 1) from the LCG. Per-call latency (eager) and throughput of
    1000 back-to-back calls replayed from a CUDA graph."""
    import torch
    from softhier_cuda import lib as L
    from softhier_cuda.runtime import Runtime
    rt = Runtime.open(local, arena_bytes=64 << 20)
    lib = rt.lib
    n = 512
    x, w, z = rt.alloc(n, n), rt.alloc(n, n), rt.alloc(n, n)
    lib.sh_test_fill_fp16(x, n, n, n, 1, -1024, 1023, 1.0 / 1024)
    lib.sh_test_fill_fp16(w, n, n, n, 2, -1024, 1023, 1.0 / 1024)
    stream = torch.cuda.Stream(device=local)
    rt.activate(stream)
    call = lambda: lib.sh_gemm(x, w, z, n, n, n, n, n, n, None, L.SH_ALL)  # noqa: E731
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            call()
    rt.check()
    with torch.cuda.stream(stream):
        lat = _event_time(torch, stream, call, max(10, args.steps))
    g = torch.cuda.CUDAGraph()
    reps = 1000
    with torch.cuda.graph(g, stream=stream):
        lib.sh_cuda_set_stream(torch.cuda.current_stream().cuda_stream)
        for _ in range(reps):
            call()
    lib.sh_cuda_set_stream(stream.cuda_stream)
    with torch.cuda.stream(stream):
        g.replay()
        thr = _event_time(torch, stream, g.replay, 3) / reps
    rt.check()
    flop = 2.0 * n ** 3
    pk, src = peaks()
    return {"metric": "GEMM 512^3 TFLOP/s", "value": round(flop / thr / 1e9, 2), "unit": "TFLOP/s", "n_gpus": 1,
            "ms_per_call_graph": round(thr, 5), "ms_per_call_eager": round(lat, 5),
            "latency_tflops": round(flop / lat / 1e9, 2), "frac_of_peak": round(flop / thr / 1e9 / pk["bf16_tflops"], 4),
            "peak": f"{src} bf16 burst {pk['bf16_tflops']} TFLOP/s", "higher_is_better": True, "dtype": "f16",
            "config": {"workload": "BASELINE config 1: 512^3 fp16 GEMM, fp32 accumulate",
                       "note": "X, W, Z = 1.5 MB: L2-resident; 1000 calls per graph replay"}}


def run_gemm(args, local: int) -> dict:
    """One encoder-shaped GEMM with its fused epilogue (`--gemm M,N,K`, `--epi bias,gelu,residual`), eager launches
    on one stream: the per-kernel line behind the roofline, and the small case the ncu captures run. X / W / residual
    N(0, 1) / N(0, 0.02) / N(0, 1) from the device fill; Z alone is larger than L2 at the default shape."""
    import torch
    from softhier_cuda import lib as L
    from softhier_cuda.runtime import Runtime
    M, N, K = (int(v) for v in args.gemm.split(","))
    flags = 0
    for e in filter(None, args.epi.split(",")):
        flags |= {"bias": L.EPI_BIAS, "gelu": L.EPI_GELU, "residual": L.EPI_RESIDUAL}[e]
    rt = Runtime.open(local, arena_bytes=(2 * (M * K + K * N + 2 * M * N + N) + (64 << 20)))
    lib = rt.lib
    x, w, z, r, b = rt.alloc(M, K), rt.alloc(K, N), rt.alloc(M, N), rt.alloc(M, N), rt.alloc(1, N)
    for i, (p, rows, cols, sd) in enumerate(((x, M, K, 1.0), (w, K, N, 0.02), (r, M, N, 1.0), (b, 1, N, 0.1))):
        lib.sh_cuda_fill_normal_fp16(p, rows, cols, cols, i + 1, 0.0, sd)
    stream = torch.cuda.Stream(device=local)
    rt.activate(stream)
    call = lambda: lib.sh_cuda_gemm(x, w, z, M, N, K, K, N, N, b, r, N, flags, 0)  # noqa: E731
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            if call():
                raise RuntimeError(lib.sh_cuda_last_error_string().decode())
        rt.check()
        clocks = ClockSampler(local)
        clocks.start()
        torch.cuda.synchronize()
        clocks.mark()
        ms = _event_time(torch, stream, call, max(1, args.steps))
        clock_info = clocks.stop()
    rt.check()
    flop = 2.0 * M * N * K
    pk, src = peaks()
    tf = flop / ms / 1e9
    # tensor work per SM clock: 8192 fp16 FLOP / clk / SM is the dense tcgen05 rate
    per_clk = (tf * 1e12 / (torch.cuda.get_device_properties(local).multi_processor_count * clock_info["sm_mhz"] * 1e6)
               if clock_info.get("sm_mhz") else None)
    out = {"metric": "GEMM TFLOP/s", "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": "f16",
           "frac_of_peak": round(tf / pk["bf16_tflops"], 4), "peak": f"{src} bf16 burst {pk['bf16_tflops']} TFLOP/s",
           "clocks": clock_info, "frac_of_clock_peak": round(per_clk / 8192, 4) if per_clk else None,
           "config": {"workload": f"sh_cuda_gemm {M}x{N}x{K} epilogue [{args.epi}]",
                      "l2": "Z alone larger than L2 at the default shape; no flush"}}
    if args.vs_cublas:
        out["vs_cublas"] = _vs_cublas(torch, stream, call, M, N, K, max(1, args.steps))
        rt.check()
    return out


def _vs_cublas(torch, stream, call, M: int, N: int, K: int, steps: int, reps: int = 3) -> dict:
    """Library comparison on the same shape: torch.matmul (cuBLAS) fp16 with the same operand distributions,
    timed the same way, alternating with this library's call so both see the same clocks. cuBLAS has no fused
    epilogue: compare against `--epi ""`."""
    a = torch.randn(M, K, device=stream.device, dtype=torch.float16)
    b = torch.randn(K, N, device=stream.device, dtype=torch.float16) * 0.02
    c = torch.empty(M, N, device=stream.device, dtype=torch.float16)
    cub = lambda: torch.matmul(a, b, out=c)  # noqa: E731
    ours, theirs = [], []
    with torch.cuda.stream(stream):
        for _ in range(3):
            cub()
        for _ in range(reps):
            ours.append(_event_time(torch, stream, call, steps))
            theirs.append(_event_time(torch, stream, cub, steps))
    flop = 2.0 * M * N * K
    med = lambda v: sorted(v)[len(v) // 2]  # noqa: E731
    return {"ours_tflops": round(flop / med(ours) / 1e9, 1), "cublas_tflops": round(flop / med(theirs) / 1e9, 1),
            "ratio": round(med(theirs) / med(ours), 3), "reps": reps, "statistic": "median of alternating reps"}


def run_attention(args, local: int) -> dict:
    """The encoder's attention launch alone (`--attn B,S,H`, dh = 64, packed q|k|v with ld 3 D as the encoder stores
    them): per-launch time and TFLOP/s (4 B S^2 D). q, k, v N(0, 1); the output is larger than L2 at B = 512."""
    import torch
    from softhier_cuda.runtime import Runtime
    B, S, H = (int(v) for v in args.attn.split(","))
    D = 64 * H
    M = B * S
    rt = Runtime.open(local, arena_bytes=2 * (M * 3 * D + M * D) + (64 << 20))
    lib = rt.lib
    qkv, o = rt.alloc(M, 3 * D), rt.alloc(M, D)
    lib.sh_cuda_fill_normal_fp16(qkv, M, 3 * D, 3 * D, 7, 0.0, 1.0)
    stream = torch.cuda.Stream(device=local)
    rt.activate(stream)
    call = lambda: lib.sh_cuda_attention_batched(qkv, qkv + 2 * D, qkv + 4 * D, o, S, D, H, 3 * D, 3 * D, 3 * D, D,  # noqa: E731
                                                 0.125, B)
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            if call():
                raise RuntimeError(lib.sh_cuda_last_error_string().decode())
        rt.check()
        ms = _event_time(torch, stream, call, max(1, args.steps))
    rt.check()
    flop = 4.0 * B * S * S * D
    pk, src = peaks()
    tf = flop / ms / 1e9
    return {"metric": "attention TFLOP/s", "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": "f16",
            "frac_of_peak": round(tf / pk["bf16_tflops"], 4), "peak": f"{src} bf16 burst {pk['bf16_tflops']} TFLOP/s",
            "exp_per_s": round(B * H * S * S / (ms * 1e-3) / 1e12, 3),
            "config": {"workload": f"sh_cuda_attention_batched B={B} S={S} H={H} dh=64 (packed qkv, ld {3 * D})"}}


def run_layer(args, local: int) -> dict:
    """Config 3: one SigLIP-base layer on one sequence (B = 1, S = 256), the 7 library calls replayed from a CUDA
    graph; per-layer latency and TFLOP/s (3,825,205,248 FLOP per layer). Weights N(0, 0.02), zero biases, gamma 1,
    beta 0, x N(0, 1), from the device fills. The 3.5 MB of activations stay in L2 between replays, as they would
    between the layers of a B = 1 encoder."""
    import torch
    from softhier_cuda import encoder
    from softhier_cuda.runtime import Runtime
    rt = Runtime.open(local, arena_bytes=96 << 20)
    lib = rt.lib
    layers, act, x_in = setup_encoder(rt, 1, 100, nlayers=1)
    sched, _ = schedule_maker(rt, act, layers, S, args.ln_fold)(x_in, None)
    stream = torch.cuda.Stream(device=local)
    rt.activate(stream)

    def enqueue():
        for kind, fn in sched:
            if fn():
                raise RuntimeError(f"{kind} failed: {lib.sh_cuda_last_error_string().decode()}")
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            enqueue()
        eager = _event_time(torch, stream, enqueue, max(10, args.steps))
    rt.check()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        lib.sh_cuda_set_stream(torch.cuda.current_stream().cuda_stream)
        enqueue()
    lib.sh_cuda_set_stream(stream.cuda_stream)
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
        ms = _event_time(torch, stream, graph.replay, max(100, args.steps))
    rt.check()
    flop = 2.0 * (4 * S * D * D + 2 * S * D * F + 2 * S * S * D)
    pk, src = peaks()
    return {"metric": "encoder layer latency (B=1)", "value": round(ms * 1e3, 2), "unit": "us", "n_gpus": 1,
            "higher_is_better": False, "steps": max(100, args.steps), "warmup": max(3, args.warmup),
            "ms_per_step": round(ms, 4), "eager_us": round(eager * 1e3, 2), "tflops": round(flop / ms / 1e9, 1),
            "frac_of_peak": round(flop / ms / 1e9 / pk["bf16_tflops"], 4),
            "peak": f"{src} bf16 burst {pk['bf16_tflops']} TFLOP/s", "dtype": "f16", "launches": len(sched),
            "reference_gvsoc_ms_per_layer": 1.920,
            "config": {"workload": "BASELINE config 3: one SigLIP-base layer, B=1, S=256, D=768, 12 heads, FFN 3072",
                       "cuda_graph": True, "ln_fold": args.ln_fold}}


def run_rowops(args, local: int) -> dict:
    """Config 2 at the HBM-resident activation shape of config 5 (131072 rows x 768 / 3072): per-op GB/s, rotating
    over buffers that total more than twice the L2 so every launch streams from HBM."""
    import torch
    from softhier_cuda import lib as L
    from softhier_cuda.runtime import Runtime
    rows = 131072
    widths = tuple(int(c) for c in args.rowops_cols.split(","))
    rt = Runtime.open(local, arena_bytes=6 * rows * max(widths) * 2 + (64 << 20))
    lib = rt.lib
    stream = torch.cuda.Stream(device=local)
    out = {}
    pk, src = peaks()
    for cols in widths:
        rt.reset()
        nbuf = 2
        xs = [rt.alloc(rows, cols) for _ in range(nbuf)]
        bs = [rt.alloc(rows, cols) for _ in range(nbuf)]
        ys = [rt.alloc(rows, cols) for _ in range(nbuf)]
        g, be = rt.alloc(1, cols), rt.alloc(1, cols)
        for i in range(nbuf):
            lib.sh_cuda_fill_normal_fp16(xs[i], rows, cols, cols, 11 + i, 0.0, 1.0)
            lib.sh_cuda_fill_normal_fp16(bs[i], rows, cols, cols, 21 + i, 0.0, 1.0)
        lib.sh_cuda_fill_normal_fp16(g, 1, cols, cols, 13, 1.0, 0.02)
        lib.sh_cuda_fill_normal_fp16(be, 1, cols, cols, 14, 0.0, 0.02)
        rt.activate(stream)
        A = L.SH_ALL
        it = {"i": 0}

        def nxt():
            it["i"] = (it["i"] + 1) % nbuf
            return it["i"]
        ops = {
            "layernorm": (lambda i: lib.sh_layernorm(ys[i], xs[i], g, be, rows, cols, cols, 1e-6, A), 2 * rows * cols * 2),
            "softmax": (lambda i: lib.sh_softmax_rows(ys[i], xs[i], rows, cols, cols, 0.125, A), 2 * rows * cols * 2),
            "gelu": (lambda i: lib.sh_gelu(ys[i], xs[i], rows, cols, cols, A), 2 * rows * cols * 2),
            "add": (lambda i: lib.sh_add(ys[i], xs[i], bs[i], rows, cols, cols, A), 3 * rows * cols * 2),
            "add_bias": (lambda i: lib.sh_add_bias(ys[i], xs[i], be, rows, cols, cols, A), 2 * rows * cols * 2),
            "scale": (lambda i: lib.sh_scale(ys[i], xs[i], rows, cols, cols, 0.125, A), 2 * rows * cols * 2),
            "transpose": (lambda i: lib.sh_transpose(ys[i], xs[i], rows, cols, cols, rows, A), 2 * rows * cols * 2),
        }
        with torch.cuda.stream(stream):
            for name, (fn, nbytes) in ops.items():
                for _ in range(3):
                    fn(nxt())
                ms = _event_time(torch, stream, lambda: fn(nxt()), max(10, args.steps))
                out[f"{name}_{rows}x{cols}"] = {"ms": round(ms, 4), "gbs": round(nbytes / ms / 1e6, 1),
                                                "frac_hbm": round(nbytes / ms / 1e6 / pk["hbm_gbs"], 3)}
        rt.check()
    worst = min(v["frac_hbm"] for v in out.values())
    return {"metric": "row-op GB/s (HBM-resident)", "value": round(min(v["gbs"] for v in out.values()), 1),
            "unit": "GB/s (slowest op)", "n_gpus": 1, "higher_is_better": True, "dtype": "f16", "ops": out,
            "min_frac_hbm": worst, "peak": f"{src} copy {pk['hbm_gbs']} GB/s",
            "small": _rowops_small(torch, rt, stream) if not args.no_small else None,
            "config": {"workload": "BASELINE config 2 ops at 131072 x {768, 3072}; 'small': the 256-row shapes",
                       "l2": "2 rotating buffer sets of 201 / 805 MB per operand (> 2 x L2)"}}


# Simulated times of the reference's row ops at 256 x 768 on all 16 clusters, GVSoC at 1 GHz, ms
# (docs/SIMULATOR_NOTES.md:184-192 of the reference)
REF_GVSOC_ROWOPS_MS = {"layernorm": 0.149, "softmax": 0.145, "gelu": 0.123, "add": 0.022, "add_bias": 0.027,
                       "scale": 0.017, "transpose": 0.025}


def _rowops_small(torch, rt, stream, reps: int = 1000) -> dict:
    """Config 2 at its own shapes (256 x 768 and 256 x 3072, L2-resident): microseconds per call, from 1000
    back-to-back calls replayed from a CUDA graph, beside the reference's simulated time where it has one."""
    from softhier_cuda import lib as L
    lib, A, rows = rt.lib, L.SH_ALL, 256
    res = {}
    for cols in (768, 3072):
        rt.reset()
        x, b, y = rt.alloc(rows, cols), rt.alloc(rows, cols), rt.alloc(rows, cols)
        g, be = rt.alloc(1, cols), rt.alloc(1, cols)
        for i, (p, r, sd, mu) in enumerate(((x, rows, 1.0, 0.0), (b, rows, 1.0, 0.0), (g, 1, 0.02, 1.0),
                                            (be, 1, 0.02, 0.0))):
            lib.sh_cuda_fill_normal_fp16(p, r, cols, cols, 31 + i, mu, sd)
        ops = {
            "layernorm": lambda: lib.sh_layernorm(y, x, g, be, rows, cols, cols, 1e-6, A),
            "softmax": lambda: lib.sh_softmax_rows(y, x, rows, cols, cols, 0.125, A),
            "gelu": lambda: lib.sh_gelu(y, x, rows, cols, cols, A),
            "add": lambda: lib.sh_add(y, x, b, rows, cols, cols, A),
            "add_bias": lambda: lib.sh_add_bias(y, x, be, rows, cols, cols, A),
            "scale": lambda: lib.sh_scale(y, x, rows, cols, cols, 0.125, A),
            "transpose": lambda: lib.sh_transpose(y, x, rows, cols, cols, rows, A),
        }
        rt.activate(stream)
        for name, fn in ops.items():
            with torch.cuda.stream(stream):
                for _ in range(3):
                    fn()
            g_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_, stream=stream):
                lib.sh_cuda_set_stream(torch.cuda.current_stream().cuda_stream)
                for _ in range(reps):
                    fn()
            lib.sh_cuda_set_stream(stream.cuda_stream)
            with torch.cuda.stream(stream):
                g_.replay()
                ms = _event_time(torch, stream, g_.replay, 3) / reps
            del g_
            ent = {"us": round(ms * 1e3, 3)}
            if cols == 768 and name in REF_GVSOC_ROWOPS_MS:
                ent["reference_gvsoc_us"] = REF_GVSOC_ROWOPS_MS[name] * 1e3
            res[f"{name}_{rows}x{cols}"] = ent
        rt.check()
    return res


def run_summa(args, rank: int, world: int, local: int) -> dict | None:
    """Config 4: C = A B, M = N = K = 16384, A / B uniform [-1, 1) from the LCG, block-distributed over the default
    grid of the world size (1x1, 1x2, 2x2, 2x4). One K-panel per step is pulled from its owners over NVLink by the
    copy engines while the tcgen05 GEMM of the previous step runs; every timed step does one full set of pulls and
    one GEMM. value = 2 n^3 / (max over ranks of the step time)."""
    import torch
    from softhier_cuda import summa as SU
    from softhier_cuda.runtime import Runtime
    init_dist(world, local)
    torch.cuda.set_device(local)
    n = args.summa_n
    pr, pc = SU.default_grid(world)
    kb = SU.default_panel(n, world)   # one panel per step: no fp32 carry; pulled during the previous step
    lay = SU.Layout(n, n, n, pr, pc, kb)
    rt = Runtime.open(local, arena_bytes=64 << 20)
    if world > 1:
        import torch.distributed as dist

        def exchange(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out
        bar = dist.barrier
    else:
        exchange, bar = (lambda x: [x]), (lambda: None)
    compute, copy = torch.cuda.Stream(device=local), torch.cuda.Stream(device=local)
    su = SU.SummaGPU(rt.lib, lay, rank, exchange, bar, (compute, copy))
    su.fill_inputs(41, 42)
    for _ in range(max(3, args.warmup)):
        assert su.step(torch, prefetch_next=True) == 0
    torch.cuda.synchronize()
    rt.check()
    clocks = ClockSampler(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    clocks.mark()
    steps = args.steps
    e0.record(compute)
    for _ in range(steps):         # each step also pulls the next step's first panel (the last one's ends in e1)
        su.step(torch, prefetch_next=True)
    su.finish(torch)
    e1.record(compute)
    e1.synchronize()
    clock_info = clocks.stop()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    rt.check()
    # one-shot C = A B: a call whose panel pull was not started by an earlier step (the pull and the GEMM in series),
    # after one un-timed step that consumes the timed loop's prefetch
    assert su.step(torch, prefetch_next=False) == 0
    torch.cuda.synchronize()
    one_shot = []
    for _ in range(3):
        barrier(world)
        torch.cuda.synchronize()
        e0.record(compute)
        assert su.step(torch, prefetch_next=False) == 0
        e1.record(compute)
        e1.synchronize()
        one_shot.append(e0.elapsed_time(e1))
    barrier(world)
    one_shot_ms = max_over_ranks(statistics.median(one_shot), world)
    rt.check()
    su.close()
    flop = 2.0 * n ** 3
    pk, src = peaks()
    tf = flop / ms / 1e9
    peer_bytes = SU.panel_peer_bytes(lay, rank)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return None
    extra = {}
    if world == 1 and not args.no_cpu_baseline:
        extra["cpu_baseline"] = summa_cpu_baseline(n)
    return {**extra, "metric": "SUMMA 16384^3 TFLOP/s", "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "strong", "dtype": "f16", "frac_of_peak_per_gpu": round(tf / world / pk["bf16_tflops_sustained"], 3),
            "peak": f"{src} bf16 sustained {pk['bf16_tflops_sustained']} TFLOP/s per GPU",
            "peer_bytes_per_step_rank0": peer_bytes, "clocks": clock_info,
            "one_shot": {"ms": round(one_shot_ms, 3), "tflops": round(flop / one_shot_ms / 1e9, 1),
                         "what": "one C = A B whose panel pulls start with it (no overlap with an earlier step), "
                                 "median of 3, max over ranks"},
            "config": {"workload": "BASELINE config 4: distributed SUMMA", "n": n, "grid": f"{pr}x{pc}", "panel": kb,
                       "transport": "CUDA IPC + copy engines (cudaMemcpy2DAsync) over NVLink"}}


def summa_cpu_baseline(n: int, sample: int = 4096) -> dict:
    """Config 4 on the host: the reference's host check of a GEMM is an fp32 numpy matmul; one sample^3 product
    with all BLAS threads, scaled to the n^3 FLOP of the full problem (TFLOP/s is size-independent enough at
    4096^3 for a baseline)."""
    import numpy as np
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (sample, sample)).astype(np.float32)
    b = rng.uniform(-1, 1, (sample, sample)).astype(np.float32)
    a @ b
    t0 = time.perf_counter()
    a @ b
    dt = time.perf_counter() - t0
    tf = 2.0 * sample ** 3 / dt / 1e12
    return {"value": round(tf, 4), "unit": "TFLOP/s", "cores": os.cpu_count(), "blas": host_blas(), "kind": "port",
            "sample": f"one fp32 {sample}^3 numpy matmul ({dt:.2f} s); the {n}^3 product at that rate would take "
                      f"{2.0 * n ** 3 / tf / 1e12:.0f} s"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--ln-fold", choices=["none", "ln1", "both"], default="none",
                    help="LayerNorms folded into the GEMMs that consume them: none, LN1 into QKV, or both")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-images", type=int, default=2)
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--workload", choices=["encoder", "layer", "gemm512", "gemm", "attention", "rowops", "summa"],
                    default="encoder")
    ap.add_argument("--attn", default="512,256,12", help="B,S,H of --workload attention")
    ap.add_argument("--gemm", default="131072,3072,768", help="M,N,K of --workload gemm")
    ap.add_argument("--epi", default="bias,gelu", help="fused epilogue of --workload gemm: bias,gelu,residual")
    ap.add_argument("--summa-n", type=int, default=16384)
    ap.add_argument("--rowops-cols", default="768,3072", help="row widths of --workload rowops (131072 rows each)")
    ap.add_argument("--no-small", action="store_true", help="--workload rowops: skip the 256-row graph timings")
    ap.add_argument("--vs-cublas", action="store_true", help="--workload gemm: also time torch.matmul on the shape")
    args = ap.parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        out = run_reference(args, rank, world)
    elif args.workload == "gemm512":
        out = run_gemm512(args, local) if rank == 0 else None
    elif args.workload == "gemm":
        out = run_gemm(args, local) if rank == 0 else None
    elif args.workload == "layer":
        out = run_layer(args, local) if rank == 0 else None
    elif args.workload == "attention":
        out = run_attention(args, local) if rank == 0 else None
    elif args.workload == "rowops":
        out = run_rowops(args, local) if rank == 0 else None
    elif args.workload == "summa":
        out = run_summa(args, rank, world, local)
    else:
        out = run_ours(args, rank, world, local)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
