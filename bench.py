#!/usr/bin/env python
"""Benchmark of the B200 MACE energy + forces step (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (the headline): medium MACE
(128x0e + 128x1o, lmax 3, correlation 3, 2 layers, r_max 6 A, 8 Bessel,
radial MLP [64,64,64]) with seeded random-init weights (seed 1), on diamond Si
5x5x5 = 1000 atoms rattled by 0.05 A (seed 1); energy + forces per step.  The
neighbour list is the calculator's cached one (cutoff r_max + 0.5 A skin), as in
the reference's own MD timing.  All data are synthetic.

One JSON line (rank 0).  ``value`` is device-timed with CUDA events, inputs
resident in HBM, L2 flushed between timed steps; ``e2e`` is the same metric
through the public calculator API (host positions in, host forces out);
``roofline`` is the dominant kernel's algorithmic work over its event-timed
launch duration; ``cpu_baseline`` times the CPU oracle port on this host.

With N > 1 (torchrun), the ranks evaluate ONE periodic diamond-Si structure
of N Si1000 blocks (5x5x5 conventional cells per rank), spatially decomposed
on the domain grid 1x1x2 / 1x2x2 / 2x2x2: each rank owns one block, holds
r_max + skin ghost shells, computes its owned atoms' edges only, and the
layer-1 input features of the ghosts and their gradients cross the ranks
inside the step (the library's NCCL halo exchange), with ghost positions
and forces moved per step: weak scaling with the halo exchange on the data
path.

``--impl reference`` times the reference algorithm's CPU restatement (the
reference itself runs on MLX/Metal, absent here) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "energy+forces atom-steps/s, medium-MACE Si1000 fp32"
UNIT = "atom-steps/s"
AVG_NUM_NEIGHBORS = 44.0
WORKLOAD = ("config1: medium MACE (128x0e+128x1o, lmax3, corr3, 2 layers, r_max 6.0) random-init seed 1; "
            "diamond Si 5x5x5 = 1000 atoms rattled 0.05 A (seed 1); energy+forces; cached NL r_max+0.5 skin")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=20.0, help="budget of the CPU baseline sample")
    ap.add_argument("--device-only", action="store_true",
                    help="only W + K plain device steps, no JSON (the command the ncu captures profile)")
    ap.add_argument("--timeline", action="store_true",
                    help="also print (to stderr) the per-launch timeline of one graph-replayed step, from the event "
                         "records the profiler places in the graph: stream, start and end of every launch")
    ap.add_argument("--config", default="c1", choices=["c0", "c1", "c2", "c3", "c4"],
                    help="c1: the headline Si1000 (default); c0: small-arch Si216 with stress; c2: large-arch "
                         "LiPSO-8000 with stress; c3: 512 OFF-like molecules sharded by structure; "
                         "c4: 1M-atom Si, spatially domain-decomposed over the ranks")
    return ap.parse_args()


SINGLE = {
    # name: (arch, seed, z_table, avg_num_neighbors, stress, workload text)
    "c0": ("small", 0, list(range(1, 90)), 46.0, True,
           "config0: small MACE (128x0e, lmax3, corr3, 2 layers, r_max 6.0) random-init seed 0; diamond Si 3x3x3 "
           "= 216 atoms rattled 0.01 A (seed 0); energy+forces+stress; cached NL r_max+0.5 skin"),
    "c1": ("medium", 1, list(range(1, 90)), AVG_NUM_NEIGHBORS, False, WORKLOAD),
    "c2": ("large", 2, [3, 8, 15, 16], 50.0, True,
           "config2: large MACE (128x0e+128x1o+128x2e, lmax3, corr3, 2 layers, r_max 6.0) random-init seed 2; "
           "cubic periodic LiPSO box of 8000 atoms (Li:P:S:O 3:1:4:0.5, 0.06 atoms/A^3, 1.8 A rejection, seed 2); "
           "energy+forces+stress; cached NL r_max+0.5 skin"),
}


def make_structure(rank: int, config: str = "c1"):
    from mace_mlx_b200.structures import diamond_si, lipso_box

    if config == "c0":
        return diamond_si(3, 0.01, 0 + 1000 * rank)
    if config == "c2":
        return lipso_box(8000, 2 + 1000 * rank)
    return diamond_si(5, 0.05, 1 + 1000 * rank)


def make_model_dir(tmp: str, config: str = "c1") -> str:
    from mace_mlx_b200.weights import write_random_model

    arch, seed, z_table, avg, _, _ = SINGLE[config]
    d = Path(tmp) / f"{arch}_seed{seed}"
    write_random_model(d, arch, seed=seed, z_table=z_table, avg_num_neighbors=avg)
    return str(d)


def cpu_model() -> str:
    """The host CPU's model name (lscpu), recorded beside every CPU number."""
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in out.splitlines():
            if line.startswith("Model name:"):
                return line.split(":", 1)[1].strip()
    except Exception:  # noqa: BLE001
        pass
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:  # noqa: BLE001
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock, power and clock-event reasons sampled every 10 ms (NVML, read-only).

    Falls back to ``nvidia-smi -lms 100`` when the NVML binding is missing.
    """

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.stop = threading.Event()
        self.proc = None
        self.lines: list[str] = []
        self.nvml = None

    def _handle(self):
        import pynvml as nv
        import torch

        nv.nvmlInit()
        props = torch.cuda.get_device_properties(self.cuda_index)
        bus = getattr(props, "pci_bus_id", None)
        if bus is not None:
            pci = f"{getattr(props, 'pci_domain_id', 0):08X}:{bus:02X}:{getattr(props, 'pci_device_id', 0):02X}.0"
            try:
                return nv, nv.nvmlDeviceGetHandleByPciBusId(pci)
            except Exception:  # noqa: BLE001
                pass
        return nv, nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def __enter__(self):
        try:
            nv, h = self._handle()
            self.nvml = (nv, h)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons

            def run():
                while not self.stop.is_set():
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), int(get_reasons(h))))
                    except Exception:  # noqa: BLE001
                        pass
                    self.stop.wait(0.01)

            self.t = threading.Thread(target=run, daemon=True)
            self.t.start()
        except Exception:  # noqa: BLE001
            self.nvml = None
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.cuda_index}", f"--query-gpu={self.Q}",
                     "--format=csv,noheader,nounits", "-lms", "100"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.t = threading.Thread(target=self._read, daemon=True)
                self.t.start()
            except Exception:  # noqa: BLE001
                self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.stop.set()
        if self.nvml is not None:
            self.t.join(timeout=1)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], self.max_mhz, set()
        if self.nvml is not None:
            for mhz, bits in self.samples:
                sm.append(mhz)
                reasons.update(nm for nm, bit in self.REASONS.items() if bits & bit)
            src = "nvml 10 ms"
        else:
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for ln in self.lines:
                parts = [p.strip() for p in ln.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for nm, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(nm)
            src = "nvidia-smi 100 ms"
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": src}


# ---------------------------------------------------------------------------
# CPU oracle port timing (cpu_baseline and --impl reference)
# ---------------------------------------------------------------------------
def time_cpu_port(st, model_dir: str, budget_s: float, max_steps: int, warmup: int = 1, stress: bool = False):
    import torch

    from mace_mlx_b200.weights import load_model_dir
    from oracle.model import OracleMACE
    from oracle.nl import neighbour_list

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    config, weights = load_model_dir(model_dir)
    orc = OracleMACE(config, weights, dtype=torch.float32)
    r_cut = float(config["r_max"]) + 0.5
    i, j, S = neighbour_list(st.positions, st.cell, st.pbc, r_cut)
    lut = {int(z): k for k, z in enumerate(config["z_table"])}
    species = np.array([lut[int(z)] for z in st.numbers])
    for _ in range(max(0, warmup)):
        orc.compute(st.positions, species, i, j, S, st.cell, stress=stress)
    times = []
    t_start = time.perf_counter()
    while len(times) < max(1, max_steps):
        t0 = time.perf_counter()
        orc.compute(st.positions, species, i, j, S, st.cell, stress=stress)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    t = statistics.median(times)
    return len(st) / t, threads, len(times), t


def cpu_sample_structure(config: str):
    """A bounded CPU sample of the workload: the full structure for c0/c1, a
    1000-atom box of the same composition and density for c2."""
    from mace_mlx_b200.structures import lipso_box

    if config == "c2":
        return lipso_box(1000, 2), "1000-atom LiPSO box of the same composition and density"
    return make_structure(0, config), "the full structure"


def reference_arm(args, rank: int, world: int):
    if rank != 0:
        return 0
    cfg = args.config if args.config in SINGLE else "c1"
    stress = SINGLE[cfg][4]
    st, what = cpu_sample_structure(cfg)
    warm = min(args.warmup, 3)
    with tempfile.TemporaryDirectory() as tmp:
        md = make_model_dir(tmp, cfg)
        budget = max(30.0, min(150.0, 6.0 * max(1, args.steps)))
        value, threads, n, t = time_cpu_port(st, md, budget, args.steps, warmup=warm, stress=stress)
    sample = (f"{n} steps on {what} (median {t:.2f} s/step) with the torch-CPU fp32 restatement of the reference "
              f"algorithm (pinned to the reference's own execution by tests/golden/ref_*.npz); warm-up {warm}; "
              f"CPU: {cpu_model()}; MLX absent on this host")
    line = {
        "metric": METRIC if cfg == "c1" else f"energy+forces atom-steps/s, {cfg}", "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": n, "warmup": warm,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": SINGLE[cfg][5], "parallelism": "single host process"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
                         "cpu_model": cpu_model()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def measure_fp32_peak(dev) -> dict:
    """FP32 FMA issue rate of this GPU, measured now with the library's probe
    kernel (8 independent FMA chains per thread, 8 CTAs of 256 threads per SM),
    CUDA events on the launching stream, best of 5."""
    import ctypes as C

    import torch

    from mace_mlx_b200 import native as nv

    lib = nv.load_library()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks, iters = sms * 8, 1000
    buf = torch.empty(blocks * 256, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    best = 0.0
    for k in range(6):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        nv.check(lib.mace_fma_probe(C.c_void_p(buf.data_ptr()), blocks, iters, C.c_void_p(stream.cuda_stream)), lib)
        b.record(stream)
        b.synchronize()
        if k:
            ms = a.elapsed_time(b)
            best = max(best, blocks * 256 * 8 * 16 * iters * 2 / (ms * 1e-3) / 1e12)
    return {"tflops": best, "how": f"mace_fma_probe: {blocks} CTAs x 256 threads x 8 FMA chains, best of 5, "
                                   "CUDA events (measured in this run)"}


# ---------------------------------------------------------------------------
# roofline of the dominant kernel of a profiled step
# ---------------------------------------------------------------------------
def roofline_of(work: dict, prof: list[dict], steps: int, fp32_peak: dict | None,
                traffic_key: str | None = None) -> dict:
    """Roofline of the kernel with the largest share of `steps` profiled steps.

    ``work`` holds one step's algorithmic FLOPs, compulsory bytes and
    materialised bytes per (kernel, layer) (``mace_mlx_b200.workmodel``); the
    kernel's time per step is its event-timed total over the steps, so a
    kernel launched once per receiver chunk is compared with its whole work.

    Tensor-core kernels (radial MLP, o3 linears) are reported against the
    measured dense bf16 GEMM peak; CUDA-core kernels against the measured HBM
    copy bandwidth with their COMPULSORY bytes (node tables and edge list), and
    -- since these kernels are FP32-issue bound rather than memory bound --
    against the FP32 FMA peak measured in this run (``fp32``).  ``traffic``
    is ncu's DRAM bytes per launch of the same kernel from
    profiles/ncu_traffic.json (captured on the named workload) and
    ``traffic_over_compulsory`` its ratio to the compulsory bytes.
    """
    peaks = {}
    pp = ROOT / "MEASURED_PEAKS.json"
    if pp.exists():
        peaks = json.loads(pp.read_text())
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    peak_src = "measured (MEASURED_PEAKS.json)" if pp.exists() else "fallback (no MEASURED_PEAKS.json)"
    prof = sorted(prof, key=lambda r: -r["ms"])
    tot_prof = sum(r["ms"] for r in prof)
    top = prof[0]
    avg_ms = top["ms"] / max(1, steps)
    wk = work.get((top["name"], top["layer"]), {"flops": 0, "bytes": 0, "bytes_materialised": 0})
    if top["name"].startswith(("mlp", "linear")):
        ach = wk["flops"] / (avg_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": ach, "peak": bf16, "unit": "TFLOP/s", "frac": ach / bf16}
    else:
        ach = wk["bytes"] / (avg_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm}
    if fp32_peak and fp32_peak.get("tflops"):
        fl = wk["flops"] / (avg_ms * 1e-3) / 1e12
        roof["fp32"] = {"achieved_tflops": fl, "peak_tflops": fp32_peak["tflops"], "frac": fl / fp32_peak["tflops"],
                        "peak_source": fp32_peak["how"]}
    traffic = None
    tp = ROOT / "profiles" / "ncu_traffic.json"
    if traffic_key and tp.exists():
        tr = json.loads(tp.read_text())
        traffic = tr.get(f"{traffic_key}:{top['name']}/{top['layer']}")
    roof.update({
        "traffic": traffic,
        "traffic_over_compulsory": (traffic / wk["bytes"]) if traffic and wk["bytes"] else None,
        "kernel": f"{top['name']} layer {top['layer']}",
        "kernel_share": top["ms"] / tot_prof, "avg_launch_ms": top["ms"] / top["count"],
        "kernel_ms_per_step": avg_ms,
        "algorithmic_flops": wk["flops"], "compulsory_bytes": wk["bytes"],
        "materialised_bytes": wk["bytes_materialised"], "peak_source": peak_src,
        "all_kernels_ms_per_step": {f"{r['name']}/{r['layer']}": r["ms"] / max(1, steps) for r in prof},
    })
    return roof

# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def print_timeline(tl: list[dict]) -> None:
    """One profiled step's launches in start order (stream 0: main, 1: radial-MLP stream), to stderr."""
    end = max((t["end_ms"] for t in tl), default=0.0)
    print(f"timeline of one profiled step: {len(tl)} launches, span {end * 1e3:.1f} us "
          "(the event records add about 3 us per launch)", file=sys.stderr)
    for t in sorted(tl, key=lambda t: t["start_ms"]):
        print(f"  s{t['stream']} {t['name']:18s} L{t['layer']:2d} {t['start_ms'] * 1e3:8.1f} {t['end_ms'] * 1e3:8.1f}"
              f" {(t['end_ms'] - t['start_ms']) * 1e3:7.1f} us", file=sys.stderr)


def b200_arm(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    from mace_mlx_b200.atoms import Atoms
    from mace_mlx_b200.calculators import MACECalculator
    from mace_mlx_b200.workmodel import kernel_work

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = args.config
    stress = SINGLE[cfg][4]
    props = ["energy", "forces", "stress"] if stress else ["energy", "forces"]
    st = make_structure(rank, cfg)
    tmp = tempfile.mkdtemp(prefix=f"bench_r{rank}_")
    md = make_model_dir(tmp, cfg)
    calc = MACECalculator(model_path=md, device=f"cuda:{local_rank}", skin=0.5)
    atoms = Atoms(st.numbers, st.positions, st.cell, st.pbc)
    calc.calculate(atoms, props)
    model = calc.model
    edges = calc._nl_cache
    N, E = len(atoms), edges.n_edges
    out = calc._out
    pos = out["pos"]
    cell = out["cell"]
    species = calc._species_dev
    gptr = calc._graph_ptr_dev
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB > L2

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def step():
        model.evaluate(pos, cell, species, gptr, edges, forces=True, virial=stress, out=out, graph=True)

    if args.device_only:
        for _ in range(args.warmup + args.steps):
            model.evaluate(pos, cell, species, gptr, edges, forces=True, virial=stress, out=out)
        torch.cuda.synchronize(dev)
        return 0
    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local_rank) as clk:
        barrier()
        for k in range(args.steps):
            flush.zero_()
            ev[k][0].record()
            step()
            ev[k][1].record()
        barrier()
    dev_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = float(sum(dev_ms))
    launches = model.last_launch_count()
    # e2e through the public API: host positions in, host energy/forces out
    rng = np.random.default_rng(7 + rank)
    jitter = [st.positions + rng.normal(0, 1e-4, st.positions.shape) for _ in range(args.steps + args.warmup)]
    for k in range(args.warmup):
        atoms.positions = jitter[k]
        calc.calculate(atoms, props)
    barrier()
    t0 = time.perf_counter()
    for k in range(args.steps):
        atoms.positions = jitter[args.warmup + k]
        calc.calculate(atoms, props)
    e2e_s = time.perf_counter() - t0
    barrier()
    # per-kernel event timing (separate pass, same inputs)
    model.profile_enable(True)
    for _ in range(args.steps):
        step()
    prof = model.profile_read()
    if args.timeline:
        print_timeline(model.profile_timeline())
    model.profile_enable(False)
    fp32 = measure_fp32_peak(dev)
    if world > 1:
        tt = torch.tensor([total_ms, e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms, e2e_s = float(tt[0]), float(tt[1])
    if rank != 0:
        return 0
    value = world * N * args.steps / (total_ms / 1e3)
    e2e_value = world * N * args.steps / e2e_s
    roof = roofline_of(kernel_work(model.spec, N, E), prof, args.steps, fp32, traffic_key=cfg)
    cpu = None
    if world == 1:
        try:
            cst, what = cpu_sample_structure(cfg)
            v, threads, n, t = time_cpu_port(cst, md, args.cpu_seconds, 3, stress=stress)
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": cpu_model(),
                   "sample": f"{n} steps on {what} (median {t:.2f} s) of the torch-CPU fp32 oracle port"}
        except Exception as e:  # noqa: BLE001
            cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {e}"}
    # the calculator moves one input block (cell + positions) and one output block
    # (energy, virial, forces, node energies) per step
    h2d = calc._blk[0].numel() * calc._blk[0].element_size()
    d2h = calc._blk[1].numel() * calc._blk[1].element_size()
    line = {
        "metric": METRIC if cfg == "c1" else f"energy+forces atom-steps/s, {cfg}", "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": SINGLE[cfg][5], "n_atoms_per_gpu": N, "n_edges_per_gpu": E,
                   "l2": "flushed between timed steps (256 MB write)",
                   "parallelism": f"structure-sharded x{world} (one independent structure per GPU)"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_s * 1e3 / args.steps},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
        "roofline": roof,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def spatial_weak_arm(args, rank: int, world: int, local_rank: int):
    """N Si1000 blocks as one periodic structure, one block per rank (see the module docstring)."""
    import torch
    import torch.distributed as dist

    from mace_mlx_b200.distributed import SpatialRunner, grid_for
    from mace_mlx_b200.model import MACEModel
    from mace_mlx_b200.spec import ModelSpec
    from mace_mlx_b200.structures import diamond_si
    from mace_mlx_b200.weights import random_config, random_weights
    from mace_mlx_b200.workmodel import kernel_work

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    grid = grid_for(world)
    st = diamond_si(tuple(5 * g for g in grid), 0.05, 1)
    config = random_config("medium", z_table=list(range(1, 90)), avg_num_neighbors=AVG_NUM_NEIGHBORS)
    model = MACEModel(config=config, weights=random_weights(ModelSpec.from_config(config), seed=1), device=dev)
    runner = SpatialRunner(model, st.numbers, st.cell, world, rank, skin=0.5)
    runner.graph = True
    pos_global = torch.tensor(st.positions, dtype=torch.float64, device=dev)
    runner.evaluate(pos_global)
    own_idx = torch.as_tensor(runner.owned_index, device=dev)
    own_pos = pos_global[own_idx].clone()
    n_total = len(st)
    pl = runner.plan

    def barrier():
        dist.barrier()
        torch.cuda.synchronize(dev)

    def step():
        return runner.step(own_pos, check_skin=False)

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local_rank) as clk:
        barrier()
        for k in range(args.steps):
            ev[k][0].record()
            step()
            ev[k][1].record()
        barrier()
    total_ms = float(sum(a.elapsed_time(b) for a, b in ev))
    launches = model.last_launch_count()
    # e2e: host owned positions in (pinned), the skin check, forces and energy back to the host
    host_pos = torch.empty(own_pos.shape, dtype=torch.float64, pin_memory=True)
    host_pos.copy_(own_pos)
    host_f = torch.empty(own_pos.shape, dtype=torch.float32, pin_memory=True)
    host_e = torch.empty(1, dtype=torch.float64, pin_memory=True)

    def step_e2e():
        own_pos.copy_(host_pos, non_blocking=True)
        res = runner.step(own_pos)
        host_f.copy_(res["forces"], non_blocking=True)
        host_e.copy_(res["energy"], non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return float(host_e[0])

    for _ in range(max(1, args.warmup // 2)):
        step_e2e()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step_e2e()
    barrier()
    e2e_s = time.perf_counter() - t0
    model.profile_enable(True)
    prof_steps = min(args.steps, 5)
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize(dev)
    prof = model.profile_read()
    model.profile_enable(False)
    fp32 = measure_fp32_peak(dev)
    tt = torch.tensor([total_ms, e2e_s], dtype=torch.float64, device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    total_ms, e2e_s = float(tt[0]), float(tt[1])
    counts = torch.tensor([pl.n_owned, pl.n_local], dtype=torch.int64, device=dev)
    all_counts = [torch.empty_like(counts) for _ in range(world)]
    dist.all_gather(all_counts, counts)
    runner.close()
    if rank != 0:
        return 0
    e_act = runner.active[1] if runner.active else runner.edges.n_edges
    roof = roofline_of(kernel_work(model.spec, pl.n_owned, e_act), prof, prof_steps, fp32)
    line = {
        "metric": METRIC, "value": n_total * args.steps / (total_ms / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": (f"medium MACE as config 1 (seed 1); one periodic diamond Si structure of "
                                f"{world} Si1000 blocks ({5 * grid[0]}x{5 * grid[1]}x{5 * grid[2]} cells, "
                                f"{n_total} atoms, rattled 0.05 A, seed 1); energy+forces"),
                   "n_atoms_total": n_total,
                   "owned_local_atoms_per_rank": [[int(c[0]), int(c[1])] for c in all_counts],
                   "parallelism": (f"spatial domains {grid[0]}x{grid[1]}x{grid[2]}, r_max+skin ghost shells, owned "
                                   "atoms the only receivers, layer-1 features and their gradients halo-exchanged "
                                   "in the step (NCCL send/recv issued by the library, step replayed as a CUDA "
                                   "graph), ghost positions/forces exchanged per step, energy all-reduced"),
                   "l2": "inputs per rank below L2; no flush (a flush would serialise the ranks' NCCL traffic)"},
        "e2e": {"value": n_total * args.steps / e2e_s, "unit": UNIT,
                "h2d_bytes_per_step": int(own_pos.numel() * 8), "d2h_bytes_per_step": int(own_pos.numel() * 4 + 8),
                "ms_per_step": e2e_s * 1e3 / args.steps},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
        "roofline": roof,
        "cpu_baseline": None,
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# partitioned configurations: c3 (structure sharding), c4 (spatial domains)
# ---------------------------------------------------------------------------
C3_WORKLOAD = ("config3: MACE-OFF-medium-like (96x0e+96x1o, lmax3, corr3, 2 layers, r_max 5.0, H/C/N/O) random-init "
               "seed 3; 512 random-walk molecules of 20-60 atoms (seed 3), non-periodic; energy+forces; molecules "
               "sharded over the ranks by atom count")
C4_WORKLOAD = ("config4: medium MACE as config 1 (seed 1); diamond Si 50x50x50 = 1,000,000 atoms rattled 0.05 A "
               "(seed 4); energy+forces+stress; spatial domains (grid 1x1x2, 1x2x2, 2x2x2) periodic along unsplit "
               "axes, r_max + skin = 6.5 A ghost shells across split axes, owned atoms the only receivers; layer-1 "
               "node features and their gradients halo-exchanged inside the step (library NCCL send/recv, step "
               "replayed as a CUDA graph); ghost positions and forces exchanged per step (halo-sized), "
               "energy/virial all-reduced")


def partition_arm(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    from mace_mlx_b200.distributed import SpatialRunner, shard_structures
    from mace_mlx_b200.model import MACEModel
    from mace_mlx_b200.spec import ModelSpec
    from mace_mlx_b200.structures import diamond_si, molecule_batch
    from mace_mlx_b200.weights import random_config, random_weights
    from mace_mlx_b200.workmodel import kernel_work

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    if args.config == "c4":
        st = diamond_si(50, 0.05, 4)
        config = random_config("medium", z_table=list(range(1, 90)), avg_num_neighbors=AVG_NUM_NEIGHBORS)
        model = MACEModel(config=config, weights=random_weights(ModelSpec.from_config(config), seed=1), device=dev)
        runner = SpatialRunner(model, st.numbers, st.cell, world, rank, skin=0.5)
        runner.graph = True
        pos_global = torch.tensor(st.positions, dtype=torch.float64, device=dev)
        n_total = len(st)
        virial = True
        runner.evaluate(pos_global, virial=True)
        own_idx = torch.as_tensor(runner.owned_index, device=dev)
        own_pos = pos_global[own_idx].clone()
        owned = {rank: runner.owned_index}
        del pos_global

        def step():
            return runner.step(own_pos, virial=True, check_skin=False)

        host_pos = torch.empty(own_pos.shape, dtype=torch.float64, pin_memory=True)
        host_pos.copy_(own_pos)
        host_f = torch.empty(own_pos.shape, dtype=torch.float32, pin_memory=True)

        def step_e2e():
            own_pos.copy_(host_pos, non_blocking=True)
            res = runner.step(own_pos, virial=True)
            host_f.copy_(res["forces"], non_blocking=True)
            e = res["energy"].item()  # synchronises
            return e

        h2d, d2h = len(owned[rank]) * 24, len(owned[rank]) * 12 + 8
        n_local = runner.plan.n_owned if runner.active else runner.plan.n_local
        e_local = runner.active[1] if runner.active else runner.edges.n_edges
        workload, scaling = C4_WORKLOAD, "strong"
        parallel = f"spatial domains {runner.grid[0]}x{runner.grid[1]}x{runner.grid[2]}"
        prof_model, prof_n, prof_e = model, n_local, e_local
    else:
        st_all = molecule_batch(512, 3)
        config = random_config("medium", hidden_irreps="96x0e + 96x1o", r_max=5.0, z_table=[1, 6, 7, 8],
                               avg_num_neighbors=12.0)
        model = MACEModel(config=config, weights=random_weights(ModelSpec.from_config(config), seed=3), device=dev)
        sizes = np.bincount(st_all.batch)
        mine = shard_structures(sizes, world)[rank]
        sel = np.isin(st_all.batch, mine)
        remap = {g: k for k, g in enumerate(mine)}
        batch = np.array([remap[g] for g in st_all.batch[sel]], dtype=np.int64)
        gp = torch.as_tensor(np.concatenate([[0], np.cumsum(np.bincount(batch, minlength=len(mine)))]).astype(np.int32),
                             device=dev)
        pos64 = torch.tensor(st_all.positions[sel], dtype=torch.float64, device=dev)
        edges = model.neighbour_list(pos64, None, (False, False, False), gp, model.r_max + 0.5)
        species = torch.as_tensor(model.species_index(st_all.numbers[sel]), device=dev)
        pos32 = pos64.float()
        n_total = len(st_all)
        virial = False
        state = {"out": None}

        def step():
            state["out"] = model.evaluate(pos32, None, species, gp, edges, forces=True, out=state["out"], graph=True)
            return state["out"]

        host_pos = torch.empty(pos32.shape, dtype=torch.float32, pin_memory=True)
        host_pos.copy_(pos32)
        host_f = torch.empty(pos32.shape, dtype=torch.float32, pin_memory=True)
        host_e = torch.empty(len(mine), dtype=torch.float64, pin_memory=True)

        def step_e2e():
            pos32.copy_(host_pos, non_blocking=True)
            out = step()
            host_f.copy_(out["forces"], non_blocking=True)
            host_e.copy_(out["energy"], non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
            return float(host_e.sum())

        h2d, d2h = pos32.numel() * 4, pos32.numel() * 4 + len(mine) * 8
        workload, scaling = C3_WORKLOAD, "strong"
        parallel = f"structure-sharded over {world} ranks ({len(mine)} molecules, {int(sel.sum())} atoms on rank 0)"
        prof_model, prof_n, prof_e = model, int(sel.sum()), edges.n_edges

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local_rank) as clk:
        barrier()
        for k in range(args.steps):
            ev[k][0].record()
            step()
            ev[k][1].record()
        barrier()
    total_ms = float(sum(a.elapsed_time(b) for a, b in ev))
    launches = prof_model.last_launch_count()
    for _ in range(max(1, args.warmup // 2)):
        step_e2e()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step_e2e()
    barrier()
    e2e_s = time.perf_counter() - t0
    prof_model.profile_enable(True)
    prof_steps = min(args.steps, 3)
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize(dev)
    prof = prof_model.profile_read()
    prof_model.profile_enable(False)
    if world > 1:
        tt = torch.tensor([total_ms, e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms, e2e_s = float(tt[0]), float(tt[1])
    if rank != 0:
        return 0
    value = n_total * args.steps / (total_ms / 1e3)
    roof = roofline_of(kernel_work(prof_model.spec, prof_n, prof_e), prof, prof_steps, measure_fp32_peak(dev))
    cpu = None
    if world == 1:
        try:
            with tempfile.TemporaryDirectory() as tmp:
                md = make_model_dir(tmp)
                v, threads, n, t = time_cpu_port(make_structure(0), md, args.cpu_seconds, 3)
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": cpu_model(),
                   "sample": f"{n} full 1000-atom Si steps of the medium model (median {t:.2f} s) of the torch-CPU "
                             f"fp32 oracle port; the per-atom rate stands in for this workload"}
        except Exception as e:  # noqa: BLE001
            cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {e}"}
    line = {
        "metric": f"energy+forces atom-steps/s, {args.config}", "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload, "n_atoms_total": n_total, "n_local_atoms_rank0": prof_n,
                   "n_edges_rank0": prof_e, "parallelism": parallel,
                   "l2": "inputs larger than L2 (c4)" if args.config == "c4" else "no flush (sub-L2 shards)"},
        "e2e": {"value": n_total * args.steps / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_s * 1e3 / args.steps},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
        "roofline": roof,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.config in ("c3", "c4"):
            return partition_arm(args, rank, world, local_rank)
        if world > 1 and args.config == "c1":
            return spatial_weak_arm(args, rank, world, local_rank)
        return b200_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
