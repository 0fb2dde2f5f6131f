#!/usr/bin/env python
"""Benchmark: atom-steps/s of DPA4C-style energy + force + virial evaluation.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200dp|reference]

One step = one evaluation of the hot path (neighbour graph from coordinates,
descriptor, fitting forward + backward, force / virial assembly) over the
12,288-atom water system of the 1-GPU configuration (4096 H2O, 49.68 A cube,
water model sel [46,92], embedding [25,50,100], axis 16, fitting [240]*3,
random-init weights, seed 0).  Inputs are seeded synthetic data.

* ``value``: device-timed throughput, inputs resident in HBM, CUDA events on
  the launch stream around each step; L2 is flushed (256 MB write) before
  every timed step, outside the events.  The force call (its 24 kernels) is
  recorded once as a CUDA graph and replayed each step.  Multi-GPU (weak scaling): one
  process per GPU, one global water box of 4096 H2O per GPU split by spatial
  domain decomposition (slab for 2 GPUs, 2x2x1 for 4, 2x2x2 for 8; 8 A ghost
  shell); a step is the forward halo of coordinates over NCCL, the force call
  on owned + ghost atoms whose assembly adds every ghost contribution straight
  into the owner's force accumulator through NVLink peer memory (CUDA IPC;
  ``--reverse nccl`` instead folds ghost forces back by NCCL send/recv), an
  all-reduce of energy and virial and the owners' conversion of their
  accumulators; time = max over ranks.
* ``e2e``: the same metric through the public API with pinned host buffers:
  1 GPU, the host C entry (b200dp_compute_host), H2D of coordinates and
  types, D2H of forces, energy and virial inside the timed region; N GPUs,
  each rank copies its owned coordinates in and its forces, energy and
  virial out around DistributedDeepPot.step.
* ``roofline``: the dominant kernel (descriptor backward), algorithmic FLOPs
  per launch over its CUDA-event duration, against the measured bf16 peak.
* ``cpu_baseline``: the CPU oracle (C++ fp64, OpenMP) on the host cores.

``--sweep`` measures the five configurations instead of the headline (one JSON
line per configuration and mode): on 1 GPU the force call on every system
(C0 fp64 and mixed, C1 fp64 and mixed, C2, C3, the C4 water sizes 1.5k-3.1M
and the 786k slab, mixed) and the device MD driver over the configuration's
steps (C1 NVT 1000, C2 NPT 500, C3 NVT 200, C4 NVT 100; neighbour candidates
rebuilt every 10 steps with a 2 A skin); on N > 1 GPUs the domain-decomposed
force call of the systems the configurations run there (C2 on 2, C3 and the
C4 786k / 3.1M / slab on 2, 4, 8; strong scaling: the global system is fixed).

``--impl reference`` times the reference arm: the reference ships no CPU (or
NVIDIA) implementation of this path, so it is the CPU restatement (oracle)
run with all host threads on the same configuration.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "dpa4c-scale-aware-md_b200")
sys.path.insert(0, PKG)

import modelgen  # noqa: E402
import systems  # noqa: E402

METRIC = "atom-steps/s (E+F+virial)"
WORKLOAD = "c1_water_12288"
L2_FLUSH_BYTES = 256 << 20
FP64_NOMINAL_TFLOPS = 37.0  # B200 (HGX) fp64 and fp64 tensor, dense
HALO = 8.0  # ghost shell: rcut 6 A + 2 A neighbour skin


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200dp", choices=["b200dp", "reference"])
    ap.add_argument("--precision", default="mixed", choices=["mixed", "fp64"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="headline device loop only (no e2e, fp64, MD, C8L2 or CPU legs): the ncu captures' command")
    ap.add_argument("--sweep", action="store_true", help="measure the five configurations (see module doc)")
    ap.add_argument("--only", default="", help="--sweep: comma-separated labels to run")
    ap.add_argument("--reverse", default="peer", choices=["peer", "nccl"],
                    help="N > 1 with --driver python: ghost forces to their owners by peer-memory atomics or by "
                         "NCCL send/recv")
    ap.add_argument("--driver", default="cpp", choices=["cpp", "python"],
                    help="N > 1: the C++ decomposed driver (b200dp_dd_*) or the torch.distributed one (domain.py)")
    ap.add_argument("--no-strong", action="store_true", help="skip the 3.1M-atom strong-scaling leg")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def model_path(kind="water"):
    d = tempfile.mkdtemp(prefix="b200dp_bench_")
    p = os.path.join(d, f"{kind}.b2dp")
    if kind == "c8l2":
        modelgen.save_c8(modelgen.random_c8_model(seed=0), p)
    else:
        modelgen.save(modelgen.random_model(kind, seed=0), p)
    return p


# ----------------------------------------------------------------- clocks
REASON_COLS = ["clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
               "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]


def start_clocks(gpu: int, path: str):
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," + ",".join(REASON_COLS))
    try:
        f = open(path, "w")
        p = subprocess.Popen(["nvidia-smi", "-i", str(gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                              "-lms", "25"], stdout=f, stderr=subprocess.DEVNULL)
        return p, f
    except OSError:
        return None, None


def stop_clocks(p, f, path):
    if p is None:
        return None
    p.terminate()
    try:
        p.wait(timeout=5)
    except subprocess.TimeoutExpired:
        p.kill()
    f.close()
    sm, smax, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in open(path):
        parts = [x.strip() for x in line.split(",")]
        if len(parts) < 9:
            continue
        try:
            sm.append(float(parts[1]))
            smax = float(parts[2])
        except ValueError:
            continue
        for n, v in zip(names, parts[5:9]):
            if v.lower() == "active":
                reasons.add(n)
    if not sm:
        return None
    return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- roofline inputs
def model_flops(m: modelgen.SeaModel, nloc: int, edges: int):
    """Algorithmic FLOPs (2 per multiply-add) per evaluation, split by kernel."""
    dims = m.emb_dims()
    emb_mac = sum(dims[l] * dims[l + 1] for l in range(len(dims) - 1))
    emb_bwd_mac = sum(dims[l] * dims[l + 1] for l in range(1, len(dims) - 1)) + dims[1]
    M1, M2 = m.emb[-1], m.axis
    fwd = 2 * (edges * (emb_mac + 4 * M1) + nloc * 4 * M1 * M2)
    bwd = 2 * (edges * (emb_mac + emb_bwd_mac + 8 * M1) + nloc * 8 * M1 * M2)
    fd = m.fit_dims()
    fit_mac = sum(fd[l] * fd[l + 1] for l in range(len(fd) - 1))
    fit = 2 * nloc * (2 * fit_mac)
    return {"descriptor_fwd": fwd, "fitting": fit, "descriptor_bwd": bwd, "total": fwd + fit + bwd}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def ncu_traffic(kernel: str):
    """DRAM bytes per launch of `kernel` recorded in the committed ncu summary, and the summary's
    note on which build of the kernel that capture measured (None when it has none)."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_c1_water.md")
    if not os.path.exists(path):
        return None, None
    value = note = None
    for line in open(path):
        m = re.match(r"\s*traffic_bytes_per_launch:\s*([0-9.eE+]+)", line)
        if m:
            value = float(m.group(1))
        m = re.match(r"\s*traffic_note:\s*(.+)", line)
        if m:
            note = m.group(1).strip()
    return value, note


# ----------------------------------------------------------------- arms
class OracleArm:
    """The CPU oracle loaded once: model read and first touch happen here, outside any timing."""

    def __init__(self, model_file, threads=None):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle

        self.cores = oracle.set_threads(threads or os.cpu_count() or 1)
        self.o = oracle.Oracle(model_file)
        s0 = systems.config0()
        self.o.compute(s0.coord, s0.atype, s0.box, atomic=False)

    def evaluate(self, system):
        """Seconds for one full E+F+virial evaluation of `system`."""
        t0 = time.perf_counter()
        self.o.compute(system.coord, system.atype, system.box, atomic=False)
        return time.perf_counter() - t0


def bench_config(world):
    """The `config` dict shared by both arms at N GPUs (same keys and values): 4096 H2O per GPU."""
    return {"workload": WORKLOAD, "atoms_per_gpu": 12288, "global_atoms": 12288 * world,
            "model": "water se_e2_a-type (sel [46,92], embedding [25,50,100], axis 16, fitting [240]*3), random init",
            "l2": "GPU arm: flushed before every timed step (256 MB write), flush outside the events"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    system, _ = global_system(1, 0)
    arm = OracleArm(model_path("water"))
    for _ in range(args.warmup):
        arm.evaluate(system)
    secs = [arm.evaluate(system) for _ in range(args.steps)]
    dt = sum(secs) / len(secs)
    value = system.natoms / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "atom-steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded water, random-init weights)",
        "config": bench_config(world),
        "cpu_baseline": {"value": value, "unit": "atom-steps/s", "cores": arm.cores, "kind": "port",
                         "sample": "one full evaluation of the 12,288-atom system per step (model loaded and "
                                   "warmed up before the timed steps)"},
        "e2e": {"value": value, "unit": "atom-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU or NVIDIA implementation of this path; the reference arm is the "
                "C++ fp64 restatement (oracle/) on all host threads; at N > 1 rank 0 times one 12,288-atom "
                "evaluation per step (the CPU cost per atom does not depend on the box size)",
    }
    print(json.dumps(line), flush=True)


class Periodic:
    """One GPU: the whole periodic box through b200dp_compute_device."""

    def __init__(self, dp, system, dev, stream, torch):
        self.dp, self.system, self.stream = dp, system, stream
        self.n = self.total = system.natoms
        self.x = torch.tensor(system.coord, device=dev)
        self.t = torch.tensor(system.atype, device=dev)
        self.e = torch.zeros(1, dtype=torch.float64, device=dev)
        self.f = torch.zeros(self.n, 3, dtype=torch.float64, device=dev)
        self.v = torch.zeros(9, dtype=torch.float64, device=dev)
        self.torch = torch
        self.graph = None

    def _call(self, stream):
        self.dp.compute_device(stream.cuda_stream, self.n, 0, self.x.data_ptr(), self.t.data_ptr(),
                               self.system.box, None, self.e.data_ptr(), self.f.data_ptr(), self.v.data_ptr())

    def capture(self):
        """Records the force call (24 kernels) as one CUDA graph; step() replays it.  The call
        is capture-safe: no host synchronisation, fixed buffers, the same box every step."""
        torch = self.torch
        side = torch.cuda.Stream()
        side.wait_stream(self.stream)
        with torch.cuda.stream(side):
            self._call(side)
        self.stream.wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            self._call(side)
        torch.cuda.synchronize()
        self.graph = g

    def release(self):
        self.graph = None

    def step(self):
        if self.graph is not None:
            self.graph.replay()
            return
        self._call(self.stream)


class Decomposed:
    """N GPUs: spatial domain decomposition of one global box (domain.py)."""

    def __init__(self, dp, system, grid, rank, dev, stream, torch, peer_fold=True):
        import domain

        self.dp, self.stream = dp, stream
        dd = domain.Decomposition(system.box, grid, rank, HALO)
        x, t, ids = domain.distribute(system.coord, system.atype, dd)

        def compute(x_all, t_all, nloc, nghost, region, e, f, v):
            dp.compute_device(torch.cuda.current_stream(dev).cuda_stream, nloc, nghost, x_all.data_ptr(),
                              t_all.data_ptr(), None, region, e.data_ptr(), f.data_ptr(), v.data_ptr())

        fold = domain.PeerFold(dp, dev) if peer_fold else None
        self.ddp = domain.DistributedDeepPot(compute, system.box, grid, rank, HALO, x, t, ids, device=dev, fold=fold)
        self.n = self.ddp.nloc
        self.total = system.natoms
        self.nghost = self.ddp.nghost

    def capture(self):
        self.ddp.capture()

    def release(self):
        self.ddp.release()

    def step(self):
        self.ddp.step()


class DecomposedCpp:
    """N GPUs: the C++ decomposed driver (b200dp_dd_*): NCCL for the setup and the plan, peer memory
    and device-side rendezvous for the per-step exchange; the step replayed as one CUDA graph."""

    def __init__(self, dp, system, grid, rank, world, dev, stream, torch, dist):
        import b200dp

        uid = [b200dp.dd_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        self.dd = b200dp.DD(dp, uid[0], world, rank, system.coord, system.atype, system.box, grid, halo=HALO)
        self.dp, self.stream, self.torch = dp, stream, torch
        self.n, self.nghost = self.dd.counts()
        self.total = system.natoms
        self.graph = None

    def capture(self):
        torch = self.torch
        side = torch.cuda.Stream()
        side.wait_stream(self.stream)
        with torch.cuda.stream(side):
            self.dd.force(side.cuda_stream)
        self.stream.wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            self.dd.force(side.cuda_stream)
        torch.cuda.synchronize()
        self.graph = g

    def release(self):
        self.graph = None

    def step(self):
        if self.graph is not None:
            self.graph.replay()
            return
        self.dd.force(self.stream.cuda_stream)

    def close(self):
        self.graph = None
        self.dd.close()


def overlap_probe(torch, b200dp, mp, system, dev, local, flush, steps=10):
    """Speed-up of two force calls running concurrently on two streams over the same two calls in turn."""
    engines, works, streams = [], [], []
    for _ in range(2):
        st = torch.cuda.Stream(device=dev)
        dp = b200dp.DeepPot(mp, precision=b200dp.MIXED, device=local)
        w = Periodic(dp, system, dev, st, torch)
        for _ in range(3):
            with torch.cuda.stream(st):
                w.step()
        w.capture()
        engines.append(dp)
        works.append(w)
        streams.append(st)
    torch.cuda.synchronize()

    def run(concurrent):
        flush.fill_(1)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        base = torch.cuda.current_stream(dev)
        t0.record(base)
        for st in streams:
            st.wait_stream(base)
        for _ in range(steps):
            if concurrent:
                for w, st in zip(works, streams):
                    with torch.cuda.stream(st):
                        w.step()
            else:
                for w, st in zip(works, streams):
                    with torch.cuda.stream(streams[0]):
                        w.step()
        for st in streams:
            base.wait_stream(st)
        t1.record(base)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1)

    serial = min(run(False) for _ in range(2))
    both = min(run(True) for _ in range(2))
    for w, dp in zip(works, engines):
        w.release()
        dp.close()
    torch.cuda.empty_cache()
    return {"atoms": system.natoms, "serial_ms_per_pair": serial / steps, "concurrent_ms_per_pair": both / steps,
            "speedup": serial / both}


def global_system(world, rank):
    """Weak scaling: 4096 H2O per GPU, the global box grows with the rank grid."""
    import domain

    if world == 1:
        return systems.config1(), (1, 1, 1)
    grid = domain.rank_grid(world)
    return systems.water(16 * grid[0], 16 * grid[1], 16 * grid[2], seed=0, name=WORKLOAD), grid


def run_b200dp(args, world, rank, local):
    import torch

    import b200dp

    torch.cuda.set_device(local)
    dist = None
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    system, grid = global_system(world, rank)
    mp = model_path("water")
    m = modelgen.load(mp)
    prec = b200dp.MIXED if args.precision == "mixed" else b200dp.FP64
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    sync = torch.zeros(1, device=dev)

    def workload(dp, sys_=None, grid_=None):
        sys_ = sys_ or system
        grid_ = grid_ or grid
        if world == 1:
            return Periodic(dp, sys_, dev, stream, torch)
        if args.driver == "cpp":
            return DecomposedCpp(dp, sys_, grid_, rank, world, dev, stream, torch, dist)
        return Decomposed(dp, sys_, grid_, rank, dev, stream, torch, peer_fold=args.reverse == "peer")

    def device_loop(dp, w, steps, warmup):
        """Timed steps: CUDA events around each step on the launch stream, L2 flushed before each,
        no host synchronisation inside the loop.  The step is replayed as a CUDA graph (the periodic
        force call on 1 GPU, the decomposed step on N); its kernel count per step is the number the
        capture recorded."""
        for _ in range(warmup):
            w.step()
        dp.check()
        dp.set_stage_timing(False)
        per_step = None
        if hasattr(w, "capture"):
            l0 = b200dp.kernel_launches()
            w.capture()
            per_step = (b200dp.kernel_launches() - l0) // 2  # the capture runs one eager step, then records one
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        l0 = b200dp.kernel_launches()
        for k in range(steps):
            flush.fill_(k & 0xFF)
            if dist:  # ranks enter the step together (device-side, no host sync)
                dist.all_reduce(sync)
            starts[k].record(stream)
            w.step()
            ends[k].record(stream)
        torch.cuda.synchronize()
        launches = b200dp.kernel_launches() - l0 if per_step is None else per_step * steps
        if dist:
            dist.barrier()
        dp.check()
        if hasattr(w, "release"):
            w.release()
        ms = sum(s.elapsed_time(en) for s, en in zip(starts, ends))
        return ms, launches

    def stage_pass(dp, w, nsteps):
        """Per-stage device times from the engine's stage events (a host sync per step, so this
        runs apart from the timed loop)."""
        dp.set_stage_timing(True)
        stages = []
        for k in range(nsteps):
            flush.fill_(k & 0xFF)
            if dist:
                dist.all_reduce(sync)
            w.step()
            stages.append(dp.stage_times())
        dp.set_stage_timing(False)
        return np.array(stages).mean(0)

    def max_over_ranks(x):
        if not dist:
            return x
        tt = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    dp = b200dp.DeepPot(mp, precision=prec, device=local)
    w = workload(dp)
    n = w.n
    clk_path = os.path.join(tempfile.gettempdir(), f"b200dp_clocks_{rank}.csv")
    cp, cf = start_clocks(local, clk_path)
    ms, launches = device_loop(dp, w, args.steps, args.warmup)
    clocks = stop_clocks(cp, cf, clk_path)
    stage_ms = stage_pass(dp, w, max(5, min(args.steps, 20)))
    ms = max_over_ranks(ms)
    value = w.total * args.steps / (ms / 1e3)
    # edges (real neighbours) of this rank's owned atoms for the FLOP count
    nl = dp.last_nlist(n)["nlist"]
    edges = int((nl >= 0).sum())
    fl = model_flops(m, n, edges)
    pk, pk_kind = peaks()
    bwd_ms = float(stage_ms[3])
    achieved = fl["descriptor_bwd"] / (bwd_ms / 1e3) / 1e12 if bwd_ms > 0 else 0.0
    mixed = prec == b200dp.MIXED
    if mixed:
        peak = float(pk["bf16_tflops"])
        peak_source = (f"{pk_kind} bf16 burst (MEASURED_PEAKS.json)" if pk_kind == "measured"
                       else "fallback 1.59 PFLOP/s")
    else:  # the fp64 products and fp64 instructions share one pipe; no fp64 peak is measured on this pool
        peak = FP64_NOMINAL_TFLOPS
        peak_source = "nominal B200 fp64 (tensor and vector), no measured fp64 peak"
    traffic, traffic_note = ncu_traffic("embed_bwd_tc" if mixed else "embed_f64")
    roofline = {"kernel": "k_embed_bwd_tc" if mixed else "k_embed_bwd_f64", "bound": "tensor",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": traffic, "peak_source": peak_source,
                "flops_per_launch": fl["descriptor_bwd"], "avg_launch_ms": bwd_ms,
                "note": "algorithmic FLOPs of the embedding backward over the CUDA-event time of its stage"}
    if traffic_note:
        roofline["traffic_note"] = traffic_note
    if mixed:
        # the pipe that bounds the embedding kernels: the multi-function unit (MUFU / XU), 16 results per
        # clock per SM; every tanh feature of every edge costs one ex2 and one rcp, and the backward
        # recomputes all layers
        mufu = 2 * edges * sum(m.emb)
        mhz = (clocks or {}).get("sm_mhz") or float(pk.get("sm_max_mhz", 1965.0))
        xu_peak = 148 * 16 * mhz * 1e6
        roofline["xu"] = {"mufu_ops_per_launch": mufu, "sm_mhz": mhz, "peak_ops_per_s": xu_peak,
                          "frac": mufu / (bwd_ms / 1e3) / xu_peak if bwd_ms > 0 else 0.0,
                          "note": "MUFU ops (2 per tanh feature per edge) over the stage time, against "
                                  "148 SMs x 16 per clock at the median SM clock of the timed region"}
    # e2e through the public API with pinned host buffers
    e2e = None
    if args.profile:
        e2e = {"skipped": "--profile"}
    else:
        try:
            e2e = e2e_loop(dp, w, system, args.steps, max(1, min(args.warmup, 3)), torch, dist)
        except Exception as ex:  # report, never hide
            e2e = {"error": repr(ex)}
    if "seconds" in e2e:
        secs = max_over_ranks(e2e["seconds"])
        e2e["value"] = w.total * args.steps / secs
        e2e["seconds"] = secs
    # fp64 mode (secondary line item)
    fp64 = None
    if prec == b200dp.MIXED and not args.profile:
        dp64 = b200dp.DeepPot(mp, precision=b200dp.FP64, device=local)
        w64 = workload(dp64)
        k64 = max(2, min(args.steps, 5))
        ms64, _ = device_loop(dp64, w64, k64, max(1, min(args.warmup, 2)))
        ms64 = max_over_ranks(ms64)
        st64 = stage_pass(dp64, w64, 2)
        fp64 = {"value": w.total * k64 / (ms64 / 1e3), "ms_per_step": ms64 / k64,
                "stage_ms": [round(float(q), 4) for q in st64]}
        del w64
        dp64.close()
    # MD loop (N = 1): the same force call inside the device MD driver (NVT Nose-Hoover chain,
    # velocity Verlet), reported beside the force-call metric
    md_loop = None
    if world == 1 and prec == b200dp.MIXED and not args.profile:
        try:
            md = b200dp.MD(dp, system.coord, system.atype, system.box, [15.9994, 1.00794], dt=0.0005,
                           ensemble=b200dp.NVT, t_init=300.0, t_target=300.0, t_damp=0.05, seed=1)
            md.run(max(3, args.warmup))
            md.thermo()
            k_md = max(10, args.steps)
            t0 = time.perf_counter()
            md.run(k_md)
            th = md.thermo()
            dt_md = time.perf_counter() - t0
            md_loop = {"ms_per_step": 1e3 * dt_md / k_md, "value": n * k_md / dt_md, "unit": "atom-steps/s",
                       "steps": k_md, "ensemble": "NVT (Nose-Hoover chain 3, 300 K, dt 0.5 fs)",
                       "temperature_K": th["temp"], "timing": "host wall clock around the enqueued steps + sync"}
            md.close()
        except Exception as ex:  # report, never hide
            md_loop = {"error": repr(ex)}
    # C8L2 profile (the reference's production descriptor), secondary line item at N = 1:
    # the same device loop on the headline water system and on a 98,304-atom water box
    c8 = None
    if world == 1 and prec == b200dp.MIXED and not args.profile:
        try:
            c8 = {"model": "C8L2: 8 channels, lmax 2, 70 invariants, 70-96-96-96 SiLU fitting (random-init)",
                  "dtype": "f32 (the reference's precision for this model)", "unit": "atom-steps/s"}
            cp8 = model_path("c8l2")
            for label, sysf in (("c1_water_12288", systems.config1), ("c4_water_98k", lambda: systems.config4("98k"))):
                s8 = sysf()
                dp8 = b200dp.DeepPot(cp8, precision=b200dp.MIXED, device=local)
                w8 = Periodic(dp8, s8, dev, stream, torch)
                k8 = max(5, min(args.steps, 20))
                ms8, l8 = device_loop(dp8, w8, k8, max(3, min(args.warmup, 3)))
                st8 = stage_pass(dp8, w8, 3)
                c8[label] = {"value": s8.natoms * k8 / (ms8 / 1e3), "ms_per_step": ms8 / k8, "atoms": s8.natoms,
                             "steps": k8, "gpu_launches_per_step": int(l8 // k8),
                             "stage_ms": {k: round(float(q), 4) for k, q in
                                          zip(["neighbour", "descriptor_fwd", "fitting", "backward", "assembly"],
                                              st8)}}
                del w8
                dp8.close()
        except Exception as ex:  # report, never hide
            c8 = {"error": repr(ex)}
    # execution-window probe (N = 1): two independent force calls on two streams at once against one
    # after the other.  Windowed overlap of one call's stages (the reference's model_pipeline) can only
    # use the capacity that two whole calls running together find idle, so a ratio near 1 bounds it.
    overlap = None
    if world == 1 and prec == b200dp.MIXED and not args.profile and not args.no_strong:
        try:
            overlap = {"note": "throughput of two concurrent force calls (two engines, two streams, each replaying "
                               "its CUDA graph) over that of one call after the other; 1.0 = no idle capacity for "
                               "execution windows to use"}
            for label, sysf in (("c1_water_12288", systems.config1), ("c4_water_786k", lambda: systems.config4("786k"))):
                overlap[label] = overlap_probe(torch, b200dp, mp, sysf(), dev, local, flush)
        except Exception as ex:  # report, never hide
            overlap = {"error": repr(ex)[:400]}
    # strong scaling of the 3,145,728-atom water box (the same global system at every N): periodic on one
    # GPU, the decomposed driver on N; a secondary key beside the weak-scaling headline
    strong = None
    if not (args.no_strong or args.profile) and prec == b200dp.MIXED:
        import domain

        if hasattr(w, "release"):
            w.release()
        try:
            s3 = systems.config4("3.1M")
            g3 = domain.rank_grid(world)
            dp3 = b200dp.DeepPot(mp, precision=b200dp.MIXED, device=local)
            w3 = workload(dp3, s3, g3)
            k3 = 5
            ms3, _ = device_loop(dp3, w3, k3, 3)
            ms3 = max_over_ranks(ms3)
            strong = {"atoms": s3.natoms, "value": s3.natoms * k3 / (ms3 / 1e3), "unit": "atom-steps/s",
                      "ms_per_step": ms3 / k3, "steps": k3, "n_gpus": world, "grid": list(g3),
                      "scaling": "strong (the same 3.1M-atom system at every N)",
                      "driver": "periodic engine" if world == 1 else
                      ("C++ decomposed driver" if args.driver == "cpp" else "domain.py"),
                      "timing": "CUDA events per step, max over ranks, L2 flushed before each, step as a CUDA graph"}
            if hasattr(w3, "close"):
                w3.close()
            del w3
            dp3.close()
            torch.cuda.empty_cache()
        except Exception as ex:  # report, never hide
            strong = {"error": repr(ex)[:400]}
    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.profile):
        arm = OracleArm(mp)
        dt = min(arm.evaluate(system) for _ in range(2))
        cpu = {"value": system.natoms / dt, "unit": "atom-steps/s", "cores": arm.cores, "kind": "port",
               "sample": f"best of two full evaluations of the 12,288-atom system ({dt:.2f} s each), fp64 C++ "
                         "oracle, OpenMP, model loaded beforehand"}
    if world > 1 and args.driver == "cpp":
        parallelism = (f"C++ decomposed driver (b200dp_dd), domain decomposition {grid[0]}x{grid[1]}x{grid[2]}, "
                       f"halo {HALO} A: ghost rows gathered from the owners over NVLink peer memory, ghost forces "
                       "added into the owners' accumulators, device-side rendezvous for the barrier and the "
                       "energy/virial sum (no collective library per step), step replayed as one CUDA graph")
        cfg_extra = {"global_atoms": w.total, "ghosts_rank0": w.nghost}
    elif world > 1:
        rev = ("ghost forces added into the owners' accumulators over NVLink peer memory"
               if args.reverse == "peer" else "ghost forces folded back by NCCL send/recv")
        parallelism = (f"domain decomposition {grid[0]}x{grid[1]}x{grid[2]}, halo {HALO} A, coordinate halo by "
                       f"NCCL send/recv, {rev}, step replayed as one CUDA graph")
        cfg_extra = {"global_atoms": w.total, "ghosts_rank0": w.nghost}
    else:
        parallelism, cfg_extra = "single GPU, force call replayed as one CUDA graph", {}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "atom-steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32-mixed" if prec == b200dp.MIXED else "f64",
            "data": "synthetic (seeded water, random-init weights)",
            "config": bench_config(world),
            "setup": {"atoms_rank0": n, "edges_rank0": edges, "precision": args.precision,
                      "parallelism": parallelism, **cfg_extra},
            "stage_ms": {k: round(float(q), 4) for k, q in
                         zip(["neighbour", "descriptor_fwd", "fitting", "descriptor_bwd", "assembly"], stage_ms)},
            "stage_note": "stage times from a separate pass with the engine's stage events (rank 0)",
            "gpu_launches": int(launches),
            "roofline": roofline,
            "e2e": e2e,
            "fp64": fp64,
            "md_loop": md_loop,
            "c8l2": c8,
            "strong_3.1M": strong,
            "overlap_probe": overlap,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "flops_per_step": fl["total"],
        }
        print(json.dumps(line), flush=True)
    if hasattr(w, "close"):
        w.close()
    del w
    dp.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def e2e_loop(dp, w, system, steps, warmup, torch, dist):
    """Host buffers in, host buffers out: coordinates H2D and forces, energy, virial D2H every step."""
    import ctypes

    import b200dp

    if dist is not None:
        return e2e_decomposed(w, steps, warmup, torch, dist)
    n = system.natoms
    coord = torch.tensor(system.coord).pin_memory()
    atype = torch.tensor(system.atype).pin_memory()
    force = torch.zeros(n, 3, dtype=torch.float64).pin_memory()
    e = torch.zeros(1, dtype=torch.float64).pin_memory()
    v = torch.zeros(9, dtype=torch.float64).pin_memory()
    box = np.ascontiguousarray(system.box.reshape(9))
    L = dp.L
    dptr = ctypes.POINTER(ctypes.c_double)
    iptr = ctypes.POINTER(ctypes.c_int)

    def call():
        rc = L.b200dp_compute_host(dp.h, n, 0, ctypes.cast(coord.data_ptr(), dptr), ctypes.cast(atype.data_ptr(), iptr),
                                   box.ctypes.data_as(dptr), ctypes.cast(e.data_ptr(), dptr),
                                   ctypes.cast(force.data_ptr(), dptr), ctypes.cast(v.data_ptr(), dptr), None, None)
        if rc != 0:
            raise b200dp.B200DPError(rc, L.b200dp_last_error(dp.h).decode())

    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        call()
    dt = time.perf_counter() - t0
    return {"value": n * steps / dt, "unit": "atom-steps/s", "seconds": dt,
            "h2d_bytes_per_step": n * 3 * 8 + n * 4, "d2h_bytes_per_step": n * 3 * 8 + 8 * 10,
            "entry": "b200dp_compute_host (pinned host buffers, synchronous)"}


def e2e_decomposed(w, steps, warmup, torch, dist):
    """Per rank: owned coordinates from pinned host memory, owned forces and energy/virial back."""
    if isinstance(w, DecomposedCpp):
        return e2e_decomposed_cpp(w, steps, warmup, torch, dist)
    ddp = w.ddp
    n = ddp.nloc
    x_host = ddp.x[:n].cpu().pin_memory()
    f_host = torch.zeros(n, 3, dtype=torch.float64).pin_memory()
    ev_host = torch.zeros(10, dtype=torch.float64).pin_memory()

    def call():
        ddp.x[:n].copy_(x_host, non_blocking=True)
        e, f, v = ddp.step()
        f_host.copy_(f, non_blocking=True)
        ev_host.copy_(ddp.ev, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(warmup):
        call()
    ddp.capture()
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        call()
    dt = time.perf_counter() - t0
    ddp.release()
    return {"value": None, "unit": "atom-steps/s", "seconds": dt,
            "h2d_bytes_per_step": n * 3 * 8, "d2h_bytes_per_step": n * 3 * 8 + 8 * 10,
            "entry": "domain.DistributedDeepPot.step (captured CUDA graph) over "
                     + ("b200dp_compute_device_fold + b200dp_fold_finish" if ddp.fold is not None
                        else "b200dp_compute_device") + " (pinned host buffers, per rank)",
            "bytes_rank": "rank 0's own counts"}


def e2e_decomposed_cpp(w, steps, warmup, torch, dist):
    """The C++ driver through its C ABI: owned positions H2D from pinned memory, the step (replayed
    graph), owned forces and the global energy + virial D2H, every step."""
    dd = w.dd
    n = w.n
    _, x0, _, _ = dd.owned()
    x_host = torch.tensor(x0).pin_memory()
    f_host = torch.zeros(n, 3, dtype=torch.float64).pin_memory()
    ev_host = torch.zeros(10, dtype=torch.float64).pin_memory()
    st = w.stream.cuda_stream

    def call():
        dd.set_positions(st, x_host.data_ptr())
        w.step()
        dd.get_forces(st, f_host.data_ptr(), ev_host.data_ptr())
        w.stream.synchronize()

    for _ in range(warmup):
        call()
    w.capture()
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        call()
    dt = time.perf_counter() - t0
    w.release()
    return {"value": None, "unit": "atom-steps/s", "seconds": dt,
            "h2d_bytes_per_step": n * 3 * 8, "d2h_bytes_per_step": n * 3 * 8 + 8 * 10,
            "entry": "b200dp_dd_set_positions + b200dp_dd_force (captured CUDA graph) + b200dp_dd_get_forces "
                     "(pinned host buffers, per rank)",
            "bytes_rank": "rank 0's own counts"}


# ----------------------------------------------------------------- configuration sweep
MASSES = {"water": [15.9994, 1.00794], "cu": [63.546], "alloy": [55.845, 51.996, 58.693, 58.933]}


def sweep_table():
    """(label, system factory, model kind, force-call precisions, MD (ensemble, steps, T), GPU counts)."""
    c4 = lambda size: (lambda: systems.config4(size))  # noqa: E731
    return [
        ("c0_water_192", systems.config0, "water", ("fp64", "mixed"), None, (1,)),
        ("c1_water_12288", systems.config1, "water", ("fp64", "mixed"), ("nvt", 1000, 300.0), (1,)),
        ("c2_cu_131072", systems.config2, "cu", ("mixed",), ("npt", 500, 800.0), (1, 2)),
        ("c3_bcc_524288", systems.config3, "alloy", ("mixed",), ("nvt", 200, 300.0), (1, 2, 4, 8)),
        ("c4_water_1.5k", c4("1.5k"), "water", ("mixed",), ("nvt", 100, 300.0), (1,)),
        ("c4_water_12k", c4("12k"), "water", ("mixed",), ("nvt", 100, 300.0), (1,)),
        ("c4_water_98k", c4("98k"), "water", ("mixed",), ("nvt", 100, 300.0), (1,)),
        ("c4_water_786k", c4("786k"), "water", ("mixed",), ("nvt", 100, 300.0), (1, 2, 4, 8)),
        ("c4_water_3.1M", c4("3.1M"), "water", ("mixed",), ("nvt", 100, 300.0), (1, 2, 4, 8)),
        ("c4_water_786k-slab", c4("786k-slab"), "water", ("mixed",), ("nvt", 100, 300.0), (1, 2, 4, 8)),
    ]


def sweep_grid(label, world):
    """The slab's vacuum half holds no atoms: it is never split along z."""
    import domain

    if "slab" in label:
        return {1: (1, 1, 1), 2: (2, 1, 1), 4: (2, 2, 1), 8: (4, 2, 1)}.get(world, (world, 1, 1))
    return domain.rank_grid(world)


def timed_steps(torch, w, steps, warmup, dist, flush, stream, sync):
    """Device time of `steps` force calls (CUDA events on the launch stream, L2 flushed before each)."""
    for _ in range(warmup):
        w.step()
    if hasattr(w, "capture"):
        w.capture()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for k in range(steps):
        flush.fill_(k & 0xFF)
        if dist:
            dist.all_reduce(sync)
        starts[k].record(stream)
        w.step()
        ends[k].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    if hasattr(w, "release"):
        w.release()
    return sum(a.elapsed_time(b) for a, b in zip(starts, ends))


def run_sweep(args, world, rank, local):
    import datetime

    import torch

    import b200dp

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    sync = torch.zeros(1, device=dev)
    models = {}
    only = set(filter(None, args.only.split(",")))
    for label, sysf, kind, precisions, md_cfg, gpus in sweep_table():
        if world not in gpus or (only and label not in only):
            continue
        if kind not in models:
            models[kind] = model_path(kind)
        system = sysf()
        for prec_name in precisions:
            prec = b200dp.MIXED if prec_name == "mixed" else b200dp.FP64
            line = {"sweep": label, "n_gpus": world, "atoms": system.natoms, "precision": prec_name,
                    "model": kind, "unit": "atom-steps/s", "data": "synthetic (seeded system, random-init weights)"}
            try:
                dp = b200dp.DeepPot(models[kind], precision=prec, device=local)
                if world == 1:
                    w = Periodic(dp, system, dev, stream, torch)
                else:
                    grid = sweep_grid(label, world)
                    if args.driver == "cpp":
                        w = DecomposedCpp(dp, system, grid, rank, world, dev, stream, torch, dist)
                        line["parallelism"] = (f"C++ decomposed driver, {grid[0]}x{grid[1]}x{grid[2]}, peer memory, "
                                               "device-side rendezvous")
                    else:
                        w = Decomposed(dp, system, grid, rank, dev, stream, torch, peer_fold=args.reverse == "peer")
                        line["parallelism"] = f"domain.py decomposition {grid[0]}x{grid[1]}x{grid[2]}, peer fold"
                # about 2 s of timed work, at least 3 steps
                w.step()
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                w.step()
                torch.cuda.synchronize()
                one = time.perf_counter() - t0
                k = int(min(max(3, 2.0 / max(one, 1e-4)), 50))
                if dist:  # every rank runs the same number of steps
                    kk = torch.tensor([k], device=dev)
                    dist.all_reduce(kk, op=dist.ReduceOp.MIN)
                    k = int(kk.item())
                ms = timed_steps(torch, w, k, 3, dist, flush, stream, sync)
                if dist:
                    tt = torch.tensor([ms], dtype=torch.float64, device=dev)
                    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                    ms = float(tt.item())
                dp.check()
                line.update({"mode": "force call", "value": system.natoms * k / (ms / 1e3), "ms_per_step": ms / k,
                             "steps": k, "timing": "CUDA events per step, max over ranks, L2 flushed before each"})
                if hasattr(w, "close"):
                    w.close()
                del w
                dp.close()
            except Exception as ex:  # report, never hide
                line["error"] = repr(ex)[:400]
            if rank == 0:
                print(json.dumps(line), flush=True)
            torch.cuda.empty_cache()
        if md_cfg and world == 1:
            ens, nsteps, temp = md_cfg
            line = {"sweep": label, "n_gpus": 1, "atoms": system.natoms, "precision": "mixed", "model": kind,
                    "unit": "atom-steps/s", "mode": f"MD {ens.upper()} {nsteps} steps, dt 0.5 fs, {temp:g} K"
                    + (", 1 bar" if ens == "npt" else "") + ", candidates rebuilt every 10 steps (2 A skin)"}
            try:
                dp = b200dp.DeepPot(models[kind], precision=b200dp.MIXED, device=local)
                kw = dict(dt=0.0005, ensemble=b200dp.NPT if ens == "npt" else b200dp.NVT, t_init=temp,
                          t_target=temp, t_damp=0.05, seed=1, skin=2.0, rebuild_every=10)
                if ens == "npt":
                    kw.update(p_target=1.0, p_damp=0.5)
                md = b200dp.MD(dp, system.coord, system.atype, system.box, MASSES[kind], **kw)
                md.run(3)
                md.thermo()
                t0 = time.perf_counter()
                md.run(nsteps)
                th = md.thermo()
                dt = time.perf_counter() - t0
                line.update({"value": system.natoms * nsteps / dt, "ms_per_step": 1e3 * dt / nsteps,
                             "steps": nsteps, "temperature_K": th["temp"], "conserved": th["conserved"],
                             "timing": "host wall clock around the enqueued steps + final read"})
                md.close()
                dp.close()
            except Exception as ex:  # report, never hide
                line["error"] = repr(ex)[:400]
            print(json.dumps(line), flush=True)
            torch.cuda.empty_cache()
        if md_cfg and world > 1 and args.driver == "cpp":
            # MD over the decomposition (the C++ driver): atoms migrate and the ghost plan is rebuilt
            # every 10 steps; time = max over ranks of the host wall clock around the run
            ens, nsteps, temp = md_cfg
            grid = sweep_grid(label, world)
            line = {"sweep": label, "n_gpus": world, "atoms": system.natoms, "precision": "mixed", "model": kind,
                    "unit": "atom-steps/s",
                    "mode": f"decomposed MD {ens.upper()} {nsteps} steps, dt 0.5 fs, {temp:g} K"
                    + (", 1 bar" if ens == "npt" else "") + ", migration and ghost plan every 10 steps",
                    "parallelism": f"C++ decomposed driver, {grid[0]}x{grid[1]}x{grid[2]}"}
            try:
                dp = b200dp.DeepPot(models[kind], precision=b200dp.MIXED, device=local)
                w = DecomposedCpp(dp, system, grid, rank, world, dev, stream, torch, dist)
                kw = dict(dt=0.0005, ensemble=b200dp.NPT if ens == "npt" else b200dp.NVT, t_init=temp,
                          t_target=temp, t_damp=0.05, seed=1, rebuild_every=10)
                if ens == "npt":
                    kw.update(p_target=1.0, p_damp=0.5)
                w.dd.md_start(MASSES[kind], **kw)
                w.dd.md_run(3)
                w.dd.thermo()
                dist.barrier()
                t0 = time.perf_counter()
                w.dd.md_run(nsteps)
                th = w.dd.thermo()
                dt = time.perf_counter() - t0
                tt = torch.tensor([dt], dtype=torch.float64, device=dev)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                dt = float(tt.item())
                line.update({"value": system.natoms * nsteps / dt, "ms_per_step": 1e3 * dt / nsteps,
                             "steps": nsteps, "temperature_K": th["temp"], "conserved": th["conserved"],
                             "volume": th["volume"],
                             "timing": "host wall clock around the run + final read, max over ranks"})
                w.close()
                dp.close()
            except Exception as ex:  # report, never hide
                line["error"] = repr(ex)[:400]
            if rank == 0:
                print(json.dumps(line), flush=True)
            torch.cuda.empty_cache()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.sweep:
        run_sweep(args, world, rank, local)
        return
    run_b200dp(args, world, rank, local)


if __name__ == "__main__":
    main()
