"""Benchmark: eSCN-MD (uma-s-1 shape) energy + forces + stress, atom-steps/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (N = 1): the periodic 2,000-atom fcc Cu/Ni alloy (10x10x5 conventional cells,
a = 3.55 A, jitter 0.05 A, seed 1), uma-s-1 shape (128 channels, 4 layers, 512 Gaussians,
cutoff 6 A, at most 30 neighbours), random-init fp32 weights (seed 0).

* ``value``: atom-steps/s of the device step (geometry -> forward -> hand-written backward ->
  forces + virial) replayed from a CUDA graph with positions resident in HBM; timed with CUDA
  events over exactly K steps; the per-step working set (~10 GB) is far larger than L2.
* ``e2e``: the same metric through the public API (``TTAtomCalculator.calculate``, trace=True): host
  positions -> H2D copy -> GPU neighbour list -> step -> D2H of energy, forces, stress.
* Multi-GPU (torchrun, N ranks): each rank runs its own replica structure (independent
  systems, no collective on the data path); value = all ranks' atoms x steps / max-over-ranks
  time ("scaling": "weak").
* The same launch also measures, at the same N, the two partitioned configurations and adds
  them as keys of the line: ``screen`` (config 4: 512 molecules dealt over the ranks, no
  collectives, through ``evaluate_batch``) and ``slab`` (config 5: the 65,536-atom bcc Fe cell
  slab-decomposed over the ranks, NCCL halo exchange per layer and an all-reduce of energy and
  virial, with the collectives' CUDA-event time per step and the limiting one named).
* ``orb``: config 3 (Orb-v3 shape, 1,002-atom SiO2) at the same N, device step and end to end.
* ``md``: GPU-resident Langevin MD on the config-2 cell (neighbour list rebuilt every step).
* ``--impl reference``: the reference's CPU path (this repo's CPU restatement of it, the oracle)
  on the box's host cores, on the same full workload, median of the timed steps.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "tt-atom_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "atom-steps/s (E+F+stress)"
WORKLOADS = {
    "uma": "uma-s-1-shape eSCN-MD, periodic 2000-atom fcc Cu/Ni, E+F+stress",
    "orb": "Orb-v3-conservative-shape GNN, periodic 1002-atom amorphous SiO2, E+F+stress",
    "fe65k": "uma-s-1-shape eSCN-MD, periodic 65536-atom bcc Fe, slab-decomposed, E+F+stress",
    "screen": "uma-s-1-shape eSCN-MD, 512 molecules (10-60 atoms) partitioned over GPUs, E+F",
}
DATA = {
    "uma": "synthetic (seeded fcc Cu/Ni, random-init weights)",
    "orb": "synthetic (seeded amorphous SiO2, random-init weights)",
    "fe65k": "synthetic (seeded bcc Fe, random-init weights)",
    "screen": "synthetic (seeded molecules, random-init weights)",
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class _SmiSampler:
    """nvidia-smi clock / throttle sampling (fallback when NVML bindings are missing)."""

    def __init__(self, index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


class ClockSampler:
    """SM clock, max clock and clock-event (throttle) reasons of this rank's GPU, polled every
    10 ms through NVML (read-only queries) in a background thread while the timed region runs.
    The constructor returns once the first sample is taken, so even a short timed region is
    covered; ``stop`` adds a final sample."""

    _REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
                ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
                ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
                ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4))

    def __new__(cls, index):
        try:
            import pynvml  # noqa: F401
        except ImportError:
            return _SmiSampler(index)
        return super().__new__(cls)

    def __init__(self, index):
        import threading

        import pynvml as nv
        self.nv = nv
        nv.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(index).uuid)
            self.h = nv.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
        except Exception:
            self.h = nv.nvmlDeviceGetHandleByIndex(index)
        self.bits = [(nm, getattr(nv, attr, val)) for nm, attr, val in self._REASONS]
        self.sm, self.reasons = [], set()
        self.mx = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
        self.done = threading.Event()
        self._sample()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _sample(self):
        nv = self.nv
        self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
        try:
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except AttributeError:
            r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        for nm, bit in self.bits:
            if r & bit:
                self.reasons.add(nm)

    def _run(self):
        while not self.done.wait(0.01):
            self._sample()

    def stop(self):
        self._sample()
        self.done.set()
        self.t.join()
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": float(self.mx),
                "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml"}


def make_workload(device, cells=(10, 10, 5), precision="3xtf32"):
    from tt_atom import configs
    from tt_atom.calculator import TTAtomCalculator
    from tt_atom.weights import WeightBundle
    cfg = configs.model_config("uma-s-1")
    bundle = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.fcc_alloy(reps=cells)
    calc = TTAtomCalculator(bundle, device=device, precision=precision)
    return cfg, bundle, s, calc


def init_dist():
    """(world size, rank, local rank, device): one process per GPU, NCCL when N > 1."""
    ws_n, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws_n > 1:
        import torch.distributed as dist
        if not dist.is_initialized():
            dist.init_process_group("nccl", device_id=device)
    return ws_n, rank, local, device


def _max_over_ranks(values, device, ws_n):
    t = torch.tensor(values, device=device, dtype=torch.float64)
    if ws_n > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def _barrier(ws_n):
    torch.cuda.synchronize()
    if ws_n > 1:
        import torch.distributed as dist
        dist.barrier()


def measure_slab(args, steps, warmup):
    """Config 5: one 65,536-atom cell split into slabs over the ranks, halo exchange per layer
    (NCCL point-to-point), energy and virial all-reduced; value = atoms x steps / max time.
    The halo exchanges and the all-reduce are timed with CUDA events on the compute stream
    (each exchange's span includes waiting for the slowest peer). Returns rank 0's dict."""
    import torch.distributed as dist
    from tt_atom import configs
    from tt_atom.engine import UMAEngine
    from tt_atom.graph import build_graph, csd_embedding
    from tt_atom.slab import DistExchange, local_graph, plans_for, run_partition, slab_order
    from tt_atom.weights import WeightBundle
    ws_n, rank, local, device = init_dist()
    cfg = configs.model_config("uma-s-1")
    b = WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0))
    s = configs.bcc_iron()
    perm, ranges = slab_order(s["pos"], s["cell"], ws_n)
    pos = torch.from_numpy(s["pos"][perm]).to(device)
    torch.cuda.synchronize()
    t_nl = time.perf_counter()
    g = build_graph(pos, s["Z"][perm], cfg["cutoff"], s["cell"], [True] * 3,
                    max_neighbors=cfg["max_neighbors"], device=device)
    torch.cuda.synchronize()
    t_nl = time.perf_counter() - t_nl
    plan = plans_for(g, ranges)[rank]
    lg = local_graph(g, plan)
    E_total = g.E
    del g
    eng = UMAEngine(b.weights, cfg, b.tables(), device=device, precision=args.precision)
    se = csd_embedding(b.weights, [0.0], [0.0], cfg["sphere_channels"])
    # one GPU cannot hold the full per-edge workspace of 1.97M edges: run the edge stages over
    # receiver chunks (recomputed in the reverse pass); ranks of a partitioned run fit whole
    chunk = args.chunk_edges if args.chunk_edges > 0 else (262144 if ws_n == 1 else None)
    ws = eng.workspace(lg, se, chunk_edges=chunk)
    ws.pos.copy_(pos[plan.global_ids.to(device)])
    exch = DistExchange(plan, timed=True)
    red = torch.zeros(10, device=device, dtype=torch.float64)
    ar_events = []

    def step(timed=False):
        run_partition(eng, ws, exch, forces=True, virial=True)
        red[0] = ws.energy[0]
        red[1:] = ws.virial.reshape(-1)
        if ws_n > 1:
            if timed:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            dist.all_reduce(red)
            if timed:
                e1.record()
                ar_events.append((e0, e1))
    for _ in range(warmup):
        step()
    _barrier(ws_n)
    exch.reset_timing()
    clk = ClockSampler(local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step(timed=True)
    t1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms = t0.elapsed_time(t1)
    halo = exch.timing_ms()
    ar_ms = sum(a.elapsed_time(b_) for a, b_ in ar_events)
    ms, halo_fwd, halo_rev, ar_ms = _max_over_ranks(
        [ms, halo["forward"], halo["reverse"], ar_ms], device, ws_n)
    N = len(s["Z"])
    per = lambda v: v / steps  # noqa: E731
    out = {"metric": METRIC, "value": N * steps / (ms / 1e3), "unit": "atom-steps/s",
           "n_gpus": ws_n, "steps": steps, "warmup": warmup, "ms_per_step": ms / steps,
           "scaling": "strong", "dtype": "fp32",
           "data": "synthetic (seeded bcc Fe, random-init weights)",
           "config": {"workload": WORKLOADS["fe65k"], "atoms": N, "edges": E_total,
                      "edges_rank0": lg.E, "halo_rank0": plan.n_halo,
                      "precision": args.precision, "parallelism": f"slab x{ws_n}",
                      "chunk_edges": chunk, "chunks": len(ws.chunks) if ws.chunks else None,
                      "workspace_GB_rank0": round(ws.nbytes() / 1e9, 1)},
           "energy": float(red[0]), "clocks": clocks,
           # CUDA-event spans on the compute stream per step, max over ranks; a halo span
           # includes waiting for the slowest peer to reach the exchange
           "collectives_ms_per_step": {
               "halo_forward": per(halo_fwd), "halo_reverse": per(halo_rev),
               "energy_virial_allreduce": per(ar_ms),
               "exchanges_per_step": exch.count_per_step(steps),
               "halo_bytes_per_layer_rank0": plan.n_halo * 9 * cfg["sphere_channels"] * 4},
           "neighbor_list_s": round(t_nl, 3)}
    lim = max(("halo_forward", per(halo_fwd)), ("halo_reverse", per(halo_rev)),
              ("energy_virial_allreduce", per(ar_ms)), key=lambda kv: kv[1])
    out["collectives_ms_per_step"]["limiting"] = lim[0] if ws_n > 1 else None
    del ws, eng, lg, plan
    torch.cuda.empty_cache()
    return out


def measure_screen(args, steps, warmup):
    """Config 4: 512 independent molecules split over the ranks (no collective on the data
    path); each rank evaluates its share as disjoint-union batches through the public
    ``evaluate_batch``. A step is one pass over all 512 molecules; value = total atoms / max
    over ranks of the step time. Returns rank 0's dict."""
    from tt_atom import configs
    from tt_atom.calculator import TTAtomCalculator
    from tt_atom.weights import WeightBundle
    ws_n, rank, local, device = init_dist()
    cfg = configs.model_config("uma-s-1")
    calc = TTAtomCalculator(WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0)),
                            device=device, precision=args.precision)
    mols = configs.screening_set()
    # partition: molecules sorted by size and dealt round-robin, so ranks get equal work
    order = sorted(range(len(mols)), key=lambda i: -len(mols[i]["Z"]))
    mine = [mols[i] for i in order[rank::ws_n]]
    bs = 64
    batches = [mine[i:i + bs] for i in range(0, len(mine), bs)]

    def step():
        for bt in batches:
            calc.evaluate_batch(bt)
    for _ in range(warmup):
        step()
    _barrier(ws_n)
    clk = ClockSampler(local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    (ms,) = _max_over_ranks([t0.elapsed_time(t1)], device, ws_n)
    N = sum(len(m["Z"]) for m in mols)
    out = {"metric": "atom-steps/s (E+F)", "value": N * steps / (ms / 1e3),
           "unit": "atom-steps/s", "n_gpus": ws_n, "steps": steps, "warmup": warmup,
           "ms_per_step": ms / steps, "scaling": "strong", "dtype": "fp32",
           "data": "synthetic (seeded molecules, random-init weights)",
           "config": {"workload": WORKLOADS["screen"], "molecules": len(mols), "atoms": N,
                      "batch": bs, "precision": args.precision,
                      "parallelism": f"partition x{ws_n}, no collectives",
                      "timing": "end to end through evaluate_batch (host inputs, GPU "
                                "neighbour lists, host results)"},
           "clocks": clocks}
    calc.close()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def measure_orb(args, steps, warmup):
    """Config 3 at this N (replicas): the Orb-v3-shape 1,002-atom SiO2 step replayed from a
    CUDA graph (value), end to end through ``OrbCalculator.calculate`` (e2e), and the
    edge-MLP hidden GEMM's tensor roofline. Returns rank 0's dict."""
    from tt_atom import configs
    from tt_atom.ase_compat import SimpleAtoms
    from tt_atom.engine import CapturedStep
    from tt_atom.orb import OrbCalculator
    ws_n, rank, local, device = init_dist()
    cfg = configs.orb_config("orb-v3")
    s = configs.amorphous_sio2()
    calc = OrbCalculator(configs.orb_random_weights(cfg, seed=0), cfg=cfg, device=device,
                         precision=args.precision)
    calc._evaluate(s["pos"], s["Z"], s["cell"], [True] * 3, True, True)
    ws, eng = calc._ws, calc.engine
    step = CapturedStep(eng, ws, forces=True, virial=True)
    for _ in range(warmup):
        step()
    _barrier(ws_n)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    kern = eng.time_kernels(ws, reps=3)
    calc.trace = True
    atoms = SimpleAtoms(s["Z"], s["pos"], s["cell"], True)
    rng = np.random.default_rng(99)
    jit = [SimpleAtoms(s["Z"], s["pos"] + rng.normal(0.0, 0.01, s["pos"].shape), s["cell"], True)
           for _ in range(steps)]
    for _ in range(max(1, warmup)):
        calc.calculate(atoms, ("energy", "forces", "stress"))
    torch.cuda.synchronize()
    te = time.perf_counter()
    for a in jit:
        calc.calculate(a, ("energy", "forces", "stress"))
    e2e_ms = 1e3 * (time.perf_counter() - te) / len(jit)
    ms, e2e_ms = _max_over_ranks([ms, e2e_ms], device, ws_n)
    N = len(s["Z"])
    _, bf16, src = peaks()
    ach = kern["flop"] / (kern["ms"] / 1e3) / 1e12
    out = {"metric": METRIC, "value": N * ws_n * steps / (ms / 1e3), "unit": "atom-steps/s",
           "n_gpus": ws_n, "steps": steps, "warmup": warmup, "ms_per_step": ms / steps,
           "scaling": "weak", "dtype": "fp32", "data": DATA["orb"],
           "config": workload_config("orb", N, ws.graph.E,
                                     dict(cfg, max_neighbors=cfg["max_num_neighbors"]), ws_n),
           "e2e": {"value": N * ws_n / (e2e_ms / 1e3), "unit": "atom-steps/s",
                   "h2d_bytes_per_step": N * 3 * 4 + N * 8,
                   "d2h_bytes_per_step": 8 + N * 3 * 8 + 9 * 8},
           "roofline": {"bound": "tensor", "kernel": kern["name"], "achieved": ach,
                        "peak": bf16, "unit": "TFLOP/s", "frac": ach / bf16,
                        "peak_source": f"{src} bf16 dense (MEASURED_PEAKS.json)",
                        "launch_ms": kern["ms"]}}
    calc.close()
    del step, ws, eng
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def measure_tiny(args, steps, warmup):
    """Config 1 (the reference's CPU-runnable case): the tiny eSCN-MD model on the 24-atom
    molecule, energy + forces, device step replayed from a CUDA graph and end to end through
    ``calculate``. Launch-bound at this size; reported for completeness."""
    from tt_atom import configs
    from tt_atom.ase_compat import SimpleAtoms
    from tt_atom.calculator import TTAtomCalculator
    from tt_atom.engine import CapturedStep
    from tt_atom.weights import WeightBundle
    ws_n, rank, local, device = init_dist()
    cfg = configs.model_config("tiny")
    calc = TTAtomCalculator(WeightBundle.from_arrays(configs.random_bundle_arrays(cfg, seed=0)),
                            device=device, precision=args.precision)
    m = configs.tiny_molecule(seed=0)
    calc._evaluate(m["pos"], m["Z"], None, None, [0.0], [0.0], forces=True)
    step = CapturedStep(calc.engine, calc._ws, forces=True, virial=False)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    calc.trace = True
    atoms = SimpleAtoms(m["Z"], m["pos"])
    for _ in range(max(1, warmup)):
        calc.calculate(atoms)
    te = time.perf_counter()
    for _ in range(steps):
        calc.calculate(atoms)
    e2e_ms = 1e3 * (time.perf_counter() - te) / steps
    ms, e2e_ms = _max_over_ranks([ms, e2e_ms], device, ws_n)
    N = len(m["Z"])
    calc.close()
    return {"metric": "atom-steps/s (E+F)", "value": N * ws_n * steps / (ms / 1e3),
            "unit": "atom-steps/s", "ms_per_step": ms / steps, "steps": steps,
            "config": {"workload": "tiny eSCN-MD (16 channels, 2 layers), 24-atom molecule, E+F",
                       "atoms_per_gpu": N, "edges_per_gpu": calc_edges(m, cfg)},
            "e2e": {"value": N * ws_n / (e2e_ms / 1e3), "unit": "atom-steps/s"}}


def calc_edges(m, cfg):
    from tt_atom.graph import build_graph
    return build_graph(m["pos"], m["Z"], cfg["cutoff"], max_neighbors=cfg.get("max_neighbors")).E


def run_standalone(args, measure):
    out = measure(args, args.steps, args.warmup)
    ws_n, rank, _ = dist_env()
    if rank == 0:
        out.update(higher_is_better=True, vs_baseline=None)
        print(json.dumps(out))
    if ws_n > 1:
        torch.distributed.destroy_process_group()


def run_ours(args):
    ws_n, rank, local, device = init_dist()
    from tt_atom.ase_compat import SimpleAtoms
    from tt_atom.engine import CapturedStep
    cells = tuple(int(v) for v in args.cells.split(","))
    if args.workload == "orb":
        from tt_atom import configs
        from tt_atom.orb import OrbCalculator
        cfg = configs.orb_config("orb-v3")
        s = configs.amorphous_sio2()
        calc = OrbCalculator(configs.orb_random_weights(cfg, seed=0), cfg=cfg, device=device,
                             precision=args.precision)
        cfg = dict(cfg, max_neighbors=cfg["max_num_neighbors"])
        evaluate = lambda: calc._evaluate(s["pos"], s["Z"], s["cell"], [True] * 3, True, True)  # noqa: E731
    else:
        cfg, bundle, s, calc = make_workload(device, cells, args.precision)
        evaluate = lambda: calc._evaluate(s["pos"], s["Z"], s["cell"], [True] * 3, [0.0], [0.0],  # noqa: E731
                                          forces=True, stress=True)
    N = len(s["Z"])
    cell, pbc = s["cell"], [True] * 3
    # positions re-jittered every step (0.01 A, seeded): each step evaluates new coordinates
    rng = np.random.default_rng(1234)
    jit = [(s["pos"] + rng.normal(0.0, 0.01, s["pos"].shape)).astype(np.float32)
           for _ in range(max(args.steps, 1))]
    # ---- device step on a fixed topology (CUDA graph), positions resident in HBM
    evaluate()
    ws = calc._ws
    eng = calc.engine
    step = CapturedStep(eng, ws, forces=True, virial=True)
    pos_dev = torch.from_numpy(np.stack(jit)).to(device)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if args.profile_one_step:
        # one captured step between profiler start / stop (ncu --profile-from-start off)
        torch.cuda.profiler.start()
        ws.pos.copy_(pos_dev[0])
        step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"profiled": "one captured step", "launches_per_step":
                          eng.launches_per_step(ws)}))
        return
    if ws_n > 1:
        torch.distributed.barrier()
    clk = ClockSampler(local)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for k in range(args.steps):
        ws.pos.copy_(pos_dev[k])
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    clocks = clk.stop()
    # ---- dominant kernel, timed live with CUDA events on its own stream
    kern = eng.time_kernels(ws, reps=3)
    edge = eng.time_edge_kernel(ws, reps=3) if hasattr(eng, "time_edge_kernel") else None
    edge_all = (eng.time_edge_kernels(ws, reps=5) if hasattr(eng, "time_edge_kernels")
                and ws.chunks is None else None)
    # ---- end to end through the public API (host positions in, host results out)
    atoms = SimpleAtoms(s["Z"], s["pos"], cell, True)
    # the calculator's trace option (the reference's Calculator(trace=True)): the step is
    # captured as a CUDA graph per topology and replayed while the neighbour list is unchanged
    calc.trace = True
    atoms.calc = calc
    for _ in range(max(1, args.warmup)):
        calc.calculate(atoms, ("energy", "forces", "stress"))
    torch.cuda.synchronize()
    e2e_steps = max(3, min(args.steps, 20))
    jit_atoms = [SimpleAtoms(s["Z"], jit[k % len(jit)], cell, True) for k in range(e2e_steps)]
    te = time.perf_counter()
    for a in jit_atoms:
        # host positions in; the neighbour list is rebuilt and compared on every call
        calc.calculate(a, ("energy", "forces", "stress"))
    te = time.perf_counter() - te
    e2e_ms = 1e3 * te / e2e_steps
    md = None
    if args.workload == "uma":
        # GPU-resident Langevin MD on the same cell: every step rebuilds the neighbour list on
        # the device inside the captured step and reads back one status word
        from tt_atom.simulate import md_atoms
        md_a = SimpleAtoms(s["Z"], s["pos"], cell, True)
        md_a.calc = calc
        md_atoms(md_a, steps=3, dt=1.0, temp=300.0, seed=1, native=True)
        md_steps = 20
        torch.cuda.synchronize()
        tm = time.perf_counter()
        md_atoms(md_a, steps=md_steps, dt=1.0, temp=300.0, seed=2, native=True)
        torch.cuda.synchronize()
        tm = 1e3 * (time.perf_counter() - tm) / (md_steps + 1)   # +1: the initial force call
        md = {"unit": "atom-steps/s", "steps": md_steps,
              "integrator": "BAOAB Langevin, 1 fs, 300 K, GPU-resident",
              "timing": "host wall clock around the loop (one status read-back per step), "
                        "max over ranks; every rank runs its own replica"}
    ms, e2e_ms, tm = _max_over_ranks([ms, e2e_ms, tm if md is not None else 0.0], device, ws_n)
    if md is not None:
        md.update(value=N * ws_n / (tm / 1e3), ms_per_step=tm)
    eng_precision = {0: "fp32", 1: "tf32", 2: "3xtf32", 3: "3xf16"}[eng.precision]
    ms_step = ms / args.steps
    value = N * ws_n * args.steps / (ms / 1e3)
    hbm, bf16, src = peaks()
    achieved = kern["flop"] / (kern["ms"] / 1e3) / 1e12
    traffic = None
    prof = ROOT / "profiles" / "traffic.json"
    if prof.exists():
        traffic = json.loads(prof.read_text()).get(kern["name"])
    out = {
        "metric": METRIC, "value": value, "unit": "atom-steps/s", "n_gpus": ws_n,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": DATA[args.workload],
        "config": workload_config(args.workload, N, ws.graph.E, cfg, ws_n),
        "precision": eng_precision,
        "workspace_GB": round(ws.nbytes() / 1e9, 2),
        "e2e": {"value": N * ws_n / (e2e_ms / 1e3), "unit": "atom-steps/s",
                "h2d_bytes_per_step": N * 3 * 4 + N * 8,
                "d2h_bytes_per_step": 8 + N * 3 * 8 + 9 * 8},
        "gpu_launches": eng.launches_per_step(ws) * args.steps,
        "md": md,
        "roofline": {"bound": "tensor", "kernel": kern["name"], "achieved": achieved,
                     "peak": bf16, "unit": "TFLOP/s", "frac": achieved / bf16,
                     "peak_source": f"{src} bf16 dense (MEASURED_PEAKS.json)",
                     "traffic": traffic, "launch_ms": kern["ms"], "flop_per_launch": kern["flop"],
                     # the split modes issue three MMAs per product (hi*hi, hi*lo, lo*hi): the
                     # tensor pipe does 3x the algorithmic FLOPs, at tf32 rate (3xTF32) or at
                     # f16 rate (fp16 pair)
                     "mma_products": 3 if eng.precision in (2, 3) else 1,
                     "mma_work_tflops": achieved * (3 if eng.precision in (2, 3) else 1)},
        "clocks": clocks,
    }
    if edge is not None:
        # the HBM-bound edge kernel beside the tensor-bound GEMM (algorithmic bytes / event time)
        ach = edge["bytes"] / (edge["ms"] / 1e3) / 1e9
        out["roofline_edge"] = {"bound": "hbm", "kernel": edge["name"], "achieved": ach,
                                "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                                "peak_source": f"{src} HBM copy (MEASURED_PEAKS.json)",
                                "launch_ms": edge["ms"], "bytes_per_launch": edge["bytes"]}
    if edge_all is not None:
        # every HBM-bound edge kernel of layer 0 (forward and reverse) against the HBM roofline
        out["edge_kernels"] = [dict(k, frac=k["gbs"] / hbm) for k in edge_all]
    if cells != (10, 10, 5):
        out["config"]["workload"] += f" (reduced: {cells} cells, not the headline size)"
    out["positions"] = "re-jittered every step (0.01 A)"
    # release this workload's buffers and captured graphs before the next measurements
    calc.close()
    del step, ws, eng, pos_dev
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if args.workload == "uma" and not args.no_partitioned:
        # the partitioned configurations at this N, from the same launch: config 4 (screening,
        # no collectives) and config 5 (65,536-atom slab, halo exchange + all-reduce)
        out["screen"] = measure_screen(args, steps=5, warmup=2)
        out["slab"] = measure_slab(args, steps=3, warmup=2)
        # config 3 (Orb-v3 shape) at this N, from the same launch
        out["orb"] = measure_orb(args, steps=20, warmup=3)
        out["tiny"] = measure_tiny(args, steps=20, warmup=3)        # config 1
    if rank == 0:
        if not args.no_cpu and ws_n == 1:        # the CPU baseline leg runs at N = 1 only
            cpu = cpu_baseline(bounded=True, workload=args.workload)
            cpu.pop("cfg")
            out["cpu_baseline"] = cpu
        print(json.dumps(out))
    if ws_n > 1:
        torch.distributed.destroy_process_group()


def workload_config(workload, atoms, edges, cfg, ws_n):
    """The ``config`` object of both arms (this build's and the reference's): the same keys
    and values for the same workload, so the two lines describe one configuration."""
    return {"workload": WORKLOADS[workload], "atoms_per_gpu": atoms, "edges_per_gpu": edges,
            "cutoff": cfg["cutoff"], "max_neighbors": cfg["max_neighbors"],
            "parallelism": f"replicas x{ws_n}",
            "l2": "inputs larger than L2: the per-step working set (GBs) exceeds the 126 MB "
                  "L2, no flush"}


def _cpu_sample_orb():
    """The CPU baseline's Orb workload: config 3 itself (1,002-atom SiO2 at 2.2 g/cm^3)."""
    from tt_atom import configs
    cfg = configs.orb_config("orb-v3")
    return cfg, configs.orb_random_weights(cfg, seed=0), configs.amorphous_sio2()


def _cpu_sample():
    """The CPU baseline's UMA workload: config 2 itself (10x10x5 fcc cells, 2,000 atoms, the
    same model, weights and cap as the device arm)."""
    from tt_atom import configs
    cfg = configs.model_config("uma-s-1")
    arrs = configs.random_bundle_arrays(cfg, seed=0)
    s = configs.fcc_alloy(reps=(10, 10, 5), seed=1)
    return cfg, arrs, s


def cpu_baseline(bounded=True, steps=3, warmup=1, workload="uma"):
    if workload == "orb":
        return _cpu_baseline_orb(steps, warmup)
    from oracle import uma as O
    from tt_atom import configs
    from tt_atom.weights import WeightBundle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg, arrs, s = _cpu_sample()
    w = WeightBundle.from_arrays(arrs).weights
    t = configs.lmax2_tables()
    off, coeff = configs.gaussian_basis(cfg)
    tables = dict(t, gauss_offset=off, gauss_coeff=coeff)
    pos = torch.from_numpy(s["pos"])
    cell = torch.from_numpy(s["cell"])

    edges = [0]

    def one():
        ei, sh = O.neighbor_list(pos, cfg["cutoff"], cell, [True] * 3, cfg["max_neighbors"])
        edges[0] = int(ei.shape[1])
        return O.energy_forces(w, cfg, tables, pos, torch.from_numpy(s["Z"]), ei, sh,
                               compute_stress=True)
    for _ in range(warmup):
        one()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    n = len(s["Z"])
    v = n / statistics.median(times)
    return {"value": v, "unit": "atom-steps/s", "cores": threads, "kind": "port",
            "sample": f"the full workload: {n}-atom fcc Cu/Ni (10x10x5 cells), same model, "
                      f"weights and cap, neighbour list + E+F+stress per step, median of "
                      f"{steps} step(s) after {warmup} warm-up",
            "seconds_per_step": statistics.median(times), "atoms": n, "edges": edges[0],
            "cfg": cfg}


def _cpu_baseline_orb(steps, warmup):
    from oracle import orb as OB
    from oracle import uma as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg, w, s = _cpu_sample_orb()
    pos, cell = torch.from_numpy(s["pos"]), torch.from_numpy(s["cell"])

    edges = [0]

    def one():
        ei, sh = O.neighbor_list(pos, cfg["cutoff"], cell, [True] * 3, cfg["max_num_neighbors"])
        edges[0] = int(ei.shape[1])
        return OB.energy_forces(w, cfg, pos, torch.from_numpy(s["Z"]), ei, sh,
                                compute_stress=True)
    for _ in range(warmup):
        one()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    n = len(s["Z"])
    return {"value": n / statistics.median(times), "unit": "atom-steps/s", "cores": threads,
            "kind": "port", "sample": f"the full workload: {n}-atom amorphous SiO2, same "
                                      f"model, weights and cap, neighbour list + E+F+stress "
                                      f"per step, median of {steps} step(s) after {warmup} "
                                      f"warm-up",
            "seconds_per_step": statistics.median(times), "atoms": n, "edges": edges[0],
            "cfg": dict(cfg, max_neighbors=cfg["max_num_neighbors"])}


def run_reference(args):
    ws_n, rank, _ = dist_env()
    if rank != 0:
        return
    steps = args.steps
    cpu = cpu_baseline(bounded=True, steps=steps, warmup=args.warmup, workload=args.workload)
    cfg = cpu.pop("cfg")
    out = {"metric": METRIC, "value": cpu["value"], "unit": "atom-steps/s", "n_gpus": ws_n,
           "steps": steps, "warmup": args.warmup,
           "ms_per_step": 1e3 * cpu["seconds_per_step"], "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
           "data": DATA[args.workload],
           "config": workload_config(args.workload, cpu["atoms"], cpu["edges"], cfg, ws_n),
           "precision": "fp32 (torch CPU)",
           "impl": "reference", "cpu_baseline": cpu,
           "e2e": {"value": cpu["value"], "unit": "atom-steps/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cells", default="10,10,5", help="fcc cells (profiling uses a smaller cell)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--profile-one-step", action="store_true",
                    help="profile exactly one captured step (for ncu --profile-from-start off)")
    ap.add_argument("--no-partitioned", action="store_true",
                    help="uma workload: skip the config-4 / config-5 measurements")
    ap.add_argument("--precision", default="3xtf32", choices=["3xtf32", "3xf16", "fp32", "tf32"])
    ap.add_argument("--chunk-edges", type=int, default=0,
                    help="fe65k: receiver-chunk size of the edge stages (0: automatic, chunked "
                         "on one GPU only)")
    ap.add_argument("--workload", default="uma", choices=sorted(WORKLOADS),
                    help="uma: config 2 (the headline); orb: config 3; fe65k: config 5; screen: config 4")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "fe65k":
        run_standalone(args, measure_slab)
    elif args.workload == "screen":
        run_standalone(args, measure_screen)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
