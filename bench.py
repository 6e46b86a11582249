"""Throughput benchmark: atom-steps/s for PET energy + forces + stress.

Default workload (the configuration the headline metric is quoted on): the
periodic random fcc alloy of 32^3 primitive cells (32,768 atoms, triclinic
cell, a = 3.6 A, 20 random elements among Z = 1..89, jitter N(0, 0.08 A))
with random-init pet-oam-l-shaped weights (d_pet 512, 16 heads, d_ff 1024,
d_head 256, cutoff 4.5 A); seeded synthetic data.  One step = one
prediction of energy, forces and stress: neighbour list, featuriser, both
GNN layers, readout and the full backward pass.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload fcc|si216|water|molecules|si] [--precision f32|f16]
                  [--mode forces|energy|nc]

Other workloads (one JSON line each; pet-mad-s-shaped weights):
  si216      diamond Si 3x3x3 (216 atoms), E+F+stress
  water      liquid water, 4,096 atoms, E+F+stress
  molecules  512 non-periodic molecules of 10-60 atoms, E+F, one batched
             call on the packed batch (predict_packed; structures sharded
             over the ranks for N > 1)
  si         diamond Si 32^3 (262,144 atoms), E+F+stress, spatial domains
             over N >= 2 GPUs (strong scaling)

Timing.  Every timed step is one public predict call from host arrays.
`e2e` is the host clock around it: the host-to-device copy of the inputs, the
step, and the device-to-host copy of the forces and stress.  `value` is the
same call's device time with its inputs already in HBM: the library's CUDA
events, recorded on its stream, from the end of its input copy to the start
of its result copy.  On the spatial-domain path it is the domain engine's
events around its step.  So e2e <= value holds call by call.  Multi-GPU
(launched with torch.distributed.run): barriers around the timed region and
the max over ranks.  With --gpus N > 1 the fcc workload is weak scaling at
32,768 atoms per GPU (one cell of N x 32,768 atoms split into spatial
domains).

`--impl reference` times the CPU implementation of the path on the host
cores: the reference's model cannot be built here (its ggml dependency is
absent), so this is the PyTorch restatement in oracle/ at float32.
"""
import argparse
import importlib.util
import json
import math
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "atom-steps/s (E+F+stress), 32k-atom PET cell, 1/2/4/8 B200; % of roofline"
L2_BYTES = 126 << 20


def _package():
    if "mlipcpp_b200" in sys.modules:
        return sys.modules["mlipcpp_b200"]
    pkg_dir = os.path.join(ROOT, "mlip.cpp_b200")
    spec = importlib.util.spec_from_file_location(
        "mlipcpp_b200", os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mlipcpp_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.first = 0
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # the sampler is live before the timed region starts: its first
            # sample (taken at start-up, before the region) is set aside
            t0 = time.time()
            while not self.rows and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.first = len(self.rows)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        # samples from inside the timed region; a region shorter than the
        # 200 ms period may hold none, and then the sample taken just before
        # it is reported and flagged
        rows, before = self.rows[self.first:], False
        if not rows and self.rows:
            rows, before = self.rows[-1:], True
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows if len(r) > 8
                          for k in range(4) if r[5 + k].lower() == "active"})
        out = {"sm_mhz": float(np.median(sm)) if sm else None,
               "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}
        if before:
            out["sampled_before_region"] = True
        return out


def cpu_reference(structures, gguf_path, steps, warmup, repeats=1, forces=True, nc=False):
    """Time the CPU implementation of the path (float32, all host threads)
    on `structures` (one batched predict per step): `warmup` untimed steps,
    then `repeats` runs of `steps` steps each, timed with the host clock.
    Returns (median atom-steps/s, threads, median per-step seconds,
    [atom-steps/s of every run])."""
    import torch
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import pet_oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    orc = pet_oracle.load_oracle(gguf_path, torch.float32)
    n_atoms = sum(s.n_atoms for s in structures)
    for _ in range(warmup):
        orc.predict(list(structures), compute_forces=forces, compute_nc=nc)
    runs = []
    for _ in range(max(repeats, 1)):
        t0 = time.perf_counter()
        for _ in range(steps):
            orc.predict(list(structures), compute_forces=forces, compute_nc=nc)
        runs.append((time.perf_counter() - t0) / max(steps, 1))
    dt = float(np.median(runs))
    return n_atoms / dt, threads, dt, [n_atoms / r for r in runs]


def device_ms(t):
    """Device time of one predict call without its host<->device copies:
    the library's CUDA-event phases from the end of the input copy to the
    start of the result copy."""
    return t["total"] - t["h2d"] - t["d2h"]


def spread(values):
    """Relative half-range of repeated measurements."""
    v = np.asarray(values, np.float64)
    return float((v.max() - v.min()) / (2.0 * np.median(v))) if len(v) > 1 else 0.0


class Workload:
    """One benchmark configuration: its structures, weights and CPU sample."""

    def __init__(self, name, args, wl):
        self.name = name
        self.periodic = name != "molecules"
        if name == "fcc":
            self.hname = args.hypers
            reps = args.reps
            self.structures = None  # built per world size (weak scaling)
            self.reps = reps
            self.cpu_sample = [wl.fcc_alloy(args.cpu_reps, seed=0)]
            self.cpu_desc = f"{args.cpu_reps ** 3}-atom cell of the same alloy"
            self.desc = (f"fcc alloy {reps}^3 primitive cells ({reps ** 3} atoms per GPU, triclinic, a=3.6, "
                         f"20 elements, jitter 0.08)")
        elif name == "si216":
            self.hname = "pet-mad-s"
            self.structures = [wl.si_diamond(3, seed=0)]
            self.cpu_sample = self.structures
            self.cpu_desc = "the same 216-atom cell"
            self.desc = "diamond Si 3x3x3 conventional cells (216 atoms, a=5.431, jitter 0.05)"
        elif name == "water":
            self.hname = "pet-mad-s"
            self.structures = [wl.water_box(4096, seed=0)]
            self.cpu_sample = [wl.water_box(384, seed=0)]
            self.cpu_desc = "384-atom box of the same liquid water (density, geometry, generator)"
            self.desc = ("liquid water, 4,096 atoms (1,365 H2O + 1 H), 1.0 g/cm^3, O-H 0.96, H-O-H 104.5, "
                         "2.0 A min O-O")
        elif name == "molecules":
            self.hname = "pet-mad-s"
            self.structures = wl.molecules(512, seed=0)
            self.cpu_sample = self.structures[:8]
            self.cpu_desc = (f"the first 8 molecules of the batch "
                             f"({sum(s.n_atoms for s in self.cpu_sample)} atoms)")
            n = sum(s.n_atoms for s in self.structures)
            self.desc = (f"512 non-periodic molecules of 10-60 atoms ({n} atoms), Z from H/C/N/O "
                         f"(.5/.3/.1/.1), 0.9 A min pair distance")
        elif name == "si":
            self.hname = "pet-mad-s"
            self.structures = [wl.si_diamond(32, seed=0)]
            self.cpu_sample = [wl.si_diamond(3, seed=0)]
            self.cpu_desc = "216-atom cell of the same diamond Si (3x3x3)"
            self.desc = "diamond Si 32^3 conventional cells (262,144 atoms, a=5.431, jitter 0.05)"
        else:
            raise ValueError(name)
        self.h = wl.HYPERS[self.hname]

    def metric(self, mode):
        what = {"forces": "E+F+stress" if self.periodic else "E+F", "energy": "E only (forward pass)",
                "nc": "E + non-conservative F and stress heads (forward pass)"}[mode]
        if self.name == "fcc":
            return METRIC if mode == "forces" else METRIC.replace("(E+F+stress)", f"({what})")
        label = {"si216": "216-atom Si cell", "water": "4,096-atom water box",
                 "molecules": "512-molecule batch", "si": "262k-atom Si cell, spatial domains"}[self.name]
        return f"atom-steps/s ({what}), {label}, PET, B200"

    def weights_desc(self, mode):
        h = self.h
        return (f"{self.hname}-shaped random-init weights (d={h.d_pet}, heads={h.num_heads}, "
                f"ff={h.d_feedforward}, d_head={h.d_head}, rc={h.cutoff}{', nc heads' if mode == 'nc' else ''})")


def roofline(kstats, t_dev_s, f16_mode, traffic, peaks):
    hbm, bf16, bf16_sus, src = peaks
    f16 = kstats["gemm_f16"]["launches"] > 0
    g = kstats["gemm_f16" if f16 else "gemm_tc"]
    gemm_ms = kstats["gemm_f16"]["ms"] + kstats["gemm_tc"]["ms"] + kstats["gemm_simt"]["ms"]
    achieved = g["flops"] / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else 0.0
    # achieved counts 2MNK.  3xFP16 runs three fp16 MMAs per fp32 product at
    # the bf16 rate (ceiling: measured bf16 peak / 3); 3xTF32 three tf32
    # MMAs at half that rate (ceiling / 6).
    div = (1.0 if f16_mode else 3.0) if f16 else 6.0
    att = kstats["attention"]
    return {"bound": "tensor",
            "kernel": ("k_gemm_3xf16" if f16 else "k_gemm_3xtf32") + " (tcgen05, all dense layers)",
            "achieved": achieved, "peak": bf16_sus / div, "unit": "TFLOP/s",
            "frac": achieved / (bf16_sus / div),
            "peak_source": ((f"{src} bf16 sustained (1 fp16 MMA per product)" if f16_mode else
                             f"{src} bf16 sustained / 3 (3 fp16 MMAs per product at the bf16 rate)")
                            if f16 else f"{src} bf16 sustained / 6 (3 tf32 MMAs at half bf16 rate)"),
            "tensor_pipe_frac_of_bf16": div * achieved / bf16_sus,
            # DRAM bytes per average GEMM launch: ncu dram__bytes_read.sum +
            # dram__bytes_write.sum over all GEMM launches of one step of the
            # 1,728-atom cell of this alloy (5,371 B per token for the 3xFP16
            # build), scaled by this step's tokens; null where not captured
            "traffic": traffic,
            "traffic_unit": "bytes per GEMM launch (scaled from the 1,728-atom capture)",
            "timing": "CUDA events around every launch on the library's stream, over a second pass of the "
                      "same K steps",
            "gemm_share_of_step": gemm_ms / (t_dev_s * 1e3) if t_dev_s else None,
            "attention": {"ms_per_launch": att["ms"] / att["launches"] if att["launches"] else None,
                          "achieved_gbs": (att["bytes"] / (att["ms"] / 1e3) / 1e9) if att["ms"] > 0 else None,
                          "peak_gbs": hbm, "frac": ((att["bytes"] / (att["ms"] / 1e3) / 1e9) / hbm)
                          if att["ms"] > 0 else None,
                          "bound": "hbm", "peak_source": f"{src} copy bandwidth"}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="fcc", choices=["fcc", "si216", "water", "molecules", "si"])
    ap.add_argument("--hypers", default="pet-oam-l", help="weights shape of the fcc workload")
    ap.add_argument("--reps", type=int, default=32, help="primitive fcc cells per axis and GPU")
    ap.add_argument("--cpu-reps", type=int, default=6, help="fcc CPU-baseline sample cells per axis")
    ap.add_argument("--cpu-steps", type=int, default=10, help="timed CPU-baseline steps per repeat")
    ap.add_argument("--cpu-repeats", type=int, default=3, help="CPU-baseline repeats (median reported)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parallel", default="domains", choices=["domains", "replicas"],
                    help="fcc on N > 1 GPUs: one cell split into spatial domains, or a replica per rank")
    ap.add_argument("--precision", default="f32", choices=["f32", "f16"],
                    help="f16: MLIPCPP_PRECISION_F16, dense layers with one fp16 product (looser tolerances)")
    ap.add_argument("--mode", default="forces", choices=["forces", "energy", "nc"],
                    help="forces: E + gradient forces (+ stress when periodic; headline); energy: the forward "
                         "pass only; nc: forces and stress from non-conservative heads, forward only")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    mb = _package()
    from mlipcpp_b200 import workloads as wl
    W = Workload(args.workload, args, wl)
    grad, nc = args.mode == "forces", args.mode == "nc"
    tmpdir = tempfile.mkdtemp(prefix="petbench")
    gguf = os.path.join(tmpdir, "w.gguf")
    wl.write_pet_gguf(gguf, W.h, seed=0, nc_heads=nc)
    metric = W.metric(args.mode)

    if args.impl == "reference":
        if rank != 0:
            return
        v, threads, dt, runs = cpu_reference(W.cpu_sample, gguf, 1, args.warmup, repeats=args.steps,
                                             forces=grad, nc=nc)
        n_s = sum(s.n_atoms for s in W.cpu_sample)
        line = {"metric": metric, "value": v, "unit": "atom-steps/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "impl": "reference",
                "config": {"workload": W.desc + ", " + W.weights_desc(args.mode),
                           "sample": W.cpu_desc},
                "cpu_baseline": {"value": v, "unit": "atom-steps/s", "cores": threads, "kind": "port",
                                 "sample": f"{W.cpu_desc}, {n_s} atoms per step, median of {args.steps} "
                                           "timed steps (PyTorch-CPU restatement of the reference, float32; "
                                           "ggml absent)",
                                 "spread": spread(runs)},
                "e2e": {"value": v, "unit": "atom-steps/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    torch.cuda.set_device(local)
    mb.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if dist:
            t = torch.tensor([float(x)], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            x = float(t.item())
        return x

    f16_mode = args.precision == "f16"
    pred = mb.Predictor(gguf, mb.ModelOptions(precision=1 if f16_mode else 0))
    pred.set_timing(True)
    peaks = _peaks()
    flush_buf = None

    # ---- choose the step functions ----------------------------------------
    from mlipcpp_b200 import domain as dd
    from mlipcpp_b200 import sharding as sh
    domains = world > 1 and ((W.name == "fcc" and args.parallel == "domains" and grad) or W.name == "si")
    par = f"replicas x{world}"
    scaling = "weak"
    if W.name == "si" and world < 2:
        if rank == 0:
            print(json.dumps({"metric": metric, "workload": W.desc,
                              "unavailable": "262,144 atoms need at least 2 GPUs (about 280 GB of "
                                             "activations on one)"}), flush=True)
        return
    if W.name == "si" and not grad:
        raise SystemExit("the si workload runs E+F+stress only")
    if W.name == "fcc":
        reps = (W.reps,) * 3
        if domains:
            # N x 32k atoms: double the cell along z, then y, then x
            r = list(reps)
            k, w = 2, world
            while w > 1:
                r[k] *= 2
                w //= 2
                k = (k - 1) % 3
            reps = tuple(r)
        s = wl.fcc_alloy(reps, seed=0)
        structs = [s]
    else:
        structs = W.structures
        s = structs[0]
    n_atoms_job = sum(x.n_atoms for x in structs) * (1 if domains else world)
    if W.name == "molecules" and world > 1:
        n_atoms_job = sum(x.n_atoms for x in structs)
    if W.name == "si":
        scaling = "strong"
    if W.name == "molecules":
        scaling = "strong" if world > 1 else "weak"

    dom = None
    if domains:
        grid = dd.grid_for(world)
        mine = np.nonzero(dd.owners(s.positions, s.cell, grid) == rank)[0]
        comm = dd.NcclComm()
        dom = dd.Domain(pred, s.cell, grid, rank, comm.c)
        dom.set_atoms(s.numbers[mine])
        own_pos = np.ascontiguousarray(s.positions[mine], np.float32)
        d_pos = torch.from_numpy(own_pos).cuda()
        d_F = torch.zeros_like(d_pos)
        pos_host = torch.from_numpy(own_pos).pin_memory()
        par = (f"spatial domains {'x'.join(map(str, grid))}: layer 0 and 1 on owned atoms, NCCL alltoallv of "
               "halo positions, reverse-edge layer-0 tokens and their gradients, ghost forces; all-reduce of "
               "(E, virial)")

        def step():
            t0 = time.perf_counter()
            dom.step(pos_host.to("cuda", non_blocking=True), d_F)
            d_F.cpu()
            return (time.perf_counter() - t0) * 1e3, dom.stats()["step_ms"]
        h2d_bytes = int(own_pos.nbytes)
        d2h_bytes = int(own_pos.nbytes + 8 * 7)
    elif W.name == "molecules":
        mine = sh.shard([sh.structure_cost(x.n_atoms) for x in structs], world)[rank]
        my_structs = [structs[i] for i in mine]
        # the batch as a data loader holds it: one packed block of host arrays
        batch = sh.PackedBatch.pack(structs)
        runner = sh.PackedBatchRunner(sh.predictor_packed_eval(pred, compute_forces=grad or nc), world=world,
                                      rank=rank)
        if world > 1:
            par = f"batch shards x{world} (LPT on n^3), final all-gather"

        def step():
            t0 = time.perf_counter()
            runner.run(batch)
            return (time.perf_counter() - t0) * 1e3, device_ms(pred.last_timings())
        h2d_bytes = int(sum(x.positions.nbytes + x.numbers.nbytes for x in my_structs))
        d2h_bytes = int(sum(x.positions.nbytes + 8 for x in my_structs))
    else:
        opts = mb.PredictOptions(grad or nc, grad or nc, nc)

        def step():
            t0 = time.perf_counter()
            pred.predict_with_options(s.positions, s.numbers, s.cell, s.pbc, opts)
            return (time.perf_counter() - t0) * 1e3, device_ms(pred.last_timings())
        h2d_bytes = int(s.positions.nbytes + s.numbers.nbytes)
        d2h_bytes = int(s.positions.nbytes + 6 * 4 + 8 * 7) if (grad or nc) else 8 * 7

    # small working sets: flush L2 between steps (outside the timed calls)
    small = W.name == "si216"
    if small:
        flush_buf = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")

    def flush():
        if flush_buf is not None:
            flush_buf.zero_()
            torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        step()
    # ---- timed region: K steps, each one public predict call from host
    # arrays.  e2e: the host clock around the call (host->device copy of the
    # inputs, the step, device->host copy of the results).  value: the same
    # call's device time with its inputs already in HBM, i.e. the library's
    # CUDA events from the end of its host->device copy to the start of its
    # device->host copy (on the spatial-domain path: the engine's events
    # around its step) ------------------------------------------------------
    launches = 0
    dev_ms, wall_ms = [], []
    with ClockSampler(local) as clk:
        barrier()
        for _ in range(args.steps):
            flush()
            l0 = mb.kernel_launches()
            w_ms, d_ms = step()
            launches += mb.kernel_launches() - l0
            wall_ms.append(w_ms)
            dev_ms.append(d_ms)
        barrier()
    phase = pred.last_timings()
    t_dev = max_over_ranks(float(np.sum(dev_ms)) / 1e3)
    value = n_atoms_job * args.steps / t_dev
    t_e2e = max_over_ranks(float(np.sum(wall_ms)) / 1e3)
    e2e = n_atoms_job * args.steps / t_e2e

    # ---- per-launch kernel times for the roofline: the same K steps again,
    # with CUDA events around every GEMM and attention launch on the
    # library's stream (a separate pass, so they do not perturb `value`)
    pred.set_kernel_profiling(True)
    barrier()
    for _ in range(args.steps):
        flush()
        step()
    barrier()
    kstats = pred.kernel_stats()
    pred.set_kernel_profiling(False)

    domain_stats = None
    if dom is not None:
        # per-phase device times of the last step: the max over ranks, with
        # rank 0's counts
        st = dom.stats()
        domain_stats = {k: (max_over_ranks(v) if k.endswith("_ms") else v) for k, v in st.items()}
    if rank == 0:
        shape = pred.last_shape()
        fcc_traffic = (W.name == "fcc" and not domains and not f16_mode and grad)
        line = {
            "metric": metric, "value": value, "unit": "atom-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": t_dev / args.steps * 1e3,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "f16" if f16_mode else "f32", "data": "synthetic",
            "config": {"workload": W.desc + ", " + W.weights_desc(args.mode),
                       "atoms_per_gpu": n_atoms_job // world, "atoms_total": n_atoms_job,
                       "edges_rank0": shape["edges"], "max_neighbors": shape["max_neighbors"],
                       "parallelism": par,
                       "l2": ("L2 flushed between steps (a 252 MB write outside the timed calls)" if small
                              else "inputs larger than L2 (hundreds of MB to GB working set per step)")},
            "e2e": {"value": e2e, "unit": "atom-steps/s", "h2d_bytes_per_step": h2d_bytes,
                    "d2h_bytes_per_step": d2h_bytes,
                    "timing": "host clock around each public predict call (host arrays in, numpy out)"},
            "gpu_launches": int(launches),
            "roofline": roofline(kstats, t_dev, f16_mode,
                                 5371.0 * (shape["atoms"] + shape["edges"]) if fcc_traffic else None, peaks),
            "kernel_stats": kstats,
            "phase_ms": phase,
            "domain": domain_stats,
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline and world == 1:
            v, threads, dt, runs = cpu_reference(W.cpu_sample, gguf, args.cpu_steps, 2,
                                                 repeats=args.cpu_repeats, forces=grad, nc=nc)
            n_s = sum(x.n_atoms for x in W.cpu_sample)
            line["cpu_baseline"] = {
                "value": v, "unit": "atom-steps/s", "cores": threads, "kind": "port",
                "sample": (f"{W.cpu_desc}, {n_s} atoms per step; 2 warm-up steps, then the median of "
                           f"{args.cpu_repeats} runs of {args.cpu_steps} steps (PyTorch-CPU restatement, float32)"),
                "spread": spread(runs), "runs": runs}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
