"""Throughput benchmark: atom-steps/s for PET energy + forces + stress.

Workload (the configuration the headline metric is quoted on): the periodic
random fcc alloy of 32^3 primitive cells (32,768 atoms, triclinic cell,
a = 3.6 A, 20 random elements among Z = 1..89, jitter N(0, 0.08 A)) with
random-init pet-oam-l-shaped weights (d_pet 512, 16 heads, d_ff 1024,
d_head 256, cutoff 4.5 A); seeded synthetic data.  One step = one
prediction of energy, forces and stress: neighbour list, featuriser, both
GNN layers, readout and the full backward pass.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (launched with torch.distributed.run), weak scaling at 32,768 atoms
per GPU: N ranks evaluate one cell of N x 32,768 atoms (32x32x64 primitive
cells for 2 GPUs, 32x64x64 for 4, 64^3 = 262,144 for 8) split into N spatial
domains (owned atoms plus two ghost shells of one cutoff each); the only
exchange is an NCCL all-reduce of the forces and of (energy, virial) per
step.  `--parallel replicas` instead runs an independent copy of the 32k cell
per rank.  The timed region is bracketed by barriers and the reported time is
the max over ranks.

`--impl reference` times the CPU implementation of the path on the host
cores: the reference's model cannot be built here (its ggml dependency is
absent), so this is the PyTorch restatement in oracle/ at float32.
"""
import argparse
import importlib.util
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "atom-steps/s (E+F+stress), 32k-atom PET cell, 1/2/4/8 B200; % of roofline"


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
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in self.rows if len(r) > 8
                          for k in range(4) if r[5 + k].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(self.rows)}


def cpu_reference(structure, gguf_path, steps, warmup):
    """Time the CPU implementation of the path (float32, all host threads)
    on `structure`; returns (atom-steps/s, threads, per-step seconds)."""
    import torch
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import pet_oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    orc = pet_oracle.load_oracle(gguf_path, torch.float32)
    for _ in range(warmup):
        orc.predict([structure])
    t0 = time.perf_counter()
    for _ in range(steps):
        orc.predict([structure])
    dt = (time.perf_counter() - t0) / max(steps, 1)
    return structure.n_atoms / dt, threads, dt


def run_other_workload(args, world, rank, local, mb, wl, torch, dist):
    """The 262,144-atom Si cell over N GPUs (domain decomposition, strong
    scaling) or a batch of 512 molecules sharded over N GPUs; pet-mad-s-shaped
    weights; one JSON line from rank 0."""
    from mlipcpp_b200 import domain as dd
    from mlipcpp_b200 import sharding as sh
    h = wl.PET_MAD_S
    gguf = os.path.join(tempfile.mkdtemp(prefix="petbench"), "w.gguf")
    wl.write_pet_gguf(gguf, h, seed=0)
    pred = mb.Predictor(gguf)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def max_over_ranks(x):
        if dist:
            t = torch.tensor([x], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            x = float(t.item())
        return x

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    if args.workload == "si":
        s = wl.si_diamond(32, seed=0)
        desc = (f"diamond Si 32^3 conventional cells ({s.n_atoms} atoms, a=5.431, jitter 0.05), "
                f"pet-mad-s-shaped random-init weights, E+F+stress")
        if world < 2:
            if rank == 0:
                print(json.dumps({"workload": desc, "unavailable": "262,144 atoms need at least 2 GPUs (about "
                                                                   "280 GB of activations on one)"}), flush=True)
            return
        runner = dd.DomainRunner(dd.predictor_eval(pred), s.numbers, s.cell, h.cutoff, world=world, rank=rank)
        d_pos = torch.from_numpy(s.positions).cuda()
        step = lambda: runner.step(d_pos)  # noqa: E731
        n_atoms, metric = s.n_atoms, "atom-steps/s (E+F+stress), 262k-atom Si cell, domain decomposition"
        par = f"spatial domains {'x'.join(map(str, dd.grid_for(world)))}"
    else:
        mols = wl.molecules(512, seed=0)
        runner = sh.BatchRunner(sh.predictor_batch_eval(pred), world=world, rank=rank)
        step = lambda: runner.run(mols)  # noqa: E731
        n_atoms = sum(m.n_atoms for m in mols)
        desc = f"512 molecules of 10-60 atoms ({n_atoms} atoms), pet-mad-s-shaped random-init weights, E+F"
        metric = "atom-steps/s (E+F), 512-molecule batch, structures sharded over GPUs"
        par = f"batch shards x{world} (LPT on n^3), final all-gather"
    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    ev0.record()
    for _ in range(args.steps):
        step()
    ev1.record()
    barrier()
    t = max_over_ranks(ev0.elapsed_time(ev1) / 1e3)
    if rank == 0:
        v = n_atoms * args.steps / t
        print(json.dumps({"metric": metric, "value": v, "unit": "atom-steps/s", "n_gpus": world,
                          "steps": args.steps, "warmup": max(args.warmup, 3),
                          "ms_per_step": t / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                          "config": {"workload": desc, "atoms_total": n_atoms, "parallelism": par},
                          "e2e": {"value": v, "unit": "atom-steps/s",
                                  "note": "positions enter from the device (si) or the host (molecules)"}}),
              flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--hypers", default="pet-oam-l")
    ap.add_argument("--reps", type=int, default=32, help="primitive fcc cells per axis")
    ap.add_argument("--cpu-reps", type=int, default=6, help="CPU-baseline sample cells per axis")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parallel", default="domains", choices=["domains", "replicas"],
                    help="multi-GPU mode: one cell split into spatial domains, or a replica per rank")
    ap.add_argument("--precision", default="f32", choices=["f32", "f16"],
                    help="f16: MLIPCPP_PRECISION_F16, dense layers with one fp16 product (looser tolerances)")
    ap.add_argument("--mode", default="forces", choices=["forces", "energy", "nc"],
                    help="forces: E + gradient forces + stress (headline); energy: the forward pass only; "
                         "nc: forces and stress from non-conservative heads (use_nc_forces), forward only; "
                         "energy and nc run one replica per GPU")
    ap.add_argument("--workload", default="fcc", choices=["fcc", "si", "molecules"],
                    help="fcc: the 32k-atom alloy per GPU (headline); si: one 262,144-atom diamond-Si "
                         "cell over N >= 2 GPUs (strong scaling); molecules: 512 molecules sharded")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    mb = _package()
    from mlipcpp_b200 import workloads as wl
    h = wl.HYPERS[args.hypers]
    what = {"forces": "E+F+stress", "energy": "E only (forward pass)",
            "nc": "E + non-conservative F and stress heads (forward pass)"}[args.mode]
    metric = METRIC if args.mode == "forces" else METRIC.replace("(E+F+stress)", f"({what})")
    workload = (f"fcc alloy {args.reps}^3 primitive cells ({args.reps ** 3} atoms per GPU, triclinic, a=3.6, "
                f"20 elements, jitter 0.08), {args.hypers}-shaped random-init weights "
                f"(d={h.d_pet}, heads={h.num_heads}, ff={h.d_feedforward}, d_head={h.d_head}, "
                f"rc={h.cutoff}{', nc heads' if args.mode == 'nc' else ''}), {what}")

    tmpdir = tempfile.mkdtemp(prefix="petbench")
    gguf = os.path.join(tmpdir, "w.gguf")
    wl.write_pet_gguf(gguf, h, seed=0, nc_heads=args.mode == "nc")

    if args.impl == "reference":
        if rank != 0:
            return
        sample = wl.fcc_alloy(args.cpu_reps, seed=0)
        v, threads, dt = cpu_reference(sample, gguf, args.steps, args.warmup)
        line = {"metric": METRIC, "value": v, "unit": "atom-steps/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "impl": "reference",
                "config": {"workload": workload, "sample": f"{sample.n_atoms}-atom cell of the same alloy"},
                "cpu_baseline": {"value": v, "unit": "atom-steps/s", "cores": threads, "kind": "port",
                                 "sample": f"{sample.n_atoms}-atom fcc alloy cell, {args.steps} steps "
                                           "(PyTorch-CPU restatement of the reference; ggml absent)"},
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

    if args.workload != "fcc":
        run_other_workload(args, world, rank, local, mb, wl, torch, dist)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return

    domains = world > 1 and args.parallel == "domains" and args.mode == "forces"
    grad, nc = args.mode == "forces", args.mode == "nc"
    reps = (args.reps,) * 3
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
    f16_mode = args.precision == "f16"
    pred = mb.Predictor(gguf, mb.ModelOptions(precision=1 if f16_mode else 0))
    pred.set_timing(True)
    d_pos = torch.from_numpy(s.positions).cuda()
    torch.cuda.synchronize()

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if dist:
            t = torch.tensor([x], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            x = float(t.item())
        return x

    from mlipcpp_b200 import domain as dd
    if domains:
        runner = dd.DomainRunner(dd.predictor_eval(pred), s.numbers, s.cell, h.cutoff, world=world, rank=rank)

        def step_device():
            return runner.step(d_pos)
    else:
        def step_device():
            return pred.predict_device(d_pos.data_ptr(), s.n_atoms, s.numbers, s.cell, s.pbc,
                                       compute_forces=grad or nc, compute_stress=grad or nc, copy_forces=False,
                                       use_nc_forces=nc)

    for _ in range(max(args.warmup, 3)):
        step_device()
    # ---- device-resident timed region (value) -----------------------------
    pred.set_kernel_profiling(True)
    launches0 = mb.kernel_launches()
    barrier()
    with ClockSampler(local) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dev_ms = []
        ev0.record()
        for _ in range(args.steps):
            step_device()
            if not domains:
                dev_ms.append(pred.last_timings()["total"])
        ev1.record()
        barrier()
    launches = mb.kernel_launches() - launches0
    kstats = pred.kernel_stats()
    pred.set_kernel_profiling(False)
    # single cell: the library's own events on its stream; domains: torch
    # events around whole steps (the library synchronises its stream before
    # returning, so they span its work, the partition and the all-reduces)
    t_dev = float(np.sum(dev_ms)) / 1e3 if not domains else ev0.elapsed_time(ev1) / 1e3
    t_dev = max_over_ranks(t_dev)
    n_job = s.n_atoms if domains else world * s.n_atoms
    value = n_job * args.steps / t_dev

    # ---- end-to-end through the public API with host buffers --------------
    pos_host = torch.from_numpy(s.positions).pin_memory()
    barrier()
    if domains:
        ev0.record()
        for _ in range(args.steps):
            e, F, vir = runner.step(pos_host.to("cuda", non_blocking=True))
            F_host = F.cpu()
        ev1.record()
        barrier()
        t_e2e = ev0.elapsed_time(ev1) / 1e3
        d2h = int(F_host.numel() * 4 + 8 * 7)
    else:
        e2e_ms = []
        opts = mb.PredictOptions(grad or nc, grad or nc, nc)
        for _ in range(args.steps):
            r = pred.predict_with_options(pos_host.numpy(), s.numbers, s.cell, s.pbc, opts)
            e2e_ms.append(pred.last_timings()["total"])
        barrier()
        t_e2e = float(np.sum(e2e_ms)) / 1e3
        d2h = int(r.forces.nbytes + r.stress.nbytes + 4)
    t_e2e = max_over_ranks(t_e2e)
    e2e = n_job * args.steps / t_e2e

    if rank == 0:
        hbm, bf16, bf16_sus, src = _peaks()
        f16 = kstats["gemm_f16"]["launches"] > 0
        g = kstats["gemm_f16" if f16 else "gemm_tc"]
        gemm_ms = kstats["gemm_f16"]["ms"] + kstats["gemm_tc"]["ms"] + kstats["gemm_simt"]["ms"]
        achieved = g["flops"] / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else 0.0
        # achieved counts 2MNK.  3xFP16 runs three fp16 MMAs per fp32 product at
        # the bf16 rate (ceiling: measured bf16 peak / 3); 3xTF32 three tf32
        # MMAs at half that rate (ceiling / 6).
        div = (1.0 if f16_mode else 3.0) if f16 else 6.0
        shape = pred.last_shape()
        line = {
            "metric": metric, "value": value, "unit": "atom-steps/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": t_dev / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16" if f16_mode else "f32",
            "data": "synthetic",
            "config": {"workload": workload, "atoms_per_gpu": n_job // world, "atoms_total": n_job,
                       "edges_rank0": shape["edges"], "max_neighbors": shape["max_neighbors"],
                       "parallelism": (f"spatial domains {'x'.join(map(str, dd.grid_for(world)))} "
                                       "(owned + 2 ghost shells), NCCL all-reduce of F and (E, virial)"
                                       if domains else f"replicas x{world}"),
                       "l2": "inputs larger than L2 (multi-GB working set per step)"},
            "e2e": {"value": e2e, "unit": "atom-steps/s",
                    "h2d_bytes_per_step": int(s.positions.nbytes + (0 if domains else s.numbers.nbytes)),
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor",
                         "kernel": ("k_gemm_3xf16 (+ k_split_a where an input is fp32)" if f16 else "k_gemm_3xtf32")
                                   + " (tcgen05, all dense layers)",
                         "achieved": achieved, "peak": bf16_sus / div, "unit": "TFLOP/s",
                         "frac": achieved / (bf16_sus / div),
                         "peak_source": ((f"{src} bf16 sustained (1 fp16 MMA per product)" if f16_mode else
                                          f"{src} bf16 sustained / 3 (3 fp16 MMAs per product at the bf16 rate)")
                                         if f16 else f"{src} bf16 sustained / 6 (3 tf32 MMAs at half bf16 rate)"),
                         "tensor_pipe_frac_of_bf16": div * achieved / bf16_sus,
                         # DRAM bytes per average GEMM launch: ncu dram__bytes_read.sum +
                         # dram__bytes_write.sum over all 55 GEMM launches of one step of the
                         # 1,728-atom cell of this alloy (350 MB/launch at 65,202 tokens,
                         # 5,371 B per token for the 3xFP16 build), scaled by this step's tokens
                         "traffic": (5371.0 * (shape["atoms"] + shape["edges"])
                                     if not domains and f16 and grad else None),
                         "traffic_unit": "bytes per GEMM launch (scaled from the 1,728-atom capture)",
                         "gemm_share_of_step": gemm_ms / (t_dev * 1e3) if t_dev else None},
            "kernel_stats": kstats,
            "phase_ms": pred.last_timings(),
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline and world == 1 and grad:
            sample = wl.fcc_alloy(args.cpu_reps, seed=0)
            v, threads, dt = cpu_reference(sample, gguf, 2, 1)
            line["cpu_baseline"] = {"value": v, "unit": "atom-steps/s", "cores": threads, "kind": "port",
                                    "sample": f"{sample.n_atoms}-atom cell of the same alloy, 2 steps "
                                              "(PyTorch-CPU restatement, float32)"}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
