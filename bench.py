"""Benchmark: atom-steps/s of pure-cartesian-ictd energy + forces on B200.

Workload ("si1m"): pure-cartesian-ictd, 3 interaction layers, 64 channels,
lmax 2, fp32, cutoff 5.0 A, 8 gaussian radial functions (the CLI default basis); a periodic
diamond-lattice Si crystal of 1,000,000 atoms (50^3 conventional cells x 8 atoms, a = 5.43 A,
Gaussian displacements sigma = 0.08 A), seeded synthetic positions and seeded random weights.
One step = one MD-style evaluation: GPU neighbour list (cell list, bit-exact with the
reference semantics) + forward + hand-written backward (energy, forces).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

``--impl reference`` times the reference's own CPU path (its PyTorch modules, installed unmodified
under baseline/_ref, fp32, all host threads) on a bounded replica of the same workload.  Under
torchrun (N > 1) the crystal grows with N (weak scaling, 1,000,000 owned atoms per GPU; or
``--scaling strong``: one fixed crystal) and is cut into a (2, 1, 1) / (2, 2, 1) / (2, 2, 2) grid
of blocks, one per rank: each step exchanges a one-cutoff (5 A) halo of ghost positions,
overwrites the ghost feature rows after every interaction layer that a later layer reads (and
returns their gradients in the reverse pass), returns the ghost forces to their owners and sums
the energy (fsctep_b200.domain; ``--halo recompute``: a 15 A halo of recomputed ghosts and no
per-layer exchange); the reported value is all owned atoms / the slowest rank's time, and the
clock record covers every GPU of the job.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

WORKLOADS = {
    "si1m": dict(model="ictd", cells=(50, 50, 50), channels=64, num_interaction=3, Z=14, max_atomvalue=16),
    "si64k": dict(model="ictd", cells=(20, 20, 20), channels=64, num_interaction=3, Z=14, max_atomvalue=16),
    # pure-cartesian-sparse (one GPU): config 2 in full, and config 5's model on FCC crystals
    "water3k": dict(model="sparse", system="water", n_side=10, box=31.0, channels=64, lmax=2, num_interaction=3,
                    max_atomvalue=10, cpu_n_side=4),
    "fcc32k": dict(model="sparse", system="fcc", cells=(20, 20, 20), channels=128, lmax=3, num_interaction=3,
                   max_atomvalue=30, cpu_cells=(2, 2, 2)),
    "fcc250k": dict(model="sparse", system="fcc", cells=(50, 50, 25), channels=128, lmax=3, num_interaction=3,
                    max_atomvalue=30, cpu_cells=(2, 2, 2)),
    # batched small systems (one GPU): config 1 (E + F + stress) and config 3 (o3, field, heads)
    "frames8": dict(model="ictd", system="frames", n_frames=8, n_atoms=96, box=10.0, channels=32, num_interaction=2,
                    basis="bessel", max_atomvalue=10),
    "mol256": dict(model="o3", system="molecules", n_mol=256, channels=64, num_interaction=3, basis="gaussian",
                   max_atomvalue=10),
}
BATCHED = ("frames", "molecules")
O3_HEADS = {"dipole": {"irreps": ["1o"], "reduce": "sum"}, "polarizability": {"ls": [0, 2], "reduce": "sum"}}
CPU_KEYS = ("value", "unit", "cores", "kind", "sample", "steps", "warmup", "statistic", "cpu_model")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def model_cfg(w):
    from fsctep_b200.ictd import ICTDConfig

    return ICTDConfig(channels=w["channels"], num_interaction=w["num_interaction"], number_of_basis=8,
                      max_radius=5.0, function_type=w.get("basis", "gaussian"), max_atomvalue=w["max_atomvalue"],
                      o3=w["model"] == "o3")


def seeded_weights(cfg, seed=2024):
    from fsctep_b200.models import PureCartesianICTDO3TransformerLayer, reference_state_dict_shapes
    from fsctep_b200.weights import seeded_state_dict

    if not cfg.o3:
        return seeded_state_dict(reference_state_dict_shapes(cfg), seed)
    with torch.device("meta"):
        m = PureCartesianICTDO3TransformerLayer(
            max_embed_radius=cfg.max_radius, main_max_radius=cfg.max_radius, main_number_of_basis=cfg.number_of_basis,
            hidden_dim_conv=cfg.channels, num_interaction=cfg.num_interaction, function_type_main=cfg.function_type,
            max_atomvalue=cfg.max_atomvalue, external_tensor_rank=1, external_tensor_irrep="1o",
            physical_tensor_outputs=O3_HEADS, o3_active_irreps=list(cfg.o3_irreps))
    return seeded_state_dict({k: tuple(v.shape) for k, v in m.state_dict().items()}, seed)


def batched_system(w, seed=1000):
    """Config 1's periodic frames or config 3's molecules (with one field vector per molecule)."""
    from fsctep_b200 import systems

    if w["system"] == "frames":
        s = systems.random_frames(n_frames=w["n_frames"], n_atoms=w["n_atoms"], box=w["box"], seed=seed)
    else:
        s = systems.organic_molecules(n_mol=w["n_mol"], seed=seed)
        s["field"] = np.random.default_rng(seed + 1).normal(scale=0.05, size=(w["n_mol"], 3))
    s["frame_ptr"] = np.concatenate([[0], np.cumsum(np.bincount(s["batch"], minlength=s["cell"].shape[0]))])
    return s


class ClockSampler:
    """nvidia-smi clocks during the timed region (one GPU)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index, path=None):
        self.index = index
        self.proc = None
        self.path = path or os.path.join(tempfile.mkdtemp(prefix="fsctep_clocks_"), f"clocks_rank{index}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(smax)), "reasons": sorted(reasons),
                "samples": len(sm)}


def combine_clocks(summaries):
    """One clocks record for a job of several GPUs from every rank's ClockSampler.summary():
    the slowest GPU's median SM clock, the highest max clock, the union of the throttle reasons
    seen on any GPU, and each rank's median and reasons."""
    if len(summaries) == 1:
        return summaries[0]
    meds = [c.get("sm_mhz") for c in summaries]
    known = [m for m in meds if m is not None]
    maxes = [c.get("sm_max_mhz") for c in summaries if c.get("sm_max_mhz") is not None]
    reasons = sorted({r for c in summaries for r in c.get("reasons", [])})
    return {"sm_mhz": min(known) if known else None, "sm_max_mhz": max(maxes) if maxes else None,
            "reasons": reasons, "samples": sum(c.get("samples", 0) for c in summaries),
            "per_rank": [{"sm_mhz": c.get("sm_mhz"), "reasons": c.get("reasons", [])} for c in summaries],
            "statistic": "sm_mhz: lowest per-GPU median over the ranks"}


def rank_path(path, rank, world):
    """A clock CSV path of its own for every rank of a multi-GPU run."""
    if path is None or world <= 1:
        return path
    root, ext = os.path.splitext(path)
    return f"{root}_rank{rank}{ext or '.csv'}"


def sparse_cfg(w):
    from fsctep_b200.sparse import SparseConfig

    return SparseConfig(channels=w["channels"], lmax=w["lmax"], num_interaction=w["num_interaction"],
                        number_of_basis=8, max_radius=5.0, function_type="gaussian", max_atomvalue=w["max_atomvalue"])


def sparse_weights(cfg, seed=2024):
    """Seeded weights in the reference state_dict layout of PureCartesianSparseTransformerLayer."""
    from fsctep_b200.models import PureCartesianSparseTransformerLayer
    from fsctep_b200.weights import seeded_state_dict

    with torch.device("meta"):
        m = PureCartesianSparseTransformerLayer(
            max_embed_radius=cfg.max_radius, main_max_radius=cfg.max_radius, main_number_of_basis=cfg.number_of_basis,
            hidden_dim_conv=cfg.channels, lmax=cfg.lmax, num_interaction=cfg.num_interaction,
            function_type_main=cfg.function_type, max_atomvalue=cfg.max_atomvalue)
    return seeded_state_dict({k: tuple(v.shape) for k, v in m.state_dict().items()}, seed)


def sparse_system(w, seed=1000, cpu=False):
    from fsctep_b200 import systems

    if w["system"] == "water":
        n_side = w["cpu_n_side"] if cpu else w["n_side"]
        return systems.water_box(n_side=n_side, box=w["box"] * n_side / w["n_side"], seed=seed)
    return systems.fcc_crystal(n_cells=w["cpu_cells"] if cpu else w["cells"], seed=seed)


def sparse_comps(lmax):
    from fsctep_b200.sparse import sparse_paths

    return sum(3 ** Lo for (_, _, Lo) in sparse_paths(lmax))


def algorithmic_work(stage, N, E, cfg):
    """(flops, bytes) per launch of a stage, from the per-unit figures of the hot path."""
    if stage.startswith("sparse_"):
        return sparse_work(stage, N, E, cfg)
    C, nint = cfg.channels, cfg.num_interaction
    nC = C * nint
    S = (nint - 1) * cfg.invariant_channels
    npairs = nC * (nC + 1) // 2
    table = {
        # packed Gram contraction: 2*S per pair per node, 3 l blocks (+ Gram build)
        "readout_gram_forward": (N * 3 * (2.0 * S * npairs) + N * 2.0 * npairs * 9, N * 9 * nC * 4.0),
        "readout_gram_backward": (N * 3 * (2.0 * S * nC * nC) + N * 2.0 * nC * nC * 9, N * 9 * nC * 8.0),
        # TP contraction: 115 MACs per channel per edge
        "conv2_edge_forward": (2.0 * E * C * 115, N * 9 * C * 4.0 + N * 35 * C * 4.0 + E * 100.0),
        "conv2_edge_backward_gates": (2.0 * E * C * 115, N * 9 * C * 4.0 + N * 35 * C * 4.0 + E * 100.0),
        "conv2_edge_backward_x": (2.0 * E * C * 115, N * 9 * C * 4.0 + N * 35 * C * 4.0 + E * 100.0),
        "edge_forward": (E * nint * 2.0 * (8 * 64 + 64 * 64 + 64 * 11), E * (12 + 48 + nint * 48.0)),
        "edge_backward": (E * nint * 4.0 * (8 * 64 + 64 * 64 + 64 * 11), E * (48 + 48 + nint * 48.0 + 12)),
    }
    return table.get(stage)


def sparse_work(stage, N, E, cfg):
    """(flops, bytes) per layer of a pure-cartesian-sparse stage.  Per edge and output component
    the aggregation costs 65 x C multiply-adds (radial hidden row + bias times the sender channels);
    fc.4 is one GEMM per node after the aggregation (65 x C x C per output component)."""
    C, J, K3 = cfg.channels, 65, sparse_comps(cfg.lmax)
    R = sum(3 ** L for L in range(cfg.lmax + 1))
    feat = N * R * C * 4.0
    table = {
        "sparse_conv2_forward": (2.0 * E * J * C * K3 + 2.0 * N * K3 * J * C * C, 2 * feat + E * (64 * 4.0 + 16)),
        "sparse_conv2_backward": (4.0 * E * J * C * K3 + 2.0 * N * K3 * J * C * C, 3 * feat + E * (2 * 64 * 4.0 + 16)),
    }
    return table.get(stage)


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per node of one launch of the
# stage's kernel, from the ncu captures of the si64k workload (64,000 nodes, 1,792,016 edges)
# kept as text summaries under profiles/; every term grows with the node (and edge) count, so a
# launch on another workload is scaled by its nodes.
TRAFFIC_PER_NODE = {
    "readout_gram_forward": (0.528e9 + 0.051e9) / 64000,
    "readout_gram_backward": (1.697e9 + 0.466e9) / 64000,
    "conv2_edge_forward": (0.339e9 + 0.528e9) / 64000,
    "conv2_edge_backward_gates": (1.011e9 + 0.164e9) / 64000,
    "conv2_edge_backward_x": (0.357e9 + 0.531e9) / 64000,
    "edge_forward": (0.255e9 + 0.210e9) / 64000,
    "edge_backward": (0.662e9 + 0.062e9) / 64000,
}


def fp32_context(roofline, clocks, sms=148, measured=None):
    """The dominant kernel's FP32 rate against the CUDA-core FP32 peak: ``measured`` (the FMA probe
    of this run, :func:`measure_fp32_peak`) when given, else the nominal sms x 128 lanes x 2 FLOP x
    the median SM clock sampled during the timed region.  Only for the CUDA-core kernels, which the
    HBM roofline undersells."""
    if not roofline or roofline.get("bound") != "hbm" or roofline.get("algorithmic_tflops") is None:
        return None
    mhz = (clocks or {}).get("sm_mhz") or (clocks or {}).get("sm_max_mhz") or 1965.0
    ach = float(roofline["algorithmic_tflops"])
    nominal = sms * 128 * 2 * float(mhz) * 1e6 / 1e12
    if measured:
        return {"achieved_tflops": ach, "peak_tflops": measured["tflops"], "frac": ach / measured["tflops"],
                "sm_mhz": float(mhz), "nominal_tflops": nominal,
                "peak_source": "measured: " + measured["how"]}
    return {"achieved_tflops": ach, "peak_tflops": nominal, "frac": ach / nominal, "sm_mhz": float(mhz),
            "peak_source": f"nominal: {sms} SMs x 128 FP32 lanes x 2 FLOP x SM clock"}


def measure_fp32_peak(device, reps=5):
    """FP32 CUDA-core throughput of this GPU: the library's FMA probe (8 independent chains per
    thread, 8 blocks of 256 threads per SM), scalar and packed two-lane FMAs, best of ``reps``
    CUDA-event-timed launches after a warm-up; the faster form is the peak."""
    from fsctep_b200 import _native as NAT

    sms = torch.cuda.get_device_properties(device).multi_processor_count
    blocks = 8 * sms
    out = torch.empty(blocks * 256, dtype=torch.float32, device=device)
    flops = NAT.C.c_double(0.0)
    best = {}
    for packed in (0, 1):
        times = []
        for r in range(reps + 1):
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            NAT.check(NAT.lib().fsc_fp32_fma_probe(packed, blocks, 4096, NAT.ptr(out), NAT.C.byref(flops),
                                                   NAT.stream_ptr(device)), "fsc_fp32_fma_probe")
            t1.record()
            torch.cuda.synchronize()
            if r:
                times.append(t0.elapsed_time(t1))
        best["packed" if packed else "scalar"] = flops.value / (min(times) / 1e3) / 1e12
    form = max(best, key=best.get)
    return {"tflops": best[form], "scalar_tflops": best["scalar"], "packed_tflops": best["packed"],
            "how": f"FMA probe (fsc_fp32_fma_probe, {form} FMAs, {blocks} x 256 threads, best of {reps}, "
                   "CUDA events)"}


def timed_steps(args, world, step):
    """args.steps steps between CUDA events on the launching stream, clocks sampled meanwhile;
    no stage profiling inside."""
    dev = torch.cuda.current_device() if world == 1 else int(os.environ.get("LOCAL_RANK", 0))
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev, rank_path(args.clocks_csv, int(os.environ.get("RANK", 0)), world)) as clk:
        t0.record()
        for _ in range(args.steps):
            step()
        t1.record()
        torch.cuda.synchronize()
    summary = clk.summary()
    if world > 1:  # every GPU of the job, not only rank 0's
        gathered = [None] * world
        torch.distributed.all_gather_object(gathered, summary)
        summary = combine_clocks(gathered)
    return t0.elapsed_time(t1), summary


def stage_pass(args, world, step):
    """Per-stage CUDA-event times from a separate, untimed pass of the same steps.  Two extra
    entries: ``__step__`` (each step's time, for the time outside the stage marks) and, at N > 1,
    ``__halo__`` (each step's time inside its halo phases: the halo plan with its position
    exchange, the per-layer feature and gradient exchanges, the reverse force exchange)."""
    from fsctep_b200 import _native as NAT
    from fsctep_b200 import domain as D

    if world > 1:
        torch.distributed.barrier()
    stage_ms = {}
    NAT.profile_enable(True)
    for _ in range(args.stage_steps if args.stage_steps is not None else args.steps):
        D.HALO_TIMER = [] if world > 1 else None
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        step()
        t1.record()
        for name, ms in NAT.profile_read():
            stage_ms.setdefault(name, []).append(ms)
        torch.cuda.synchronize()
        stage_ms.setdefault("__step__", []).append(t0.elapsed_time(t1))
        if D.HALO_TIMER is not None:
            marks, halo, begin = D.HALO_TIMER, 0.0, None
            for which, ev in marks:
                if which == "begin":
                    begin = ev
                elif begin is not None:
                    halo += begin.elapsed_time(ev)
                    begin = None
            stage_ms.setdefault("__halo__", []).append(halo)
        D.HALO_TIMER = None
    NAT.profile_enable(False)
    torch.cuda.synchronize()
    return stage_ms


def run_native(args, rank, world, device):
    from fsctep_b200 import domain as D
    from fsctep_b200 import systems
    from fsctep_b200.ictd import ICTDEngine
    from fsctep_b200.neighbors import build_graph

    w = WORKLOADS[args.workload]
    cfg = model_cfg(w)
    eng = ICTDEngine(seeded_weights(cfg), cfg, device)
    dims = D.grid_for(world)
    if world == 1:
        sysd = systems.diamond_crystal(n_cells=w["cells"], seed=1000 + rank, Z=w["Z"])
    elif args.scaling == "strong":  # this rank's block of the one fixed crystal
        per = tuple(c // d for c, d in zip(w["cells"], dims))
        if any(p * d != c for p, d, c in zip(per, dims, w["cells"])):
            raise SystemExit(f"--scaling strong: cells {w['cells']} do not split into {dims} blocks")
        sysd = systems.diamond_block(D.block_of(rank, dims), dims, n_cells=per, seed=1000 + rank, Z=w["Z"])
    else:  # this rank's block of a (dims * cells) crystal
        sysd = systems.diamond_block(D.block_of(rank, dims), dims, n_cells=w["cells"], seed=1000 + rank, Z=w["Z"])
    n = sysd["pos"].shape[0]
    pos_d = torch.tensor(sysd["pos"], device=device)
    cell_d = torch.tensor(sysd["cell"], device=device)
    Z = torch.tensor(sysd["Z"], device=device, dtype=torch.int32)
    batch = torch.zeros(n, device=device, dtype=torch.int32)
    pos_h = torch.tensor(sysd["pos"]).pin_memory()
    forces_h = torch.empty(n, 3, dtype=torch.float32).pin_memory()
    energy_h = torch.empty(1, dtype=torch.float32).pin_memory()

    if world == 1:
        def step(pos, cell):
            g = build_graph(pos, cell, cfg.max_radius)
            energy, _ = eng.forward(pos, Z, batch, cell, g)
            out = eng.backward(want_virial=False)
            return energy, out["forces"], {"edges": g.num_edges, "ghosts": 0}
    elif args.halo == "layer":
        dec = D.Decomposition(sysd["cell"][0], dims, cfg.max_radius)
        info = {}

        def step(pos, cell):
            r = D.run_dist(D.layer_exchange_step(dec, rank, pos, Z, eng, cfg.max_radius))
            info["ghosts"], info["edges"] = r["num_ghosts"], r["num_edges"]
            return r["energy"].reshape(1), r["forces"], dict(info)
    else:
        dec = D.Decomposition(sysd["cell"][0], dims, cfg.num_interaction * cfg.max_radius)
        evaluate = D.ictd_evaluator(eng, sysd["cell"][0], cfg.max_radius)
        info = {}

        def counting_eval(p, s, nl, pbc):
            out = evaluate(p, s, nl, pbc)
            info["edges"] = eng._last[4].num_edges
            return out

        def step(pos, cell):
            r = D.run_dist(D.decomposed_step(dec, rank, pos, Z, counting_eval))
            info["ghosts"] = r["num_ghosts"]
            return r["energy"].reshape(1), r["forces"], dict(info)

    def e2e_step():
        pos = pos_h.to(device, non_blocking=True)
        energy, forces, g = step(pos, cell_d)
        forces_h.copy_(forces, non_blocking=True)
        energy_h.copy_(energy.to(torch.float32), non_blocking=True)
        return g

    for _ in range(args.warmup):
        _, _, info = step(pos_d, cell_d)
    torch.cuda.synchronize()
    E_edges = info["edges"]

    # kernel launches per step (counted once, outside the timed region)
    ours = None
    if not args.no_launch_count:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step(pos_d, cell_d)
            torch.cuda.synchronize()
        ours = sum(e.count for e in prof.key_averages() if "fsc::" in e.key or "cub::" in e.key)

    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ms_total, clk = timed_steps(args, world, lambda: step(pos_d, cell_d))
    stage_ms = stage_pass(args, world, lambda: step(pos_d, cell_d))
    if world > 1:
        torch.distributed.barrier()
    # end-to-end through the public API with host buffers
    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = e1 and e0.elapsed_time(e1)
    ms_total_t = torch.tensor([ms_total, ms_e2e], device=device, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(ms_total_t, op=torch.distributed.ReduceOp.MAX)
    ms_total, ms_e2e = float(ms_total_t[0]), float(ms_total_t[1])
    return dict(n=n, E=E_edges, ms_step=ms_total / args.steps, ms_e2e=ms_e2e / args.steps, stage_ms=stage_ms,
                clocks=clk, launches=None if ours is None else ours * args.steps, cfg=cfg,
                ghosts=info["ghosts"], dims=dims)


def run_batched(args, rank, world, device):
    """Config 1 (8 periodic frames, E + F + stress) or config 3 (256 molecules, o3 model with an
    external field per molecule, dipole and polarizability heads, E + F) on one GPU: one step =
    batched neighbour list + forward (+ heads) + backward."""
    from fsctep_b200.ictd import ICTDEngine
    from fsctep_b200.neighbors import build_graph

    w = WORKLOADS[args.workload]
    cfg = model_cfg(w)
    eng = ICTDEngine(seeded_weights(cfg), cfg, device)
    sysd = batched_system(w)
    n = sysd["pos"].shape[0]
    pos_d = torch.tensor(sysd["pos"], device=device)
    cell_d = torch.tensor(sysd["cell"], device=device)
    Z = torch.tensor(sysd["Z"], device=device, dtype=torch.int32)
    batch = torch.tensor(sysd["batch"], device=device, dtype=torch.int32)
    fp, pbc = sysd["frame_ptr"], sysd["pbc"]
    field = torch.tensor(sysd["field"], device=device) if "field" in sysd else None
    stress = w["system"] == "frames"
    B = cell_d.shape[0]
    pos_h = torch.tensor(sysd["pos"]).pin_memory()
    forces_h = torch.empty(n, 3, dtype=torch.float32).pin_memory()
    energy_h = torch.empty(B, dtype=torch.float32).pin_memory()
    info = {}

    def step(pos, cell):
        g = build_graph(pos, cell, cfg.max_radius, frame_ptr=fp, pbc=pbc)
        energy, _ = eng.forward(pos, Z, batch, cell, g, field=field)
        if cfg.o3:
            info["heads"] = eng.heads()
        out = eng.backward(want_virial=stress)
        info["edges"] = g.num_edges
        return energy, out["forces"]

    def e2e_step():
        energy, forces = step(pos_h.to(device, non_blocking=True), cell_d)
        forces_h.copy_(forces, non_blocking=True)
        energy_h.copy_(energy, non_blocking=True)

    for _ in range(args.warmup):
        step(pos_d, cell_d)
    torch.cuda.synchronize()
    if eng.status() != 0:
        raise RuntimeError(f"engine status {eng.status()}")
    ours = None
    if not args.no_launch_count:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step(pos_d, cell_d)
            torch.cuda.synchronize()
        ours = sum(e.count for e in prof.key_averages() if "fsc::" in e.key or "cub::" in e.key)
    torch.cuda.synchronize()
    ms_total, clk = timed_steps(args, world, lambda: step(pos_d, cell_d))
    stage_ms = stage_pass(args, world, lambda: step(pos_d, cell_d))
    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    return dict(n=n, E=info["edges"], ms_step=ms_total / args.steps, ms_e2e=e0.elapsed_time(e1) / args.steps,
                stage_ms=stage_ms, clocks=clk, launches=None if ours is None else ours * args.steps, cfg=cfg,
                ghosts=0, dims=(1, 1, 1), graphs=B)


def run_sparse(args, rank, world, device):
    """pure-cartesian-sparse energy + forces (+ virial) of a seeded crystal or water box; under
    torchrun the FCC crystal grows with the ranks and is decomposed as the ictd workloads are."""
    from fsctep_b200 import domain as D
    from fsctep_b200 import systems
    from fsctep_b200.neighbors import build_graph
    from fsctep_b200.sparse import SparseEngine

    w = WORKLOADS[args.workload]
    cfg = sparse_cfg(w)
    eng = SparseEngine(sparse_weights(cfg), cfg, device)
    dims = D.grid_for(world)
    if world == 1:
        sysd = sparse_system(w)
    else:  # this rank's block of a (dims * cells) FCC crystal
        sysd = systems.fcc_block(D.block_of(rank, dims), dims, n_cells=w["cells"], seed=1000 + rank)
    n = sysd["pos"].shape[0]
    pos_d = torch.tensor(sysd["pos"], device=device)
    cell_d = torch.tensor(sysd["cell"], device=device)
    Z = torch.tensor(sysd["Z"], device=device, dtype=torch.int32)
    batch = torch.zeros(n, device=device, dtype=torch.int32)
    pos_h = torch.tensor(sysd["pos"]).pin_memory()
    forces_h = torch.empty(n, 3, dtype=torch.float32).pin_memory()
    energy_h = torch.empty(1, dtype=torch.float32).pin_memory()
    info = {"ghosts": 0}
    if world == 1:
        def step(pos, cell):
            g = build_graph(pos, cell, cfg.max_radius)
            energy, _ = eng.forward(pos, Z, batch, cell, g)
            out = eng.backward(want_virial=True)
            info["edges"] = g.num_edges
            return energy, out["forces"]
    elif args.halo == "layer":
        dec = D.Decomposition(sysd["cell"][0], dims, cfg.max_radius)

        def step(pos, cell):
            r = D.run_dist(D.layer_exchange_step(dec, rank, pos, Z, eng, cfg.max_radius, want_virial=True))
            info["ghosts"], info["edges"] = r["num_ghosts"], r["num_edges"]
            return r["energy"].reshape(1), r["forces"]
    else:
        dec = D.Decomposition(sysd["cell"][0], dims, cfg.num_interaction * cfg.max_radius)
        evaluate = D.sparse_evaluator(eng, sysd["cell"][0], cfg.max_radius, want_virial=True)

        def counting_eval(p, s_, nl, pbc):
            out = evaluate(p, s_, nl, pbc)
            info["edges"] = eng._last[4].num_edges
            return out

        def step(pos, cell):
            r = D.run_dist(D.decomposed_step(dec, rank, pos, Z, counting_eval, want_virial=True))
            info["ghosts"] = r["num_ghosts"]
            return r["energy"].reshape(1), r["forces"]

    def e2e_step():
        energy, forces = step(pos_h.to(device, non_blocking=True), cell_d)
        forces_h.copy_(forces, non_blocking=True)
        energy_h.copy_(energy, non_blocking=True)

    for _ in range(args.warmup):
        step(pos_d, cell_d)
    torch.cuda.synchronize()
    if eng.status() != 0:
        raise RuntimeError(f"sparse engine status {eng.status()}")
    if world > 1:
        torch.distributed.barrier()
    ours = None
    if not args.no_launch_count:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step(pos_d, cell_d)
            torch.cuda.synchronize()
        ours = sum(e.count for e in prof.key_averages() if "fsc::" in e.key or "cub::" in e.key)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ms_total, clk = timed_steps(args, world, lambda: step(pos_d, cell_d))
    stage_ms = stage_pass(args, world, lambda: step(pos_d, cell_d))
    if world > 1:
        torch.distributed.barrier()
    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([ms_total, e0.elapsed_time(e1)], device=device, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    return dict(n=n, E=info["edges"], ms_step=float(ms[0]) / args.steps, ms_e2e=float(ms[1]) / args.steps,
                stage_ms=stage_ms, clocks=clk, launches=None if ours is None else ours * args.steps,
                cfg=cfg, ghosts=info["ghosts"], dims=dims)


REF_DIR = os.path.join(ROOT, "baseline", "_ref")
# CPU replicas (1/64 of the GPU workload's atoms where the reference can hold it in host memory;
# the sparse reference materialises per-edge fc.4 weights, P x C x C floats per edge and layer)
CPU_SAMPLES = {"si1m": (12, 12, 13), "si64k": (6, 6, 6), "water3k": 4, "fcc32k": (2, 2, 2), "fcc250k": (2, 2, 2)}


def cpu_sample(workload):
    """Seeded system of the CPU replica and a one-line description (shared by both CPU legs)."""
    from fsctep_b200 import systems

    w = WORKLOADS[workload]
    if w.get("system") in BATCHED:  # configs 1 and 3 run in full on the CPU
        sysd = batched_system(w)
        return sysd, f"the full workload ({sysd['pos'].shape[0]} atoms in {sysd['cell'].shape[0]} graphs)"
    rep = CPU_SAMPLES[workload]
    if w["model"] == "ictd":
        sysd = systems.diamond_crystal(n_cells=rep, seed=1000, Z=w["Z"])
        n = sysd["pos"].shape[0]
        what = (f"{n}-atom diamond Si replica ({rep[0]}x{rep[1]}x{rep[2]} conventional cells, "
                f"{n / (8 * np.prod(w['cells'])):.4f} of the GPU workload's atoms) of the same model")
    elif w["system"] == "water":
        sysd = systems.water_box(n_side=rep, box=w["box"] * rep / w["n_side"], seed=1000)
        what = f"{rep ** 3}-molecule water box of the same density ({3 * rep ** 3} atoms) and model"
    else:
        sysd = systems.fcc_crystal(n_cells=rep, seed=1000)
        what = f"{4 * int(np.prod(rep))}-atom FCC replica ({rep[0]}x{rep[1]}x{rep[2]} cells) of the same model"
    return sysd, what


def _reference_model(w, sd):
    """The reference's own module (installed unmodified under baseline/_ref), fp32, seeded weights."""
    from oracle import ref_import

    ref_import.install(REF_DIR)
    kw = dict(max_embed_radius=5.0, main_max_radius=5.0, main_number_of_basis=8, hidden_dim_conv=w["channels"],
              hidden_dim_sh=32, hidden_dim=64, num_interaction=w["num_interaction"], function_type_main="gaussian",
              max_atomvalue=w["max_atomvalue"], device=torch.device("cpu"))
    kw["function_type_main"] = w.get("basis", "gaussian")
    if w["model"] == "ictd":
        from molecular_force_field.models.pure_cartesian_ictd_layers_full import PureCartesianICTDTransformerLayer

        m = PureCartesianICTDTransformerLayer(lmax=2, internal_compute_dtype=torch.float32, **kw)
    elif w["model"] == "o3":
        from molecular_force_field.models.pure_cartesian_ictd_layers_o3 import PureCartesianICTDO3TransformerLayer

        m = PureCartesianICTDO3TransformerLayer(lmax=2, internal_compute_dtype=torch.float32, external_tensor_rank=1,
                                                external_tensor_irrep="1o", physical_tensor_outputs=O3_HEADS,
                                                o3_active_irreps=["0e", "1e", "1o", "2e"], **kw)
    else:
        from molecular_force_field.models.pure_cartesian_sparse_layers import PureCartesianSparseTransformerLayer

        m = PureCartesianSparseTransformerLayer(lmax=w["lmax"], **kw)
    m = m.float()
    m.load_state_dict({k: v.float() for k, v in sd.items()})
    return m.eval()


def cpu_reference(workload, steps, warmup):
    """Time the reference's CPU path on the workload's CPU replica: its own PyTorch modules from
    baseline/_ref (fp32 eager, all host threads); one step = forward + autograd forces (and the
    strain derivative for the virial where the GPU step computes one), neighbour list excluded.
    Without the installed reference, the oracle port of the same path is timed (kind "port")."""
    from oracle import neighbors as ON

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = WORKLOADS[workload]
    sparse = w["model"] == "sparse"
    cfg = sparse_cfg(w) if sparse else model_cfg(w)
    stress = sparse or w.get("system") == "frames"  # the GPU step's virial / stress
    sd = sparse_weights(cfg) if sparse else seeded_weights(cfg)
    sysd, what = cpu_sample(workload)
    batched = w.get("system") in BATCHED
    if batched:
        src, dst, S = ON.batched_neighbor_list(sysd["pos"], sysd["batch"], sysd["cell"], 5.0, sysd["pbc"])
    else:
        src, dst, S = ON.neighbor_list(sysd["pos"], sysd["cell"][0], 5.0)
    pos0 = torch.tensor(sysd["pos"], dtype=torch.float32)
    Z, b = torch.tensor(sysd["Z"]).long(), torch.tensor(sysd["batch"]).long()
    src_t, dst_t, S_t = torch.tensor(src).long(), torch.tensor(dst).long(), torch.tensor(S, dtype=torch.float32)
    cell = torch.tensor(sysd["cell"], dtype=torch.float32)
    kind = "reference" if os.path.isdir(os.path.join(REF_DIR, "molecular_force_field")) else "port"
    if kind == "reference":
        model = _reference_model(w, sd)

        kw = {}
        if "field" in sysd:
            kw = {"external_tensor": torch.tensor(sysd["field"], dtype=torch.float32), "return_physical_tensors": True}

        def step():
            pos = pos0.clone().requires_grad_(True)
            if stress:  # virial through the strain derivative (trainer convention)
                nb = cell.shape[0]
                strain = torch.zeros(nb, 3, 3, requires_grad=True)
                D = torch.eye(3) + 0.5 * (strain + strain.transpose(-1, -2))
                e = model(torch.einsum("ni,nij->nj", pos, D[b]), Z, b, src_t, dst_t, S_t, torch.bmm(cell, D))
                torch.autograd.grad(e.sum(), [pos, strain])
            else:
                out = model(pos, Z, b, src_t, dst_t, S_t, cell, **kw)
                e = out[0] if isinstance(out, tuple) else out
                torch.autograd.grad(e.sum(), [pos])
        how = "the reference's own PyTorch modules (baseline/_ref, unmodified; import shims: bare models package, " \
              "torch_scatter -> its utils/scatter fallback, e3nn soft_one_hot_linspace restated)"
    else:
        from oracle import ictd_model as OM
        from oracle import sparse_model as OS

        sd32 = {k: v.float() for k, v in sd.items()}
        args = (pos0, Z, b, src_t, dst_t, S_t, cell)
        if w["model"] == "o3":
            raise SystemExit("the o3 workload's CPU leg needs the reference installed under baseline/_ref")
        if sparse:
            def step():
                OS.sparse_energy_forces_stress(sd32, cfg, *args, want_stress=True)
        else:
            ocfg = OM.ICTDConfig(channels=cfg.channels, num_interaction=cfg.num_interaction,
                                 function_type=cfg.function_type, max_atomvalue=cfg.max_atomvalue)
            tabs = OM._TPTables(2, torch.float32)

            def step():
                OM.energy_forces_stress(sd32, ocfg, *args, want_stress=stress, tabs=tabs)
        how = "the oracle port of the reference CPU path (the reference is not installed under baseline/_ref)"
    for _ in range(warmup):
        step()
    times = []
    for _ in range(steps):
        t = time.perf_counter()
        step()
        times.append(time.perf_counter() - t)
    n = sysd["pos"].shape[0]
    med = float(np.median(times))
    try:
        cpu_model = next((ln.split(":", 1)[1].strip() for ln in open("/proc/cpuinfo") if ln.startswith("model name")),
                         "unknown")
    except OSError:
        cpu_model = "unknown"
    return {"value": n / med, "unit": "atom-steps/s", "cores": threads, "kind": kind,
            "sample": f"{what}, {len(src)} edges; fp32 PyTorch eager, energy + forces"
                      + (" + virial" if stress else "") + (" + field and heads" if "field" in sysd else "")
                      + f", neighbour list excluded; {how}",
            "steps": steps, "warmup": warmup, "statistic": "median", "cpu_model": cpu_model,
            "seconds_per_step": med}


def main():
    from fsctep_b200.domain import grid_for

    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--workload", default="si1m", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-launch-count", action="store_true", help="skip the torch.profiler launch count (for ncu)")
    ap.add_argument("--halo", default="layer", choices=["layer", "recompute"],
                    help="N > 1, pure-cartesian-ictd: per-layer ghost-feature exchange over a one-cutoff halo "
                         "(default) or ghosts recomputed over a num_interaction x cutoff halo")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="N > 1, pure-cartesian-ictd: a fixed crystal per GPU (weak, default) or one fixed "
                         "crystal cut over the GPUs (strong)")
    ap.add_argument("--stage-steps", type=int, default=None,
                    help="steps of the untimed per-stage pass (default: --steps)")
    ap.add_argument("--clocks-csv", default=None, help="where to write the nvidia-smi clock samples (default: a "
                                                        "temporary directory)")
    ap.add_argument("--conv2-tc", action="store_true",
                    help="pure-cartesian-ictd: the conv2 gate gradients on the tensor-core kernel instead of the "
                         "(faster, default) CUDA-core one")
    args = ap.parse_args()
    if args.conv2_tc and args.impl == "native":
        from fsctep_b200 import _native as NAT

        NAT.lib().fsc_ictd_set_conv2_path(1)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    metric = "atom-steps/s (E+F)"
    w = WORKLOADS[args.workload]
    sparse = w["model"] == "sparse"
    batched = w.get("system") in BATCHED
    if batched and (world > 1 or args.gpus > 1):
        raise SystemExit(f"--workload {args.workload}: runs on one GPU")
    if sparse and w["system"] != "fcc" and (world > 1 or args.gpus > 1):
        raise SystemExit(f"--workload {args.workload}: runs on one GPU (the FCC workloads decompose over GPUs)")
    n_atoms = int(np.prod(w["cells"])) * 8 if not (sparse or batched) else None
    config = {"workload": f"{args.workload}: pure-cartesian-ictd diamond Si {n_atoms} atoms (config 4)",
              "model": "pure-cartesian-ictd", "channels": w["channels"], "num_interaction": w["num_interaction"],
              "lmax": 2, "cutoff": 5.0, "radial_basis": "gaussian x8", "atoms_per_gpu": n_atoms if args.scaling == "weak" else n_atoms // max(args.gpus, 1),
              "parallelism": ("spatial%dx%dx%d" % grid_for(args.gpus)) if args.gpus > 1 else "single",
              "decomposition": None if args.gpus == 1 else (
                  ("blocks of " + ("a (50 px, 50 py, 50 pz)-cell crystal" if args.scaling == "weak" else
                                   "one 50^3-cell crystal (1,000,000 atoms in total)") + ", ") +
                  ("halo = cutoff = 5 A: one position halo exchange, a ghost-feature exchange after each "
                   "interaction layer that a later layer reads and its adjoint in the reverse pass, one reverse "
                   "ghost-force exchange (NCCL all_to_all), energy all_reduce" if args.halo == "layer" else
                   "halo = num_interaction x cutoff = 15 A of recomputed ghosts, one position halo exchange and "
                   "one reverse ghost-force exchange per step (NCCL all_to_all), energy all_reduce")),
              "step": "neighbour list + forward + backward (energy, forces)",
              "l2": "inputs larger than L2 (features 2.3 GB per layer at 1M atoms)"}
    if sparse:
        if w["system"] == "water":
            n_atoms = 3 * w["n_side"] ** 3
            what = (f"liquid-water-like box of {n_atoms // 3} H2O ({n_atoms} atoms) in a {w['box']} A cube, "
                    "O on a jittered grid (sigma 0.3 A), O-H 0.96 A, HOH 104.5 deg, random orientations (config 2)")
        else:
            n_atoms = 4 * int(np.prod(w["cells"]))
            what = (f"FCC metal-like crystal, a = 3.61 A, sigma = 0.1 A, single species, {n_atoms} atoms "
                    + ("(config 5's 250,000 atoms per GPU)" if n_atoms == 250000 else
                       "(config 5's model and lattice; the 250,000-atom per-GPU crystal is --workload fcc250k)"))
        config = {"workload": f"{args.workload}: pure-cartesian-sparse {what}", "model": "pure-cartesian-sparse",
                  "channels": w["channels"], "num_interaction": w["num_interaction"], "lmax": w["lmax"],
                  "max_rank_other": 1, "k_policy": "k0", "cutoff": 5.0, "radial_basis": "gaussian x8",
                  "atoms_per_gpu": n_atoms,
                  "parallelism": ("spatial%dx%dx%d" % grid_for(args.gpus)) if args.gpus > 1 else "single",
                  "decomposition": None if args.gpus == 1 else (
                      "blocks of a dims x cells FCC crystal, " +
                      ("halo = cutoff = 5 A: one position halo exchange, a ghost-feature exchange after each "
                       "interaction layer that a later layer reads and its adjoint in the reverse pass, one reverse "
                       "ghost-force exchange (NCCL all_to_all), whole-system E/N, energy and virial all_reduce"
                       if args.halo == "layer" else
                       "halo = num_interaction x cutoff = 15 A of recomputed ghosts (every layer on all local "
                       "atoms), one position halo exchange and one reverse ghost-force exchange per step (NCCL "
                       "all_to_all), energy and virial all_reduce")),
                  "step": "neighbour list + forward + backward (energy, forces, virial)",
                  "l2": "inputs smaller than L2 for water3k (re-read from L2 between steps); "
                        "per-layer aggregation buffers larger than L2 for the FCC workloads"}

    if batched:
        cfgb = model_cfg(w)
        if w["system"] == "frames":
            what = (f"config 1: {w['n_frames']} periodic frames of {w['n_atoms']} atoms, uniform in a {w['box']} A "
                    "cube (0.9 A rejection), 3 species; pure-cartesian-ictd C 32, 2 layers, 8 bessel; E + F + stress")
        else:
            what = (f"config 3: {w['n_mol']} non-periodic organic-like molecules of 10-30 atoms (C:H:N:O 3:5:1:1, "
                    "bonded chains 1.1-1.5 A); pure-cartesian-ictd-o3 irreps 0e,1e,1o,2e, C 64, 3 layers, external "
                    "1o field N(0, 0.05) per molecule, dipole + polarizability heads; E + F")
        config = {"workload": f"{args.workload}: {what}", "model": "pure-cartesian-ictd" + ("-o3" if cfgb.o3 else ""),
                  "channels": w["channels"], "num_interaction": w["num_interaction"], "lmax": 2, "cutoff": 5.0,
                  "radial_basis": f"{w['basis']} x8", "parallelism": "single",
                  "step": "batched neighbour list + forward" + (" + heads" if cfgb.o3 else "") + " + backward",
                  "l2": "inputs smaller than L2 (re-read from L2 between steps)"}

    if args.impl == "reference":
        if rank != 0:
            return
        r = cpu_reference(args.workload, max(1, min(args.steps, 5)), min(max(args.warmup, 0), 2))
        line = {"metric": metric, "value": r["value"], "unit": "atom-steps/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["seconds_per_step"] * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": config, "impl": "reference",
                "cpu_baseline": {k: r[k] for k in CPU_KEYS},
                "e2e": {"value": r["value"], "unit": "atom-steps/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300))
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(device)
    if batched:
        res = run_batched(args, rank, world, device)
    else:
        res = run_sparse(args, rank, world, device) if sparse else run_native(args, rank, world, device)
    n, E = res["n"], res["E"]
    n_total = n
    if world > 1:  # atoms of all ranks (blocks of a strong-scaling crystal differ slightly)
        t = torch.tensor([float(n)], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t)
        n_total = int(t.item())
    value = n_total / (res["ms_step"] / 1e3)
    e2e_value = n_total / (res["ms_e2e"] / 1e3)
    # dominant stage and its roofline
    stage_avg = {}
    nst = args.stage_steps if args.stage_steps is not None else args.steps
    step_ms = res["stage_ms"].pop("__step__", None)
    halo_ms = res["stage_ms"].pop("__halo__", None)
    for name, lst in res["stage_ms"].items():
        stage_avg[name] = (sum(lst) / nst, len(lst) / nst)
    dom = max(stage_avg, key=lambda k: stage_avg[k][0]) if stage_avg else None
    pk = peaks()
    roofline = None
    if dom is not None:
        per_step_ms, launches = stage_avg[dom]
        work = algorithmic_work(dom, n, E, res["cfg"])
        avg_launch_ms = per_step_ms / max(launches, 1)
        if work is not None:
            flops, nbytes = work
            ach = flops / (avg_launch_ms / 1e3) / 1e12
            hbm = nbytes / (avg_launch_ms / 1e3) / 1e9
            tpn = TRAFFIC_PER_NODE.get(dom)
            common = {"kernel": dom, "traffic": tpn * n if tpn is not None else None,
                      "traffic_source": "ncu si64k capture scaled by nodes" if tpn is not None else None,
                      "avg_launch_ms": avg_launch_ms, "algorithmic_bytes_per_launch": nbytes,
                      "algorithmic_tflops": ach}
            if dom.startswith("conv2_edge"):
                # CUDA-core tensor-product kernels: reported against HBM (their inputs are L2-resident
                # re-reads; the FP32 pipe and L1/shared-memory throughput are the real limits)
                roofline = dict(common, bound="hbm", achieved=hbm, peak=pk["hbm_gbs"], unit="GB/s",
                                frac=hbm / pk["hbm_gbs"], peak_source=pk["source"] + " HBM copy")
            else:
                how = ("kind::tf32 3xTF32 contractions and fc.4 GEMMs (plus CUDA-core epilogues); useful FLOPs, "
                       "the split issues 3 tf32 products per useful one" if dom.startswith("sparse_") else
                       "kind::f16 runs at the bf16 rate; useful FLOPs, the split issues 3 products per useful one")
                roofline = dict(common, bound="tensor", achieved=ach, peak=pk["bf16_tflops"], unit="TFLOP/s",
                                frac=ach / pk["bf16_tflops"], hbm_achieved_gbs=hbm,
                                peak_source=pk["source"] + " bf16 dense (" + how + ")")
    if roofline is not None:
        try:
            ctx = fp32_context(roofline, res["clocks"], torch.cuda.get_device_properties(device).multi_processor_count,
                               measure_fp32_peak(device))
        except Exception:  # reporting context only: never block the line
            ctx = None
        if ctx is not None:
            roofline["fp32_simt"] = ctx
    line = {"metric": metric, "value": value, "unit": "atom-steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_step"], "higher_is_better": True,
            "scaling": args.scaling if (world > 1 and not sparse) else "weak", "atoms_total": n_total,
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded positions and weights)",
            "config": config, "edges_per_gpu": E, "ghost_atoms_per_gpu": res["ghosts"], "roofline": roofline,
            "clocks": res["clocks"],
            "gpu_launches": res["launches"],
            "e2e": {"value": e2e_value, "unit": "atom-steps/s", "h2d_bytes_per_step": n * 3 * 8,
                    "d2h_bytes_per_step": n * 3 * 4 + 4},
            "stages_ms": {k: round(v[0], 3) for k, v in sorted(stage_avg.items(), key=lambda kv: -kv[1][0])}}
    if step_ms:  # time of a stage-pass step outside the engine's stage marks (neighbour list, halo work)
        line["unstaged_ms"] = round(sum(step_ms) / len(step_ms) - sum(v[0] for v in stage_avg.values()), 3)
    if halo_ms:
        line["halo_ms"] = round(sum(halo_ms) / len(halo_ms), 3)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_reference(args.workload, 3, 1)
        line["cpu_baseline"] = {k: r[k] for k in CPU_KEYS}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
