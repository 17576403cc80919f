#!/usr/bin/env python
"""Benchmark: screened RI-J J-build + gradient (FP64) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config C]

Metric: "J-build+grad s/step and Gpair-aux integrals/s (FP64) at 1/2/4/8 B200".
A step = splat quantities -> pair prep -> gamma -> [allreduce gamma] -> metric solve -> reverse
pass -> chain -> per-splat reductions -> chart reverse -> [allreduce gradients]; the pair list,
aux, metric and factor are refresh products, built before the timed region and reported apart.
``value`` = N_aux x live pairs (all ranks) / step seconds, in G pair-aux integrals/s.

Workload: configuration 3 of BASELINE.json by default ((H2O)343, M = 20,000, n_occ = 1715,
eps = 1e-7, 1.29e7 significant pairs), the configuration the metric's 1/2/4/8-GPU curve is quoted
on; synthetic seeded splats (gs_dft_b200.systems). For N > 1 launch with torchrun (one rank per GPU,
NCCL); the pair representatives are partitioned across ranks (strong scaling: total work fixed).
``--pairs P`` restricts the step to the first P significant pairs (a small case of the same
workload, for profiler captures); the JSON line then says so.
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
sys.path.insert(0, os.path.join(ROOT, "gs-dft_b200"))

METRIC = "J-build+grad s/step and Gpair-aux integrals/s (FP64) at 1/2/4/8 B200"
UNIT = "G pair-aux integrals/s"
# Algorithmic FP64 work per (aux, pair) integral, fixed from the reference's expression count
# (gs_dft/coulomb/ri.py:146-151,175-185 forward; :204-220 plus the dp2 chain reverse), with all 20
# Laplace nodes: 706 = 26 + 20 x 34 (forward), 2050 = 70 + 20 x 99 (reverse). With node screening the
# kernels count the nodes they evaluate (gsdft_node_evals) and the evaluated work is
# units x fixed + node evaluations x per-node.
FLOP_FWD, FLOP_VJP = 706, 2050
FLOP_FWD_FIXED, FLOP_FWD_NODE = 26, 34
FLOP_VJP_FIXED, FLOP_VJP_NODE = 70, 99
FP64_DATASHEET = 37e12
# DRAM bytes (read + write) per launch of each integral kernel, from one ncu capture (1-pass
# dram__bytes metrics) of this bench's own workload on one GPU, per configuration. Only the
# captured workloads are filled; others (and N > 1, whose slices change the reverse kernel's split
# count) report null.
NCU_TRAFFIC_N1 = {
    3: {"j_vjp_kernel": 1065.62e6 + 763.24e6, "j_forward_kernel": 8141.51e6 + 53.38e6},
}
L2_FLUSH_BYTES = 256 << 20
# FP64 work per (pair, atom) unit of the screened nuclear attraction kernel with its reverse sums,
# counted from gsdft_vne's operations (FMA = 2): 20 nodes x 50, y and m in two node passes 48, the
# per-atom epilogue 41 (the per-pair node constants, amortised over the atoms, are not counted).
FLOP_VNE = 1089


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, default=3)
    p.add_argument("--pairs", type=int, default=0,
                   help="use only the first P significant pairs (a small case for profiling)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    return p.parse_args()


# ------------------------------------------------------------------------------------------------
# clocks during the timed region
# ------------------------------------------------------------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for k, n in enumerate(names):
                    if r[5 + k].strip() in ("Active", "1"):
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------------
# the CPU oracle (checker / baseline)
# ------------------------------------------------------------------------------------------------
def oracle_problem(sy):
    """The CPU oracle's refresh for configuration ``sy``: pair list (C sweep), product aux, metric
    (C loop) and its factor (LAPACK). Not timed."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import gsdft_oracle as O
    import numpy as np
    q = O.full_quantities(sy.quat, sy.log_scale, sy.centers)
    pi, pj, v, n_sig, _ = O.neighbor_pairs_c(q, sy.eps)
    la, R = O.init_product_aux(q)
    aq = O.aux_quantities(la, R)
    V = O.aux_metric_c(*aq)
    V[np.diag_indices_from(V)] += sy.lam
    L = np.linalg.cholesky(V)
    del V
    return O, (sy.quat, sy.log_scale, sy.centers, sy.C_occ, sy.occ), aq, L, pi, pj, v


def cpu_step(O, sa, aq, L, pi, pj, v, k):
    """Seconds of one oracle step (energy + full gradient) on the first k live pairs."""
    t0 = time.perf_counter()
    O.energy_and_grad_c(sa, aq, L, pi[:k], pj[:k], v[:k])
    return time.perf_counter() - t0


def cpu_fixed_and_k(O, sa, aq, L, pi, pj, v, target_s):
    """The oracle step's per-step overhead a (solve on the n_aux factor, chart, scatters; seconds)
    measured on a tiny slice, and the slice k whose step takes about target_s. A step on k pairs
    costs a + b k; on the whole list the per-pair cost b dominates."""
    a = min(cpu_step(O, sa, aq, L, pi, pj, v, 16) for _ in range(2))
    k0 = min(400, pi.shape[0])
    b0 = max(cpu_step(O, sa, aq, L, pi, pj, v, k0) - a, 1e-6) / k0
    return a, int(min(pi.shape[0], max(k0, (target_s - a) / b0)))


def cpu_sample_rate(sy, target_s=10.0, prob=None):
    """The oracle step's rate on the configuration: integrals per second of its per-pair cost
    (the step on the whole list is a + b n_live with a the fixed per-step overhead), from one
    ~target_s step on the first k live pairs. Returns (rate, k, seconds, overhead a, threads)."""
    O, sa, aq, L, pi, pj, v = prob or oracle_problem(sy)
    n_aux = aq[0].shape[0]
    a, k = cpu_fixed_and_k(O, sa, aq, L, pi, pj, v, target_s)
    dt = cpu_step(O, sa, aq, L, pi, pj, v, k)
    b = max(dt - a, 1e-9) / k
    return n_aux / b, k, dt, a, O.c_threads()


def run_reference(args, rank, world):
    """The reference arm: the CPU restatement of the reference's step on this box's host cores, on
    the same configuration. Each timed step is a bounded sample (the first k live pairs x all aux,
    k sized for ~4 s a step); the line's value is the rate of the step's per-pair cost (the fixed
    per-step overhead a, measured apart, excluded: on the whole list a full step is a + b n_live
    with b n_live ~ hours), so it is the figure for a full-list step."""
    if rank != 0:
        return
    from gs_dft_b200.systems import make_config
    sy = make_config(args.config)
    prob = oracle_problem(sy)
    O, sa, aq, L, pi, pj, v = prob
    n_aux = aq[0].shape[0]
    n_live = int((v != 0).sum())
    a, k = cpu_fixed_and_k(O, sa, aq, L, pi, pj, v, target_s=4.0)
    for _ in range(args.warmup):
        cpu_step(O, sa, aq, L, pi, pj, v, k)
    ts = [cpu_step(O, sa, aq, L, pi, pj, v, k) for _ in range(args.steps)]
    t = sum(ts) / len(ts)
    b = max(t - a, 1e-9) / k
    val = n_aux / b / 1e9
    cores = O.c_threads()
    sample = (f"C/OpenMP restatement of the reference's RI-J step (oracle port; the JAX reference "
              f"cannot be installed offline), energy + full gradient, all 20 nodes: each step the "
              f"first {k} of {n_live} live pairs x all {n_aux} aux ({t:.2f} s); value = n_aux / "
              f"per-pair cost, the fixed per-step overhead ({a:.2f} s, measured on 16 pairs) "
              f"excluded; a full-list step would take {a + b * n_live:.0f} s")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
        "s_per_step_extrapolated": a + b * n_live,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": f"{sy.name} (BASELINE configs[{args.config}])", "M": sy.M,
                   "n_occ": sy.n_occ, "eps": sy.eps, "n_aux": n_aux, "live_pairs": n_live,
                   "pairs_per_step": k, "extrapolated": True},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
def dfma_peak(torch, lib, ptr, stream_handle):
    """Measured FP64 FMA throughput (FLOP/s) of this device at the current clocks."""
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    blocks, threads, iters = props.multi_processor_count * 8, 256, 20000
    out = torch.empty(blocks * threads, dtype=torch.float64, device="cuda")
    s = stream_handle()
    lib.call("gsdft_dfma_probe", ptr(out), 200, blocks, threads, s)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 0.0
    for _ in range(3):
        a.record()
        lib.call("gsdft_dfma_probe", ptr(out), iters, blocks, threads, s)
        b.record()
        torch.cuda.synchronize()
        best = max(best, 2.0 * 16 * iters * blocks * threads / (a.elapsed_time(b) * 1e-3))
    return best


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import ctypes

    import numpy as np
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import gs_dft_b200 as g
    from gs_dft_b200._lib import lib, ptr, stream_handle
    from gs_dft_b200.coulomb.engine import check_device_status
    from gs_dft_b200.ks.shard import ShardedRIJ
    from gs_dft_b200.systems import make_config

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    sy = make_config(args.config)
    t = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float64, device=dev)
    quat, log_scale, centers, C, occ = (t(sy.quat), t(sy.log_scale), t(sy.centers), t(sy.C_occ),
                                        t(sy.occ))
    splats = g.Splat(quat, log_scale, centers)

    # ---- refresh (timed apart; amortised at refresh = 10 steps in the report) -------------------
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    n0 = g.screening.count_significant(splats, sy.eps)
    pad_to = g.pad_rule(n0, 2.0, world)
    pi, pj, valid = g.neighbor_pairs(splats, eps=sy.eps, pad_to=pad_to)
    n_live = n0
    if args.pairs:
        n_live = min(args.pairs, n0)
        pi, pj, valid = (x[:n_live].contiguous() for x in (pi, pj, valid))
    aux = g.init_product_aux(splats)
    L = g.aux_cholesky(aux, sy.lam)
    beta, R, KN = aux.quantities()
    R = R.contiguous()
    # (the profiling case skips the n_aux^2 inverse factor to keep the device footprint small; its
    # step then solves by blocked substitution)
    sh = ShardedRIJ(pi, pj, valid, sy.M, sy.n_occ, beta, R, KN, L, rank, world,
                    balance=(quat, log_scale, centers), inverse_solve=not args.pairs)
    torch.cuda.synchronize()
    refresh_s = time.perf_counter() - t0
    eng = sh.engine
    n_eval_local = eng.plan.n_rep          # integrals this rank evaluates per aux
    n_aux = int(beta.shape[0])

    flush = torch.empty(L2_FLUSH_BYTES // 8, dtype=torch.float64, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def step():
        return sh.step(quat, log_scale, centers, C, occ)

    # ---- the step captured as CUDA graphs (one graph on one GPU; on several, the compute segments
    # between the two NCCL allreduces, which stay eager), with event brackets around the two
    # integral kernels captured inside them. The capture runs one eager step first. -------------
    eng.timing = True
    eng.events = {"forward": [], "vjp": []}
    graph = sh.capture(quat, log_scale, centers, C, occ, warmup=1)
    eng.timing = False
    cap = {k: v[-1] for k, v in eng.events.items()}   # the bracket events captured in the graph
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    check_device_status()

    # ---- device-timed steps (inputs resident; L2 flushed between steps, outside the events) -----
    clocks = Clocks(local)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches_per_step = graph.launches    # the library's kernels captured in the step's graphs
    phases = sh.phase_events() if world > 1 else None
    clocks.start()
    time.sleep(0.5)           # let the sampler come up before the timed region
    barrier()
    torch.cuda.synchronize()
    t_fwd = t_vjp = 0.0
    ph = None
    for k in range(args.steps):
        flush.fill_(float(k))
        starts[k].record()
        graph.replay(phases)
        ends[k].record()
        ends[k].synchronize()   # between steps, outside the timed window: read the kernel brackets
        t_fwd += cap["forward"][0].elapsed_time(cap["forward"][1])
        t_vjp += cap["vjp"][0].elapsed_time(cap["vjp"][1])
        if phases is not None:
            cur = [phases[i].elapsed_time(phases[i + 1]) for i in range(len(phases) - 1)]
            ph = cur if ph is None else [a + b for a, b in zip(ph, cur)]
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    launches = launches_per_step * args.steps
    step_ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends))
    t_fwd /= args.steps
    t_vjp /= args.steps
    check_device_status()
    nph = 5
    ph = [x / args.steps for x in ph] if ph is not None else [0.0] * nph
    tt = torch.tensor([step_ms, t_fwd, t_vjp] + ph, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    vals = [float(x) for x in tt.tolist()]
    step_ms, t_fwd, t_vjp, ph = vals[0], vals[1], vals[2], vals[3:]
    ms_per_step = step_ms / args.steps
    value = n_aux * n_live / (ms_per_step * 1e-3) / 1e9

    # ---- node evaluations of one step (outside the timed region; deterministic per step) -------
    ev_f, ev_r = ctypes.c_uint64(0), ctypes.c_uint64(0)
    lib.call("gsdft_node_evals", ctypes.byref(ev_f), ctypes.byref(ev_r), 1)
    graph.replay()
    lib.call("gsdft_node_evals", ctypes.byref(ev_f), ctypes.byref(ev_r), 1)
    evals_fwd, evals_vjp = int(ev_f.value), int(ev_r.value)

    # ---- end to end through the public API with host buffers ------------------------------------
    e2e = None
    if not args.no_e2e:
        ks = g.CoulombKS(coulomb=g.df(), screen=g.pairlist(eps=sy.eps), n_devices=1)
        e2e = measure_e2e(torch, g, ks, sy, dev, pi, pj, valid, aux, L, args, world, rank, sh,
                          barrier)

    peak = dfma_peak(torch, lib, ptr, stream_handle)
    next_rows = None
    if world == 1 and not args.pairs:
        # rows beyond the metric, measured after it; a failure here is recorded, never fatal
        next_rows = {}
        for name, fn in (("vne", measure_vne), ("k", measure_k), ("exact_j", measure_exact)):
            if name != "vne" and args.config > 2:
                next_rows[name] = {"skipped": (
                    "RI-K keeps the whole list's integral block, 8 n_rep n_aux bytes (1.0 TB here)"
                    if name == "k" else "O(n_rep^2): ~25 min at this size")
                    + "; measured at configurations 1 and 2"}
                continue
            try:
                next_rows[name] = fn(torch, g, sy, pi, pj, valid, quat, log_scale, centers, C,
                                     occ, flush, peak, args, aux=aux, L=L)
            except Exception as exc:          # noqa: BLE001 - reported in the JSON line
                next_rows[name] = {"error": f"{type(exc).__name__}: {exc}"}
    del graph                 # release every CUDA graph before the process group goes away
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    cpu = None
    if not args.no_cpu and world == 1:
        rate, k2, dt, a, cores = cpu_sample_rate(sy)
        cpu = {"value": rate / 1e9, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": (f"C/OpenMP oracle (restatement of the reference step, energy + full "
                          f"gradient, all 20 nodes) on the first {k2} of {n_live} live pairs x all "
                          f"{n_aux} aux, {dt:.1f} s on {cores} threads; value = n_aux / per-pair "
                          f"cost, the fixed per-step overhead ({a:.2f} s) excluded, i.e. the rate "
                          f"of a full-list step")}

    units = n_aux * n_eval_local
    dom = "j_vjp_kernel" if t_vjp >= t_fwd else "j_forward_kernel"
    t_dom = max(t_vjp, t_fwd)
    if dom == "j_vjp_kernel":
        flop_eval = units * FLOP_VJP_FIXED + evals_vjp * FLOP_VJP_NODE
        flop_20 = units * FLOP_VJP
        nodes_per_unit = evals_vjp / max(units, 1)
        # minimal DRAM bytes: pair records in (18 FP64), the 13 per-pair sums out, 8-FP64 aux records
        alg_bytes = n_eval_local * (18 + 13) * 8 + n_aux * 8 * 8
    else:
        flop_eval = units * FLOP_FWD_FIXED + evals_fwd * FLOP_FWD_NODE
        flop_20 = units * FLOP_FWD
        nodes_per_unit = evals_fwd / max(units, 1)
        alg_bytes = n_eval_local * 18 * 8 + n_aux * 6 * 8
    achieved = flop_eval / (t_dom * 1e-3)
    workload = f"{sy.name} (BASELINE configs[{args.config}])"
    if args.pairs:
        workload += f", first {n_live} significant pairs only (profiling case)"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "s_per_step": ms_per_step * 1e-3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": workload, "M": sy.M, "n_occ": sy.n_occ,
                   "eps": sy.eps, "n_aux": n_aux, "live_pairs": n_live, "pad_to": int(pad_to),
                   "evaluated_pairs": eng.plan.n_rep_total,
                   "twin_merge": ("each live (i,j)/(j,i) twin of the ordered list is evaluated once "
                                  "with the summed weight (same integral; outputs unchanged to "
                                  "1e-10); value counts N_aux x live ordered pairs per step"),
                   "node_screening": ("a warp stops the 20-node Laplace sum once every (aux, pair) "
                                      "it holds is 2^-87 below its first node (the rest is below the "
                                      "last bit); nodes evaluated per (aux, pair) per step: "
                                      f"forward {evals_fwd / max(units, 1):.2f}, reverse "
                                      f"{evals_vjp / max(units, 1):.2f} of 20 (rank 0)"),
                   "parallelism": f"pair-partition x{world}",
                   "partition": ("contiguous slices of the representatives with equal estimated "
                                 "integral cost (node counts of the screening rule on a sample of "
                                 "the aux)" if world > 1 else "one device"),
                   "l2": "flushed between steps",
                   "execution": ("step replayed from CUDA graphs: one graph on 1 GPU; on N GPUs the "
                                 "compute segments between the two NCCL allreduces, which run eagerly")},
        "refresh_s": refresh_s,
        # the refresh (pair list, aux, metric, factor, plan, inverse) amortised over the trainer's
        # default refresh interval of 10 steps (conf/config.yaml:22 of the reference)
        "refresh_amortized": {
            "refresh_every_steps": 10,
            "s_per_step": ms_per_step * 1e-3 + refresh_s / 10,
            "value": n_aux * n_live / (ms_per_step * 1e-3 + refresh_s / 10) / 1e9,
            "unit": UNIT},
        "kernel_ms": {"j_forward": t_fwd, "j_vjp": t_vjp},
        "roofline": {"bound": "fp64", "kernel": dom, "achieved": achieved / 1e12,
                     "peak": peak / 1e12, "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": "measured DFMA probe on this GPU in this run (MEASURED_PEAKS.json has no FP64 figure); datasheet 37 TFLOP/s",
                     "frac_of_datasheet": achieved / FP64_DATASHEET,
                     "flop_counting": ("evaluated: units x fixed + node evaluations x per-node "
                                       f"({FLOP_VJP_FIXED} + {FLOP_VJP_NODE}/node reverse, "
                                       f"{FLOP_FWD_FIXED} + {FLOP_FWD_NODE}/node forward)"),
                     "nodes_per_unit": nodes_per_unit,
                     "achieved_20node_equivalent": flop_20 / (t_dom * 1e-3) / 1e12,
                     "traffic": (NCU_TRAFFIC_N1[args.config][dom]
                                 if (args.config in NCU_TRAFFIC_N1 and world == 1
                                     and not args.pairs) else None),
                     "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + write.sum)",
                     "algorithmic_bytes": alg_bytes},
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    if world > 1:
        line["phases_ms"] = dict(zip(["forward", "allreduce_gamma", "solve_reverse_chain",
                                      "allreduce_gradients", "chart"], ph))
        line["phases_note"] = "CUDA events on rank streams between the step's segments, max over ranks"
    if e2e is not None:
        line["e2e"] = e2e
    if next_rows:
        line["next_rows"] = next_rows
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def measure_vne(torch, g, sy, pi, pj, valid, quat, log_scale, centers, C, occ, flush, peak, args,
                **_):
    """The screened nuclear attraction on the same pair list (not part of the metric): value and
    reverse-pass sums in one gsdft_vne call, device-timed with CUDA events on the launching stream,
    L2 flushed between launches outside the events."""
    from gs_dft_b200.coulomb.engine import RIJEngine
    from gs_dft_b200.screening import atom_records, pair_weight
    atoms = atom_records(sy.atoms, sy.charges, quat.device)
    eng = RIJEngine(pi, pj, pair_weight(valid).contiguous(), sy.M, sy.n_occ, atoms=atoms)
    eng.prepare(quat, log_scale, centers, C, occ)
    for _ in range(3):
        eng.external(sums=True)
    torch.cuda.synchronize()
    K = max(3, min(args.steps, 30 if args.config <= 1 else 3))
    total = 0.0
    for k in range(K):
        flush.fill_(float(k))
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        eng.external(sums=True)
        b.record()
        b.synchronize()
        total += a.elapsed_time(b)
    ms = total / K
    units = eng.plan.n_rep * eng.n_atoms
    flops = FLOP_VNE * units / (ms * 1e-3)
    return {"what": "screened V_ne on the pair list, value + reverse-pass sums (gsdft_vne: "
                    "vne_kernel + vne_sum), not part of the metric",
            "ms": ms, "launches_timed": K, "atoms": eng.n_atoms,
            "evaluated_pairs": eng.plan.n_rep, "units": "(pair, atom)",
            "units_per_s": units / (ms * 1e-3), "flop_per_unit": FLOP_VNE,
            "achieved_tflops": flops / 1e12, "frac_of_measured_fp64_peak": flops / peak,
            "E_ne": float(eng.E_ne[0])}


def measure_k(torch, g, sy, pi, pj, valid, quat, log_scale, centers, C, occ, flush, peak, args,
              aux=None, L=None):
    """Screened RI-K on the same pair list and aux (not part of the metric): E_K and its full
    gradient per step (RIKEngine.step), device-timed with CUDA events, L2 flushed between steps."""
    beta, R, KN = aux.quantities()
    eng = g.RIKEngine(pi, pj, valid, sy.M, sy.n_occ, beta, R, KN, L)
    big = args.config >= 2            # seconds per step: one warm-up, one timed step
    for _ in range(1 if big else 2):
        eng.step(quat, log_scale, centers, C)
    torch.cuda.synchronize()
    K = 1 if big else max(3, min(args.steps, 10))
    total = 0.0
    for k in range(K):
        flush.fill_(float(k))
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        eng.step(quat, log_scale, centers, C)
        b.record()
        b.synchronize()
        total += a.elapsed_time(b)
    ms = total / K
    n_aux, n_rep, K2 = eng.n_aux, eng.plan.n_rep, sy.n_occ * sy.n_occ
    integrals = n_aux * n_rep
    # integral block (forward integrand) + weighted reverse pass + the three n_aux x n_rep x K2 GEMMs
    flop = integrals * (FLOP_FWD + FLOP_VJP) + 3 * 2.0 * integrals * K2
    return {"what": "screened RI-K on the pair list: E_K + full gradient per step (integral "
                    "block, orbital products and their inverse-factor products as DMMA GEMMs, "
                    "weighted reverse pass, chain), not part of the metric",
            "ms_per_step": ms, "steps_timed": K, "evaluated_pairs": n_rep, "n_aux": n_aux,
            "n_occ": sy.n_occ, "occ_chunk": eng.occ_chunk, "integrals_per_s": integrals / (ms * 1e-3),
            "flop_per_step": flop, "achieved_tflops": flop / (ms * 1e-3) / 1e12,
            "frac_of_measured_fp64_peak": flop / (ms * 1e-3) / peak,
            "E_K": float(eng.E[0]), "workspace_bytes": eng.ws_bytes}


def measure_exact(torch, g, sy, pi, pj, valid, quat, log_scale, centers, C, occ, flush, peak,
                  args, **_):
    """The screened exact Hartree energy on the same pair list (O(n_rep^2) pair-pair integrals):
    the value, and the value with its full gradient (autograd through gsdft_exact_j_vjp); one
    warm-up and two timed evaluations of each with CUDA events (not part of the metric)."""
    def run(grad):
        if grad:
            leaves = [t.detach().clone().requires_grad_(True) for t in (quat, log_scale, centers, C)]
            E = g.screened_coulomb_energy(g.Splat(*leaves[:3]), leaves[3], occ, pi, pj,
                                          valid=valid)
            E.backward()
            return E
        return g.screened_coulomb_energy(g.Splat(quat, log_scale, centers), C, occ, pi, pj,
                                         valid=valid)

    def timed(grad):
        run(grad)
        torch.cuda.synchronize()
        total, K = 0.0, (1 if args.config >= 2 else 2)
        for k in range(K):
            flush.fill_(float(k))
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            E = run(grad)
            b.record()
            b.synchronize()
            total += a.elapsed_time(b)
        return total / K, K, E

    ms, K, E = timed(False)
    ms_grad, _, _ = timed(True)
    from gs_dft_b200.coulomb.engine import make_plan
    n_rep = make_plan(pi.to(torch.int32).contiguous(), pj.to(torch.int32).contiguous(),
                      valid.to(torch.float64).contiguous(), sy.M).n_rep_total
    pp = float(n_rep) * n_rep
    return {"what": "screened exact E_J (Schur-equivalent 20-node (pair|pair) kernel; plan, pair "
                    "prep and gsdft_exact_j per call) and E_J with its gradient (+ "
                    "gsdft_exact_j_vjp, chain, reductions), not part of the metric",
            "ms": ms, "ms_with_gradient": ms_grad, "evaluations_timed": K,
            "evaluated_pairs": n_rep, "pair_pairs_per_s": pp / (ms * 1e-3),
            "pair_pairs_per_s_reverse": pp / ((ms_grad - ms) * 1e-3), "E_J_exact": float(E)}


def measure_e2e(torch, g, ks, sy, dev, pi, pj, valid, aux, L, args, world, rank, sh, barrier):
    """Same metric through the public API (CoulombKS + autograd) with pinned host buffers: every
    step copies the parameters in and reads E and the gradients back."""
    import numpy as np
    hp = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float64).pin_memory()
    h_quat, h_ls, h_cen, h_C, h_occ = hp(sy.quat), hp(sy.log_scale), hp(sy.centers), hp(sy.C_occ), hp(sy.occ)
    d = lambda h: torch.empty(h.shape, dtype=torch.float64, device=dev)
    quat, ls, cen, C, occ = d(h_quat), d(h_ls), d(h_cen), d(h_C), d(h_occ)
    for x in (quat, ls, cen, C):
        x.requires_grad_(True)
    model = g.SplatModel(basis=g.Splat(quat, ls, cen), C=C, occupations=occ)
    state = g.SplatState(pairs=(pi, pj, valid), aux=aux, cholV=L)
    outs = [hp(np.zeros(1)), hp(sy.quat), hp(sy.log_scale), hp(sy.centers), hp(sy.C_occ)]
    h2d = sum(x.numel() * 8 for x in (h_quat, h_ls, h_cen, h_C, h_occ))
    d2h = sum(x.numel() * 8 for x in outs)

    def one():
        with torch.no_grad():
            for dst, src in ((quat, h_quat), (ls, h_ls), (cen, h_cen), (C, h_C), (occ, h_occ)):
                dst.copy_(src, non_blocking=True)
        for x in (quat, ls, cen, C):
            x.grad = None
        E = ks(model, state)
        E.backward()
        outs[0].copy_(E.detach().reshape(1), non_blocking=True)
        outs[1].copy_(quat.grad, non_blocking=True)
        outs[2].copy_(ls.grad, non_blocking=True)
        outs[3].copy_(cen.grad, non_blocking=True)
        outs[4].copy_(C.grad, non_blocking=True)

    def one_sharded():
        with torch.no_grad():
            for dst, src in ((quat, h_quat), (ls, h_ls), (cen, h_cen), (C, h_C), (occ, h_occ)):
                dst.copy_(src, non_blocking=True)
        o = sh.step(quat.detach(), ls.detach(), cen.detach(), C.detach(), occ)
        outs[0].copy_(o["E"].reshape(1), non_blocking=True)
        outs[1].copy_(o["g_quat"], non_blocking=True)
        outs[2].copy_(o["g_log_scale"], non_blocking=True)
        outs[3].copy_(o["g_centers"], non_blocking=True)
        outs[4].copy_(o["g_C"], non_blocking=True)

    fn = one if world == 1 else one_sharded
    # at the large configurations a step takes seconds: the end-to-end figure uses its own short
    # run (declared in the line), the device-timed headline the full one
    n_warm = args.warmup if args.config <= 1 else 1
    n_steps = args.steps if args.config <= 1 else min(args.steps, 3)
    for _ in range(n_warm):
        fn()
    torch.cuda.synchronize()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n_steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    barrier()
    ms = a.elapsed_time(b) / n_steps
    tt = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item())
    n_aux = int(aux.n_basis)
    n_live = int((valid != 0).sum().item())
    return {"value": n_aux * n_live / (ms * 1e-3) / 1e9, "unit": UNIT, "ms_per_step": ms,
            "steps": n_steps, "warmup": n_warm,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "api": "CoulombKS(model, state) + torch autograd" if world == 1 else "ShardedRIJ.step"}


if __name__ == "__main__":
    main()
