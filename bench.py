"""Benchmark of the FlashDiffusion DMAP matvec on B200 (kernel evals/s = N_q * N_k / t).

Workload (default, ``--config c5``): configuration 5 of the benchmark set,
the scale-out block DMAP — N = 2,000,000 points in d = 128 on a seeded
10-dimensional tanh manifold, median-rule beta, alpha = 0.5, an N x 32 N(0,1)
block right-hand side; fp16 tensor-core tiles, fp32 accumulation, P.V as a
second tcgen05 GEMM.  A step is one normalised block DMAP product
out = rscale * K(rscale * V) over all N x N pairs (row-sharded over the GPUs
for N > 1, followed by the NCCL all-gather of the output shards).  After the
timed steps: the r = 1 matvec on the same points (key ``c5r1``), and the time
to k = 32 eigenpairs by LOBPCG on the block operator.  ``--config c2|c3|c4``
measure the other configurations.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
       (N > 1: launched by torch.distributed.run, one rank per GPU)

The reference arm (--impl reference) times the reference algorithm's own CPU
implementation (the NumPy tile loop, restated in oracle/fd_oracle.py and
pinned to the reference's outputs) on the host cores, each step a bounded
seeded row sample of the same workload, scaled to evals/s.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "c2": dict(workload="c2: DMAP matvec, Gaussian mixture N={n} d=64, r=1, alpha=0.5",
               n=200_000, d=64, r=1, mode="dmap"),
    "c3": dict(workload="c3: AMAP matvec (Q != K), 6-D manifold N_q=N_k={n} d=64, r=1, alpha=0.5",
               n=500_000, d=64, r=1, mode="amap"),
    "c4": dict(workload="c4: Doob matvec, Langevin double well {n} frames d=66, r=1, alpha=0.5",
               n=500_000, d=66, r=1, mode="doob"),
    "c5": dict(workload="c5: DMAP block matvec, tanh manifold N={n} d=128, r=32, alpha=0.5",
               n=2_000_000, d=128, r=32, mode="dmap"),
    # the north-star target: the single-vector DMAP matvec at the configuration-5 size
    "c5r1": dict(workload="c5r1: DMAP matvec, tanh manifold N={n} d=128, r=1, alpha=0.5",
                 n=1_000_000, d=128, r=1, mode="dmap"),
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default="c5", choices=sorted(CONFIGS))
    p.add_argument("--no-lanczos", action="store_true")
    p.add_argument("--cpu-rows", type=int, default=0, help="rows of the CPU sample (0 = auto)")
    p.add_argument("--n", type=int, default=0, help="override the number of points (small profiling cases)")
    p.add_argument("--no-lobpcg", action="store_true", help="block configurations: skip LOBPCG to k = r eigenpairs")
    p.add_argument("--lobpcg-tol", type=float, default=1e-3)
    p.add_argument("--lobpcg-tol2", type=float, default=1e-5)
    p.add_argument("--lobpcg-final", default="f16", choices=["f16", "f16x3"],
                   help="tiles of the last LOBPCG stage: 16-bit with one key tile per accumulation group, or the "
                        "fp32-class tiles (the precision ramp; pair with --lobpcg-tol2 1e-7)")
    p.add_argument("--tiles", default="f16", choices=["f16", "bf16", "f16x3", "fp32"],
                   help="tile precision of the timed operator (default the 16-bit fp16 tiles)")
    a = p.parse_args()
    if a.n:
        for c in CONFIGS.values():
            c["n"] = a.n
    return a


def make_data(cfg, seed=0):
    """(Q, K or None, beta, h or None) for a configuration (seeded synthetic)."""
    from flashdiffusion_b200 import synthetic
    c = CONFIGS[cfg]
    if cfg == "c2":
        X, beta = synthetic.gaussian_mixture(n=c["n"], d=c["d"], seed=seed)
        return X, None, beta, None
    if cfg == "c3":
        Q, K, beta = synthetic.amap_manifold(n=c["n"], d=c["d"], seed=seed)
        return Q, K, beta, None
    if cfg == "c4":
        X, beta, h, _ = synthetic.langevin_trajectory(n_frames=c["n"], d=c["d"], seed=seed)
        return X, None, beta, h
    X, beta = synthetic.tanh_manifold(n=c["n"], d=c["d"], seed=seed)
    return X, None, beta, None


def _cpu_attach(spec):
    from multiprocessing import shared_memory
    shm = shared_memory.SharedMemory(name=spec[0])
    return shm, np.ndarray(spec[1], dtype=np.float32, buffer=shm.buf)


def _cpu_worker(job):
    """One host process: the reference tile loop on a block of query rows (timed inside)."""
    from threadpoolctl import threadpool_limits
    from oracle import fd_oracle as O
    qspec, kspec, idx, beta, r, seed = job
    qs, Q = _cpu_attach(qspec)
    ks, K = (qs, Q) if kspec is None else _cpu_attach(kspec)
    v = np.random.default_rng(seed + 1).standard_normal((K.shape[0], r))
    with threadpool_limits(limits=1):
        t0 = time.perf_counter()
        O.flash_diffusion(Q[idx], K, v, beta)
        dt = time.perf_counter() - t0
    del Q, K
    qs.close()
    if kspec is not None:
        ks.close()
    return dt


class CpuSampler:
    """Times the reference algorithm (NumPy tile loop of ``oracle/fd_oracle.py``) on
    seeded query rows x all keys, split over one host process per core (NumPy
    holds the GIL between its calls, so threads do not scale; each process
    keeps BLAS to one thread).  Q and K sit in shared memory.  The row/column
    scales are ones: they cost O(N) and do not change the tile loop timed."""

    def __init__(self, Q, K, beta, r=1, procs=None):
        import multiprocessing as mp
        from multiprocessing import shared_memory
        self.beta, self.r, self.nq = beta, r, Q.shape[0]
        self.nk = Q.shape[0] if K is None else K.shape[0]
        self.procs = max(1, procs or os.cpu_count() or 1)
        self.shms, self.specs = [], []
        for A in (Q, K):
            if A is None:
                self.specs.append(None)
                continue
            A = np.ascontiguousarray(A, dtype=np.float32)
            shm = shared_memory.SharedMemory(create=True, size=max(A.nbytes, 1))
            np.ndarray(A.shape, dtype=np.float32, buffer=shm.buf)[...] = A
            self.shms.append(shm)
            self.specs.append((shm.name, A.shape))
        self.pool = mp.get_context("spawn").Pool(self.procs)

    def sample(self, rows, seed=0):
        """(evals/s, seconds, processes) for `rows` seeded rows x all keys (wall clock over the pool)."""
        idx = np.sort(np.random.default_rng(seed).choice(self.nq, rows, replace=False))
        parts = [p_ for p_ in np.array_split(idx, self.procs) if p_.size]
        jobs = [(self.specs[0], self.specs[1], p_, self.beta, self.r, seed) for p_ in parts]
        self.pool.map(_cpu_worker, [(j[0], j[1], j[2][:4], j[3], j[4], j[5]) for j in jobs])   # warm
        t0 = time.perf_counter()
        self.pool.map(_cpu_worker, jobs, chunksize=1)
        dt = time.perf_counter() - t0
        return rows * self.nk / dt, dt, len(parts)

    def close(self):
        self.pool.close()
        self.pool.join()
        for shm in self.shms:
            shm.close()
            shm.unlink()


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# DRAM bytes per launch of the dominant kernel from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum; the capture commands are in
# the named profile summaries).
TRAFFIC = {"c2": (69.3e6, "profiles/tc_kernel_c2_dmap_matvec.md"),
           "c5": (661.2e9, "profiles/tc_block_kernel_c5_2m_traffic.md")}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), d.get("sm_max_mhz", 1965.0), "measured"
    return 6650.0, 1590.0, 1965.0, "fallback"


def workload_config(name, beta):
    """The `config` object of the JSON line: the workload only, identical in both arms."""
    c = CONFIGS[name]
    op_mb = c["n"] * (((c["d"] + 6 + 15) // 16) * 16) * 2 / 1e6
    return {"workload": c["workload"].format(n=c["n"]), "n_q": c["n"], "n_k": c["n"], "d": c["d"], "r": c["r"],
            "alpha": 0.5, "beta": beta, "mode": c["mode"], "seed": 0,
            "l2": ("packed operand %.0f MB %s the 126 MB L2; the GPU arm writes 256 MB between timed steps"
                   % (op_mb, "larger than" if op_mb > 126 else "within"))}


def run_reference(args):
    """The reference algorithm's CPU implementation, timed on the host cores.

    Each step is a bounded sample of the workload (seeded query rows x all
    keys, r right-hand-side columns), timed as a whole; `value` is the sampled
    evaluations per second and `ms_per_step` the measured time of one sampled
    step.  The projection to one full N x N product is a separate key."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    Q, K, beta, _ = make_data(args.config)
    cs = CpuSampler(Q, K, beta, cfg["r"])
    rows = args.cpu_rows or 64 * cs.procs
    for _ in range(args.warmup):
        cs.sample(min(rows, 8 * cs.procs))
    res = [cs.sample(rows, seed=s_) for s_ in range(args.steps)]
    cs.close()
    v = float(np.mean([x[0] for x in res]))
    step_s = float(np.mean([x[1] for x in res]))
    cores = res[0][2]
    n = cfg["n"]
    line = {"impl": "reference", "metric": "kernel evals/sec per matvec (N^2/t)", "value": v, "unit": "evals/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * step_s, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 GEMM + f64 exp/accumulate", "data": "synthetic (seeded generator)",
            "config": workload_config(args.config, beta),
            "arm": {"kind": "host processes, one BLAS thread each", "sample_rows_per_step": rows,
                    "evals_per_step": float(rows) * n},
            "full_product_s_projected": float(n) * n / v,
            "cpu_baseline": {"value": v, "unit": "evals/s", "cores": cores, "kind": "port",
                             "sample": f"{rows} seeded rows x all {n} keys x r={cfg['r']} per step over {cores} "
                                       "processes, scaled to evals/s"},
            "e2e": {"value": v, "unit": "evals/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from flashdiffusion_b200 import native
    from flashdiffusion_b200.distributed import ShardedOperator
    native.require_device(local)
    cfg = CONFIGS[args.config]
    Q, K, beta, h = make_data(args.config)
    nq, d = Q.shape
    nk = nq if K is None else K.shape[0]
    r = cfg["r"]
    dev = torch.device("cuda", local)
    Qd = torch.from_numpy(Q).to(dev)
    Kd = None if K is None else torch.from_numpy(K).to(dev)
    hd = None if h is None else torch.from_numpy(h).to(dev)

    # operator set-up (packing) and the Coifman-Lafon prepass, timed on the device
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    op = ShardedOperator(Qd, Kd, beta, 0.5, args.tiles, mode=cfg["mode"], h=hd)
    torch.cuda.synchronize()
    setup_s = time.perf_counter() - t0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    op.fit()
    e1.record()
    torch.cuda.synchronize()
    prepass_s = e0.elapsed_time(e1) / 1e3

    shape = (nk,) if r == 1 else (nk, r)
    v = torch.from_numpy(np.random.default_rng(1).standard_normal(shape)).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)     # 256 MB > 126 MB L2

    for _ in range(args.warmup):
        op.matvec_device(v)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.25)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ken = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    for i in range(args.steps):
        flush.zero_()                      # L2 flush between timed steps (outside the step events)
        starts[i].record()
        vl = op.matvec_shard(v)
        ken[i].record()
        op.gather_shards(vl, r == 1)
        ends[i].record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    step_ms = float(np.sum([a.elapsed_time(b) for a, b in zip(starts, ends)])) / args.steps
    kern_ms = float(np.sum([a.elapsed_time(b) for a, b in zip(starts, ken)])) / args.steps
    t = torch.tensor([step_ms, kern_ms, prepass_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, kern_ms, prepass_s = [float(x) for x in t.cpu()]

    # end to end with host buffers: pinned host V -> device, product (+ gather), result -> pinned host
    pinned_v = torch.from_numpy(np.random.default_rng(2).standard_normal(shape)).pin_memory()
    pinned_out = torch.empty((nq,) if r == 1 else (nq, r), dtype=torch.float64).pin_memory()
    for _ in range(2):
        pinned_out.copy_(op.matvec_device(pinned_v.to(dev, non_blocking=True)))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_steps = max(3, args.steps // 2)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        vd = pinned_v.to(dev, non_blocking=True)
        pinned_out.copy_(op.matvec_device(vd), non_blocking=False)
    torch.cuda.synchronize()
    e2e_s = torch.tensor([(time.perf_counter() - t0) / e2e_steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_s.item())

    # Lanczos time to k eigenpairs through the precision ramp (16-bit tiles until
    # their rounding floor, then fp32-class tiles with an fp64 Rayleigh-Ritz),
    # device fp64 basis, outside the timed region
    # block configurations: the single-vector (r = 1) DMAP matvec on the same
    # points and operator, the north-star kernel (kernel-only events, L2 flushed)
    r1 = None
    if r > 1:
        v1 = v[:, 0].contiguous()
        for _ in range(2):
            op.matvec_local(v1)
        r1_ev = []
        for _ in range(3):
            flush.zero_()
            a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a_.record()
            op.matvec_local(v1)
            b_.record()
            r1_ev.append((a_, b_))
        torch.cuda.synchronize()
        t1 = torch.tensor([float(np.mean([x.elapsed_time(y) for x, y in r1_ev]))], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t1, op=dist.ReduceOp.MAX)
        r1 = {"workload": f"DMAP matvec, r=1, same {nq} points and operator", "kernel_ms": float(t1.item()),
              "value": float(nq) * nk / (float(t1.item()) / 1e3), "unit": "evals/s"}

    lanczos = None
    if not args.no_lanczos and cfg["mode"] in ("dmap", "doob") and r == 1:
        from flashdiffusion_b200.eigensolver import ramp_eigsh
        # configuration 2: k = 16 of the DMAP operator; configuration 4: k = 8 of the
        # Doob operator, through its symmetric similar form
        kk = 16 if cfg["mode"] == "dmap" else 8
        emode = "dmap" if cfg["mode"] == "dmap" else "doob_sym"
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        lo = op if emode == "dmap" else ShardedOperator(Qd, Kd, beta, 0.5, "f16", mode=emode, h=hd).fit()
        # a Krylov basis of 4k vectors (the reference's ARPACK default is 2k+1):
        # fewer restarts, 224 instead of 237 products at c2 (2.86 s against 3.14-3.42 s)
        vals, _, info = ramp_eigsh(lo, lambda: ShardedOperator(Qd, Kd, beta, 0.5, "f16x3", mode=emode, h=hd).fit(),
                                   nq, kk, tol=1e-7, ncv=min(4 * kk, nq))
        torch.cuda.synchronize()
        lt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(lt, op=dist.ReduceOp.MAX)
        lanczos = {"k": kk, "operator": emode, "seconds": float(lt.item()), "n_matvec": info.n_matvec, "tol": 1e-7,
                   "stages": info.stages, "max_rel_residual": info.stages[-1]["max_rel_residual"],
                   "top_eigenvalues": [float(x) for x in vals[:4]]}
        # the Lanczos vector operations alone: one full reorthogonalisation
        # step (fd_lanczos_reorth) against a basis of ncv rows, HBM bytes =
        # three reads of the basis + the vectors, over CUDA-event time
        ncv = min(4 * kk, nq)
        Vb = torch.randn((ncv + 1, nq), dtype=torch.float64, device=dev)
        wv = torch.randn(nq, dtype=torch.float64, device=dev)
        cf = torch.zeros(ncv + 2, dtype=torch.float64, device=dev)
        wsz = native.lanczos_workspace(nq, ncv, dev)
        for _ in range(3):
            native.lanczos_reorth(Vb, ncv, wv, Vb[ncv], cf, wsz)
        flush.zero_()
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record()
        for _ in range(10):
            native.lanczos_reorth(Vb, ncv, wv, Vb[ncv], cf, wsz)
        b_.record()
        torch.cuda.synchronize()
        rt_ms = a_.elapsed_time(b_) / 10
        rbytes = 8.0 * (3 * ncv * nq + 5 * nq)
        lanczos["reorth"] = {"rows": ncv, "n": nq, "ms": rt_ms, "bytes": rbytes,
                             "achieved_gbs": rbytes / (rt_ms / 1e3) / 1e9,
                             "basis_bytes": 8.0 * ncv * nq}

    # configuration 5: k = 32 eigenpairs by LOBPCG whose block products are single
    # r = 32 passes of the tensor-core block kernel (16-bit tiles): stage 1 with
    # 8 key tiles per fp32 accumulation group to --lobpcg-tol, stage 2 warm-started
    # from stage 1 with one key tile per group (accumulation bias 8e-7) to
    # --lobpcg-tol2
    if not args.no_lanczos and r > 1 and not args.no_lobpcg:
        from flashdiffusion_b200.eigensolver import SolveInfo, lobpcg_core
        stages, X, vals = [], None, None
        t00 = time.perf_counter()
        for group, tol in ((0, args.lobpcg_tol), (1, args.lobpcg_tol2)):
            # stage 1 only needs residuals of 1e-3: P rounded once to fp16 (two
            # products, ~2.4e-4 noise per kernel value, 20 % faster); stage 2
            # the default three products with one key tile per accumulation group
            native.set_block_options(group, 2 if group == 0 else 0)
            info = SolveInfo()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            sop = op
            if group == 1 and args.lobpcg_final == "f16x3":
                # the ramp's fp32-class stage: block products on the split-operand tiles
                sop = ShardedOperator(Qd, Kd, beta, 0.5, "f16x3", mode=cfg["mode"], h=hd).fit()
            vals, X = lobpcg_core(lambda B: sop.matvec_device(B), nq, r, tol, 60, 42, dev, info, guard=16, X0=X)
            torch.cuda.synchronize()
            stages.append({"key_tiles_per_group": group or 8, "tiles": sop.op.precision, "tol": tol,
                           "products": 2 if group == 0 else 3,
                           "seconds": time.perf_counter() - t0,
                           "block_columns_applied": info.n_matvec, "iterations": info.n_restart,
                           "converged": info.converged, "max_rel_residual": float(np.max(info.residuals)),
                           "top_eigenvalues": [float(x) for x in vals[:4]]})
        native.set_block_options(0, 0)
        lt = torch.tensor([time.perf_counter() - t00], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(lt, op=dist.ReduceOp.MAX)
        lanczos = {"k": r, "method": "LOBPCG (16 guard columns), block tiles, two stages",
                   "seconds": float(lt.item()), "stages": stages,
                   "max_rel_residual": stages[-1]["max_rel_residual"], "top_eigenvalues": [float(x) for x in vals[:4]]}

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    hbm, bf16_tf, sm_max, peak_src = load_peaks()
    evals = float(nq) * float(nk)
    value = evals / (step_ms / 1e3)
    rows_local = op.rows[1] - op.rows[0]
    kern_evals = float(rows_local) * nk / (kern_ms / 1e3)
    sm_clock = (clk or {}).get("sm_mhz") or sm_max
    flops_per_eval = 2 * d + (2 * r if r > 1 else 0)
    mufu_peak = 16 * 148 * sm_max * 1e6          # ex2 per s at max SM clock (measured 15.9/clk/SM)
    tensor_peak_evals = bf16_tf * 1e12 / flops_per_eval
    peak_evals = min(mufu_peak, tensor_peak_evals)
    if lanczos is not None and "reorth" in lanczos:
        lanczos["reorth"]["peak_gbs"] = hbm
        lanczos["reorth"]["frac"] = lanczos["reorth"]["achieved_gbs"] / hbm
    if lanczos is not None:
        # the eigensolve against the same roofline: every product at the roofline rate
        # (Lanczos: r = 1 products; LOBPCG: r-column block products, block_columns / r of them)
        n_prod = lanczos.get("n_matvec") or sum(st["block_columns_applied"] for st in lanczos["stages"]) / r
        lanczos["roofline_seconds"] = n_prod * evals / (peak_evals * world)
        lanczos["roofline_frac"] = lanczos["roofline_seconds"] / lanczos["seconds"]
    if r1 is not None:
        r1_peak = min(mufu_peak, bf16_tf * 1e12 / (2 * d))
        r1["peak"] = r1_peak
        r1["roofline_frac"] = r1["value"] / world / r1_peak
    cpu_baseline = None
    if world == 1:   # the host baseline is taken on rank 0 of a 1-GPU run only
        cs = CpuSampler(Q, K, beta, r)
        if args.cpu_rows:
            cpu_rows = args.cpu_rows
        else:   # grow the sample until it takes 5-20 s of CPU work (per-call overheads
            # dominate small samples, so one small calibration overestimates the time)
            cpu_rows = max(64, 8 * cs.procs)
            while True:
                cpu_ev, cpu_dt, cpu_procs = cs.sample(cpu_rows)
                if cpu_dt >= 5.0 or cpu_rows >= nq:
                    break
                cpu_rows = int(min(nq, cpu_rows * min(16.0, max(2.0, 10.0 / max(cpu_dt, 1e-3)))))
        if args.cpu_rows:
            cpu_ev, cpu_dt, cpu_procs = cs.sample(cpu_rows)
        cs.close()
        cpu_baseline = {"value": cpu_ev, "unit": "evals/s", "cores": cpu_procs, "kind": "port",
                        "sample": f"{cpu_rows} seeded rows x all {nk} keys, r={r}: NumPy tile loop of the reference "
                                  f"algorithm, {cpu_procs} processes, {cpu_dt:.1f} s, scaled to evals/s"}
    line = {
        "metric": "kernel evals/sec per matvec (N^2/t)", "value": value, "unit": "evals/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": f"{args.tiles} tiles, f32 accumulate",
        "data": "synthetic (seeded generator)",
        "config": workload_config(args.config, beta),
        "arm": {"tiles": f"{op.op.precision} tcgen05" if op.op.precision != "fp32" else "fp32 SIMT",
                "parallelism": f"row-shard x{world}, NCCL all-gather of the output shards"},
        "roofline": {"bound": "mufu" if mufu_peak <= tensor_peak_evals else "tensor", "achieved": kern_evals,
                     "peak": peak_evals, "unit": "evals/s", "frac": kern_evals / peak_evals,
                     "traffic": TRAFFIC[args.config][0] if (args.config in TRAFFIC and not args.n and world == 1) else None,
                     "traffic_source": TRAFFIC.get(args.config, (None, None))[1],
                     "algorithmic_bytes_per_launch": 2 * (nq + nk) * (((d + 6 + 15) // 16) * 16) + 8 * (nk * r + nq * r),
                     "peak_basis": "min(MUFU ex2 16/clk/SM x 148 SMs x %.0f MHz, measured bf16 %.0f TFLOP/s / %d flop per eval)"
                                   % (sm_max, bf16_tf, flops_per_eval),
                     "tensor": {"achieved": kern_evals * flops_per_eval / 1e12, "peak": bf16_tf, "unit": "TFLOP/s",
                                "frac": kern_evals * flops_per_eval / 1e12 / bf16_tf, "peak_source": peak_src},
                     "frac_at_sampled_clock": kern_evals / min(16 * 148 * sm_clock * 1e6, tensor_peak_evals)},
        "cpu_baseline": cpu_baseline,
        "e2e": {"value": evals / e2e_s, "unit": "evals/s", "h2d_bytes_per_step": 8 * nk * r,
                "d2h_bytes_per_step": 8 * nq * r},
        "gpu_launches": (3 if r == 1 else 4) * args.steps,
        "prepass_s": prepass_s, "setup_s": setup_s, "kernel_ms": kern_ms,
        "lanczos": lanczos, "c5r1": r1, "clocks": clk,
    }
    print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
