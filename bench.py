"""Benchmark: LTC fwd+bwd throughput (B*T/s) of the sm_100a solver, 1..8 GPUs.

Default workload: configuration c3 (B=4096 batch-sharded over the ranks, T=128,
D=128, H=64, ode_unfolds=6, density 0.5/0.5): one training step = module forward
(LayerNorm, affine, softplus transforms, solver), sum loss, backward, gradient
all-reduce (SUM, NCCL, when N>1) and an Adam step.  Other configurations
(--config c0..c4) run forward+backward with the same harness.

  python bench.py [--gpus N --steps K --warmup W --config c3]
  torchrun --nproc-per-node N bench.py --gpus N ...
  python bench.py --impl reference     # reference CPU path (oracle port) on host cores

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "ltc-cuda_b200"))
sys.path.insert(0, REPO)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import synth  # noqa: E402

# DRAM bytes per (sample, timestep) of a kernel from one ncu capture of a smaller case
# of the same configuration, scaled to a launch by the (b,t) units it processes (the
# traffic is the saved V/R read and the g_sn/g_sd write, linear in B and T): c3 shape
# at B=1184 (dram__bytes_read + dram__bytes_write = 466.8 + 69.9 MB over 1184*128
# (b,t)); c4 at T=4 (246.5 + 57.2 MB over 1024*4 (b,t)).  Both with masked synapses
# skipped (the bench default).
NCU_TRAFFIC_PER_BT = {("c3", "recurrent_bwd"): 3541.0, ("c4", "recurrent_bwd"): 74136.0}

METRIC = "fwd+bwd sequence-timesteps/sec (B·T/s) at 1/2/4/8 B200; % FP32 roofline"
UNIT = "B*T/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c3", choices=sorted(synth.CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference_cuda"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--reference-cuda", type=int, default=1,
                    help="1 (default, N=1 only): also time the reference's own CUDA kernels in a child process")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--batch", type=int, default=None,
                    help="override the configuration's global batch (profiling captures of smaller cases)")
    ap.add_argument("--seq", type=int, default=None, help="override the sequence length T (profiling captures)")
    ap.add_argument("--lean", type=int, default=0,
                    help="1: memory-lean training (step-boundary states saved, unfolds recomputed in the backward)")
    ap.add_argument("--parity", type=int, default=1,
                    help="1 (default): check a slice against the reference before timing; 0: skip (profiling)")
    ap.add_argument("--skip-zero", type=int, default=1,
                    help="1 (default): the module lets the solver skip masked recurrent synapses (H <= 64 and 128 < H <= 512); 0: dense")
    ap.add_argument("--graph", type=int, default=None,
                    help="1 (default): replay the whole step as a captured CUDA graph; 0: eager launches")
    return ap.parse_args()


def measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "sm_max_mhz": 1965.0}, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (50 ms) of this rank's GPU while the timed region runs.

    ``start`` returns once the first sample is in, so that nvidia-smi's own start-up
    (which touches every GPU of the machine) is not inside the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        t0 = time.time()
        while not self.rows and self.proc.poll() is None and time.time() - t0 < 10:
            time.sleep(0.01)
        self.rows.clear()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 9 for i in range(4)
                          if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# --------------------------------------------------------------------------- CPU arm
# Batch/time slice of each configuration that the CPU arms time (samples are
# independent, so B*T/s on a slice is the rate of the whole workload).  The
# cpu_baseline leg of the GPU arm and the --impl reference arm use the same slice.
CPU_SLICE = {"c0": (24, 8), "c1": (16, 32), "c2": (8, 8), "c3": (256, 8), "c4": (1, 2)}


def reference_cpu_step(cfg, threads: int):
    """One fwd+bwd (sum loss) of the reference TorchScript path on a slice, on host cores.

    The reference's own ``ltc.py`` (staged by ``oracle/build_ref.py``) runs when it is
    present ("reference"); otherwise the oracle's restatement of it ("port")."""
    from oracle import reference_module as rm
    torch.set_num_threads(threads)
    Bs, Ts = CPU_SLICE[cfg.name]
    p, x = synth.make_workload(cfg, batch=Bs)
    x = x[:, :Ts].contiguous()
    # in the GPU arm's process the module name ltc_cuda is already this package's;
    # alone, the reference's own loader binds it (and must find its prebuilt kernels
    # on a CUDA machine rather than start a JIT build)
    binding = "ours" if "ltc_cuda" in sys.modules else "reference"
    why = rm.available(cuda=binding == "reference" and torch.cuda.is_available())
    if why is None:
        import logging
        logging.getLogger("ltc").setLevel(logging.ERROR)  # the reference logs its CPU fallback once
        ltc = rm.import_reference(binding)
        m = rm.reference_module(ltc, p, cfg.D, cfg.H, cfg.dt, cfg.U, cfg.density, cfg.sensory_density)

        def one():
            out, _ = m(x)  # CPU input: the reference dispatches to its TorchScript solver (ltc.py:293-326)
            out.sum().backward()
            m.zero_grad(set_to_none=True)
        kind, what = "reference", "reference ltc.py TorchScript path (module fwd+bwd, sum loss)"
    else:
        from oracle import ltc_oracle as orc
        params = {k: v.clone().requires_grad_(k in orc.parameter_names()) for k, v in p.items()}

        def one():
            out, _ = orc.module_forward(params, x, None, cfg.dt, cfg.U)
            out.sum().backward()
            for v in params.values():
                v.grad = None
        kind, what = "port", f"oracle restatement of the reference TorchScript path ({why})"
    return one, Bs, Ts, kind, what


def cpu_sample_rate(cfg, seconds: float, threads: int):
    """Reference CPU path timed on host cores for about ``seconds`` on the slice."""
    one, Bs, Ts, kind, what = reference_cpu_step(cfg, threads)
    one()
    one()  # warm-up (TorchScript profiles its first calls)
    n, t0 = 0, time.perf_counter()
    while True:
        one()
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 1000:
            break
    return {"value": n * Bs * Ts / el, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{cfg.name} slice B={Bs} T={Ts} (D={cfg.D} H={cfg.H} U={cfg.U}), {what}, "
                      f"{n} reps in {el:.1f}s"}


def run_reference(args, cfg, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    one, Bs, Ts, kind, what = reference_cpu_step(cfg, threads)
    for _ in range(max(3, args.warmup)):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    el = time.perf_counter() - t0
    value = args.steps * Bs * Ts / el
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": 1e3 * el / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": cfg.name, "B": Bs, "T": Ts, "D": cfg.D, "H": cfg.H, "U": cfg.U,
                       "sample_of": {"B": cfg.B, "T": cfg.T}},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                             "sample": f"{cfg.name} slice B={Bs} T={Ts} per step; {what}"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_cuda(args, cfg, rank):
    """The reference's own CUDA kernels (csrc/ltc_kernels.cu compiled for sm_100a by
    oracle/build_ref.py) driven through the reference module, timed like our arm:
    fwd + sum-loss bwd (+ Adam at c3) per step, L2 flushed between steps, CUDA events."""
    if rank != 0:
        return
    from oracle import reference_module as rm
    why = rm.available(cuda=True)
    if why:
        print(json.dumps({"impl": "reference_cuda", "unavailable": why}), flush=True)
        return
    ltc = rm.import_reference("reference")
    import ltc_cuda as ref_cuda  # the reference loader (oracle/_ref/ltc_cuda.py)
    if not ref_cuda._HAS_CUDA_KERNELS:
        print(json.dumps({"impl": "reference_cuda", "unavailable": "reference CUDA extension did not load"}))
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    p, x = synth.make_workload(cfg)
    m = rm.reference_module(ltc, p, cfg.D, cfg.H, cfg.dt, cfg.U, cfg.density, cfg.sensory_density).to(dev)
    x = x.to(dev)
    opt = torch.optim.Adam(m.parameters(), lr=1e-4, fused=True) if cfg.training_step else None
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def step():
        out, _ = m(x)
        out.sum().backward()
        if opt is not None:
            opt.step()
        m.zero_grad(set_to_none=True)

    # parity of the reference kernels against the reference TorchScript path on a slice
    par = module_parity(lambda mm, xx: mm(xx), lambda: rm.reference_module(
        ltc, p, cfg.D, cfg.H, cfg.dt, cfg.U, cfg.density, cfg.sensory_density).to(dev), ltc, p, cfg, dev)
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        flush.zero_()
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    line = {"metric": METRIC, "value": cfg.B * cfg.T / (ms / 1e3), "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True,
            "dtype": "f32", "data": "synthetic", "impl": "reference_cuda",
            "config": {"workload": cfg.name, "B": cfg.B, "T": cfg.T, "D": cfg.D, "H": cfg.H, "U": cfg.U,
                       "step": "train (fwd+bwd+adam)" if cfg.training_step else "fwd+bwd",
                       "kernels": "reference csrc/ltc_kernels.cu, nvcc -O3 --use_fast_math sm_100a"},
            "parity_vs_reference_torchscript": par}
    print(json.dumps(line), flush=True)


PARITY_SLICE = {"c0": (24, 8), "c1": (16, 32), "c2": (8, 64), "c3": (8, 128), "c4": (2, 64)}


def module_parity(run_ours, make_ours, ltc, p, cfg, dev):
    """Module fwd + sum-loss bwd of a candidate against the reference TorchScript path
    (``_force_torchscript``, ``ltc.py:293-326``) on the GPU, same seeded slice.
    Bars (north star): forward max-abs 1e-3; gradients rtol 5e-2 / atol 1e-2."""
    from oracle import reference_module as rm
    Bs, Ts = PARITY_SLICE[cfg.name]
    _, x = synth.make_workload(cfg, batch=Bs)
    x = x[:, :Ts].contiguous().to(dev)
    ref = rm.reference_module(ltc, p, cfg.D, cfg.H, cfg.dt, cfg.U, cfg.density, cfg.sensory_density).to(dev)
    ref._force_torchscript = True
    ro, (rh, _) = ref(x)
    ro.sum().backward()
    ours = make_ours()
    oo, (oh, _) = run_ours(ours, x)
    oo.sum().backward()
    fwd = max((oo - ro).abs().max().item(), (oh - rh).abs().max().item())
    rg = dict(ref.named_parameters())
    worst, ok = 0.0, True
    for n, q in ours.named_parameters():
        a, b = q.grad.double(), rg[n].grad.double()
        worst = max(worst, ((a - b).abs().max() / b.abs().max().clamp_min(1e-12)).item())
        ok = ok and bool(torch.allclose(a, b, rtol=5e-2, atol=1e-2))
    return {"slice": {"B": Bs, "T": Ts}, "fwd_max_abs": fwd, "grad_max_rel": worst,
            "pass": bool(fwd < 1e-3 and ok), "against": "reference ltc.py TorchScript path on the GPU"}


def rec_synapses(model, cfg, rows) -> int:
    """Recurrent synapses per unfold the kernels visit (see ltc_cuda.skip_zero_synapses)."""
    import ltc_layer
    if (getattr(model, "skip_zero_synapses", False) and (cfg.H <= 64 or cfg.H > 128) and model._skip_fits()
            and rows >= ltc_layer.SKIP_MIN_ROWS):
        return int(model.sparsity_mask.count_nonzero().item())
    return cfg.H * cfg.H


def sens_synapses(model, cfg, rows):
    """Sensory synapses per (b,t) the sensory forward and backward visit: the nonzero
    ones where the module lets the solver skip masked synapses (the forward whenever it
    skips the recurrent ones, the backward when its sensory mask fits), else D*H."""
    import ltc_layer
    full = cfg.D * cfg.H
    if not (getattr(model, "skip_zero_synapses", False) and model._skip_fits() and rows >= ltc_layer.SKIP_MIN_ROWS):
        return full, full
    nnz = int(model.sensory_sparsity_mask.count_nonzero().item())
    return nnz, (nnz if model._skip_sensory_fits() else full)


def our_parity(cfg, p, dev, skip_zero=True):
    """Parity of this build's module on a slice of the timed configuration, checked
    before the timed region against the reference TorchScript path (or, where the
    reference is not staged, the oracle restatement of it).  The slice runs the
    kernels the timed step runs: where the module skips masked synapses at full size,
    the slice's row threshold is lifted so that it skips them too."""
    import ltc_layer
    old_min = ltc_layer.SKIP_MIN_ROWS
    ltc_layer.SKIP_MIN_ROWS = 0 if skip_zero else old_min
    try:
        return _our_parity(cfg, p, dev, skip_zero)
    finally:
        ltc_layer.SKIP_MIN_ROWS = old_min


def _our_parity(cfg, p, dev, skip_zero):
    import ltc_layer
    from oracle import reference_module as rm

    def make():
        m = ltc_layer.TrueLiquidTimeConstant(cfg.D, cfg.H, dt=cfg.dt, ode_unfolds=cfg.U, sparsity=cfg.density,
                                             sensory_sparsity=cfg.sensory_density)
        m.load_state_dict(p)
        m.skip_zero_synapses = m.skip_zero_synapses and skip_zero
        return m.to(dev)
    if rm.available() is None:
        import logging
        logging.getLogger("ltc").setLevel(logging.ERROR)
        ltc = rm.import_reference("ours")
        return module_parity(lambda mm, xx: mm(xx), make, ltc, p, cfg, dev)
    from oracle import ltc_oracle as orc
    Bs, Ts = PARITY_SLICE[cfg.name]
    _, x = synth.make_workload(cfg, batch=Bs)
    x = x[:, :Ts].contiguous().to(dev)
    params = {k: v.to(dev).requires_grad_(k in orc.parameter_names()) for k, v in p.items()}
    ro, (rh, _) = orc.module_forward(params, x, None, cfg.dt, cfg.U)
    ro.sum().backward()
    m = make()
    oo, (oh, _) = m(x)
    oo.sum().backward()
    fwd = max((oo - ro).abs().max().item(), (oh - rh).abs().max().item())
    worst, ok = 0.0, True
    for n, q in m.named_parameters():
        a, b = q.grad.double(), params[n].grad.double()
        worst = max(worst, ((a - b).abs().max() / b.abs().max().clamp_min(1e-12)).item())
        ok = ok and bool(torch.allclose(a, b, rtol=5e-2, atol=1e-2))
    return {"slice": {"B": Bs, "T": Ts}, "fwd_max_abs": fwd, "grad_max_rel": worst,
            "pass": bool(fwd < 1e-3 and ok), "against": "oracle restatement (reference not staged)"}


def reference_cuda_subprocess(name, batch, seq, steps=5, warmup=3, timeout=900):
    """Run ``--impl reference_cuda`` in a child process (it binds the reference's own
    ``ltc_cuda`` module name) and return its JSON line, or why it is missing."""
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference_cuda", "--config", name,
           "--steps", str(steps), "--warmup", str(warmup)]
    if batch is not None:
        cmd += ["--batch", str(batch)]
    if seq is not None:
        cmd += ["--seq", str(seq)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"timed out after {timeout} s"}
    for ln in reversed(r.stdout.strip().splitlines()):
        if ln.startswith("{"):
            return json.loads(ln)
    return {"unavailable": f"exit {r.returncode}: {(r.stderr or r.stdout).strip().splitlines()[-1:]}"}


# --------------------------------------------------------------------------- GPU arm
def main():
    args = parse()
    cfg = synth.CONFIGS[args.config]
    if args.batch is not None:
        import dataclasses
        cfg = dataclasses.replace(cfg, B=args.batch)
    if args.seq is not None:
        import dataclasses
        cfg = dataclasses.replace(cfg, T=args.seq)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, rank)
        return
    if args.impl == "reference_cuda":
        sys.path.remove(os.path.join(REPO, "ltc-cuda_b200"))  # the reference binds its own ltc_cuda
        run_reference_cuda(args, cfg, rank)
        return

    import ltc_cuda
    ltc_cuda.set_lean_save(bool(args.lean))
    import ltc_layer
    from data_parallel import FlatGradBucket, shard_range, training_step

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # The gradient bucket is small (199 KB at c3): NCCL's NVLink-SHARP (NVLS)
        # all-reduce, replayed inside the step's CUDA graph, cost about 0.5 ms per step
        # at 8 ranks on B200 (3.36 ms/step vs 2.87 ms with it off); the default NVLink
        # algorithms are used unless the caller set NCCL_NVLS_ENABLE.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", device_id=dev)
    peaks, peaks_kind = measured_peaks()

    p, x_full = synth.make_workload(cfg)
    lo, hi = shard_range(cfg.B, rank, world)
    Bl = hi - lo
    model = ltc_layer.TrueLiquidTimeConstant(cfg.D, cfg.H, dt=cfg.dt, ode_unfolds=cfg.U,
                                             sparsity=cfg.density, sensory_sparsity=cfg.sensory_density)
    model.load_state_dict(p)
    model.skip_zero_synapses = model.skip_zero_synapses and bool(args.skip_zero)
    model = model.to(dev)
    bucket = FlatGradBucket(model.parameters())
    use_graph = bool(args.graph) if args.graph is not None else True
    opt = torch.optim.Adam(model.parameters(), lr=1e-4, fused=True, capturable=use_graph)
    x_host = x_full[lo:hi].contiguous().pin_memory()
    x_dev = x_host.to(dev)
    del x_full
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > 126 MB L2

    def step(x):
        if cfg.training_step:
            return training_step(model, x, bucket, opt)
        bucket.zero()
        out, _ = model(x)
        loss = out.sum()
        loss.backward()
        bucket.all_reduce()
        return loss.detach()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    parity = None
    if rank == 0 and args.parity:
        import ltc_layer
        # the slice takes the timed step's path: skipping where the step's rows reach the threshold
        parity = our_parity(cfg, p, dev, bool(args.skip_zero) and Bl * cfg.T >= ltc_layer.SKIP_MIN_ROWS)
    for _ in range(max(3, args.warmup)):
        step(x_dev)
    torch.cuda.synchronize()

    # CUDA-graph mode: the whole step (module forward, backward, all-reduce, Adam) is
    # captured once per input buffer and replayed; the same kernels run, without the
    # host launch overhead that dominates the small configurations.
    graphs = {}
    launches_per_step = None

    def capture(xbuf):
        nonlocal launches_per_step
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                step(xbuf)
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        n_before = ltc_cuda.launch_count()
        with torch.cuda.graph(g):
            out = step(xbuf)
        launches_per_step = ltc_cuda.launch_count() - n_before
        graphs[xbuf.data_ptr()] = (g, out)

    def run(xbuf):
        if not use_graph:
            return step(xbuf)
        g, out = graphs[xbuf.data_ptr()]
        g.replay()
        return out

    graph_note = None
    if use_graph:
        try:
            capture(x_dev)
            for _ in range(3):
                run(x_dev)
            torch.cuda.synchronize()
        except Exception as exc:  # capture unsupported here: measure eagerly and say so
            graphs.clear()
            use_graph = False
            graph_note = f"graph capture failed, eager launches: {type(exc).__name__}: {exc}"[:200]

    # ---- device-resident timed region ----
    clocks = ClockSampler(physical_gpu_index(local))
    clocks.start()
    ltc_cuda.timing_enable(not use_graph)
    n0 = ltc_cuda.launch_count()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        flush.zero_()
        run(x_dev)
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    launches = (launches_per_step * args.steps) if use_graph else (ltc_cuda.launch_count() - n0)
    if use_graph:
        # per-kernel event times need host-side launches: one eager window of the same step
        ltc_cuda.timing_enable(True)
        for _ in range(args.steps):
            flush.zero_()
            step(x_dev)
        torch.cuda.synchronize()
    ktimes = ltc_cuda.timing_collect()
    ltc_cuda.timing_enable(False)
    clk = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    value = cfg.B * cfg.T / (ms / 1e3)

    # ---- end to end through the public API: pinned host input -> device, loss -> host ----
    barrier()
    torch.cuda.synchronize()
    # the next step's input is uploaded on a copy stream while the current step runs
    # (double-buffered, as a data loader would); the first upload is inside the region
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    copy_stream = torch.cuda.Stream(dev)
    bufs = [torch.empty_like(x_dev), torch.empty_like(x_dev)]
    if use_graph:
        for bf in bufs:
            bf.copy_(x_dev)
            capture(bf)
        torch.cuda.synchronize()
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    free = [torch.cuda.Event(), torch.cuda.Event()]
    compute = torch.cuda.current_stream(dev)

    def upload(k):
        copy_stream.wait_event(free[k % 2])
        with torch.cuda.stream(copy_stream):
            bufs[k % 2].copy_(x_host, non_blocking=True)
            ready[k % 2].record(copy_stream)

    for ev in free:
        ev.record(compute)
    e0.record()
    copy_stream.wait_event(e0)
    upload(0)
    for k in range(args.steps):
        if k + 1 < args.steps:
            upload(k + 1)
        flush.zero_()
        compute.wait_event(ready[k % 2])
        loss = run(bufs[k % 2])
        free[k % 2].record(compute)
        float(loss.item())
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    e2e = {"value": cfg.B * cfg.T / (ms_e2e / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": x_host.numel() * x_host.element_size() * world,
           "d2h_bytes_per_step": 4 * world, "ms_per_step": ms_e2e}

    # ---- roofline of the dominant kernel (MUFU pipe: 2 MUFU ops per synapse visit) ----
    f_mhz = float(peaks.get("sm_max_mhz", 1965.0))
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    # recurrent synapses the kernels visit: the nonzero ones when the module lets the
    # solver skip masked synapses (H <= 64 or 128 < H <= 512), else all H*H
    rec_syn = rec_synapses(model, cfg, Bl * cfg.T)
    sens_syn = sens_synapses(model, cfg, Bl * cfg.T)
    visits = {"recurrent_fwd": Bl * cfg.T * cfg.U * rec_syn,
              "recurrent_bwd": Bl * cfg.T * cfg.U * rec_syn,
              "sensory_fwd": Bl * cfg.T * sens_syn[0],
              "sensory_bwd": Bl * cfg.T * sens_syn[1]}
    # Work per step of each kernel kind.  Memory-lean training runs the forward
    # kernels twice per step (the forward, then the recompute inside the backward,
    # once per segment), so their work per step doubles; every figure below is
    # work over the window's steps / the kind's total time in the window, so it
    # does not depend on how many launches a pass is split into.
    twice = 2 if args.lean else 1
    work = {k: v * (twice if k.endswith("_fwd") else 1) for k, v in visits.items()}
    dom = max(visits, key=lambda k: ktimes[k][0])
    tot_ms, n_l = ktimes[dom]
    per_launch_s = tot_ms / max(1, n_l) / 1e3
    achieved = work[dom] * args.steps / (tot_ms / 1e3) / 1e9
    ms_per_launch = per_launch_s * 1e3
    peak = sms * 16 / 2 * f_mhz * 1e6 / 1e9  # Gvisits/s: 16 MUFU/clk/SM, 2 MUFU per visit
    # the kernels' own bound: tanh-form gates issue 1 MUFU op per visit; the
    # forward kernels then need 3 FP32 lane-ops per visit (MUFU-bound, 16
    # visits/clk/SM), the backward ones 10 (FP32-pipe-bound, 128/10 per clk/SM)
    own_rate = {"recurrent_fwd": 16.0, "sensory_fwd": 16.0, "recurrent_bwd": 12.8, "sensory_bwd": 12.8}
    peak_own = sms * own_rate[dom] * f_mhz * 1e6 / 1e9
    kernels = {k: {"ms_total": round(v[0], 3), "launches": v[1], "share": round(v[0] / max(1e-9, sum(
        t for t, _ in ktimes.values())), 4)} for k, v in ktimes.items()}
    # whole-step ceiling with the survey's counting convention (4 MUFU per fwd+bwd synapse visit)
    S = sens_syn[0] + cfg.U * rec_syn  # nonzero synapses when they are skipped
    t_roof = cfg.B * cfg.T * S * 4 / (16 * sms * f_mhz * 1e6 * world)
    # recurrent kernels alone, same convention (the H=128 north-star figure)
    per_step = lambda k: ktimes[k][0] / args.steps / 1e3  # seconds of kernel kind k per step
    t_roof_rec = Bl * cfg.T * cfg.U * rec_syn * 4 / (16 * sms * f_mhz * 1e6)
    rec_frac = t_roof_rec / (per_step("recurrent_fwd") + per_step("recurrent_bwd"))
    # sensory forward: reads x (4 D B per (b,t)), writes sn/sd (8 H B); MUFU-bound, not HBM-bound
    sens_gbs = twice * Bl * cfg.T * (4 * cfg.D + 8 * cfg.H) / per_step("sensory_fwd") / 1e9

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; distributions of the config)",
        "config": {"workload": cfg.name, "B": cfg.B, "T": cfg.T, "D": cfg.D, "H": cfg.H, "U": cfg.U,
                   "density": cfg.density, "sensory_density": cfg.sensory_density,
                   "step": "train (fwd+bwd+allreduce+adam)" if cfg.training_step else "fwd+bwd",
                   "parallelism": f"dp{world}", "per_rank_batch": Bl,
                   "l2": "256 MB flush write between steps (inside the timed region)",
                   "cuda_graph": use_graph if graph_note is None else graph_note,
                   "saved_state": "step boundaries, unfolds recomputed (lean)" if args.lean else "every unfold",
                   "recurrent_synapses_visited": rec_syn, "recurrent_synapses_dense": cfg.H * cfg.H,
                   "sensory_synapses_visited": list(sens_syn), "sensory_synapses_dense": cfg.D * cfg.H},
        "e2e": e2e,
        "roofline": {"bound": "mufu", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "Gsynapse-visits/s",
                     "frac": achieved / peak, "ms_per_launch": ms_per_launch,
                     "traffic": (NCU_TRAFFIC_PER_BT[(cfg.name, dom)] * Bl * cfg.T
                                 if (cfg.name, dom) in NCU_TRAFFIC_PER_BT else None),
                     "traffic_unit": "bytes per launch (ncu capture, scaled)",
                     "peak_basis": f"{sms} SMs x 16 MUFU/clk / 2 MUFU per visit at sm_max {f_mhz:.0f} MHz ({peaks_kind})",
                     "step_frac_survey_convention": t_roof / (ms / 1e3),
                     "frac_own_bound": achieved / peak_own,
                     "own_bound_basis": ("1 MUFU + 10 FP32 lane-ops per visit (FP32-bound, 12.8 visits/clk/SM)"
                                         if own_rate[dom] < 16 else "1 MUFU per visit (16 visits/clk/SM)"),
                     "recurrent_frac_survey_convention": rec_frac,
                     "sensory_fwd_hbm_gbs": sens_gbs,
                     "sensory_fwd_hbm_frac": sens_gbs / float(peaks.get("hbm_gbs", 6650.0))},
        "kernels": kernels,
        "kernels_source": "eager window of the same step (graph replay has no host launches)" if use_graph
                          else "timed region",
        "gpu_launches": launches,
        "clocks": clk,
    }
    line["parity"] = parity
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sample_rate(cfg, args.cpu_seconds, os.cpu_count() or 1)
    if rank == 0 and world == 1 and args.reference_cuda:
        line["reference_cuda"] = reference_cuda_subprocess(cfg.name, args.batch, args.seq)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        # Every rank has finished its device work (max-over-ranks reductions above);
        # captured graphs hold NCCL work, and tearing the communicator down under them
        # can block, so the ranks leave without a teardown once the line is out.
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)


if __name__ == "__main__":
    main()
