"""Benchmark of the selective-scan hot path (BASELINE config 4 at seqlen 4096).

One step = selective-scan forward + backward (all 8 gradients) over one batch of
batch 32, d_inner 3072, d_state 16, seqlen 4096, bf16 I/O, fp32
state, z gate, D, delta_bias, softplus.  Inputs are seeded synthetic tensors with the
config's distributions (no dataset is involved).  Every tensor is ~0.8 GB, far larger
than the 126 MB L2, so no L2 flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun each rank runs its own batch (weak scaling; the scan has no
cross-batch exchange, so there is no data-path collective) and the reported time is
the max over ranks.  ``--impl reference`` times the reference's CPU path (the oracle
restatement of ``selective_scan_ref`` + autograd, on the host cores) on a bounded
sample of the same workload and prints the same metric.

Algorithmic bytes follow the reference's I/O contract (E = b*d*l, S = b*n*l, s = 2,
C = ceil(l/2048) chunk states as in the reference's x):
  fwd = 5*E*s + 2*S*s + b*d*C*2n*4 + d*(n+2)*4
  bwd = 8*E*s + 2*S*s + 2*S*4 + b*d*C*2n*4 + 2*d*(n+2)*4
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "motif-mamba_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

CFG = dict(batch=32, dim=3072, seqlen=4096, dstate=16)
METRIC = "selective-scan HBM GB/s (fwd+bwd)"
FALLBACK_HBM = 6650.0


def algo_bytes(batch, dim, seqlen, dstate, s=2):
    E, S = batch * dim * seqlen, batch * dstate * seqlen
    C = math.ceil(seqlen / 2048)
    fwd = 5 * E * s + 2 * S * s + batch * dim * C * 2 * dstate * 4 + dim * (dstate + 2) * 4
    bwd = 8 * E * s + 2 * S * s + 2 * S * 4 + batch * dim * C * 2 * dstate * 4 + 2 * dim * (dstate + 2) * 4
    return fwd, bwd


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


def ncu_inst(kernel):
    """Warp-instructions per launch of `kernel` for this workload, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    try:
        for line in open(p):
            parts = line.split()
            if len(parts) >= 3 and parts[0] == kernel + ".inst" and parts[1] == "config4_l4096":
                return int(float(parts[2]))
    except OSError:
        pass
    return None


def ncu_traffic(kernel):
    """DRAM bytes per launch of `kernel` for this workload, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    try:
        for line in open(p):
            parts = line.split()
            if len(parts) >= 3 and parts[0] == kernel and parts[1] == "config4_l4096":
                return int(float(parts[2]))
    except OSError:
        pass
    return None


def make_inputs(device, seed):
    b, d, l, n = CFG["batch"], CFG["dim"], CFG["seqlen"], CFG["dstate"]
    g = torch.Generator(device=device).manual_seed(seed)
    bf = torch.bfloat16
    t = dict(
        u=torch.randn(b, d, l, device=device, generator=g).to(bf),
        delta=torch.randn(b, d, l, device=device, generator=g).to(bf),
        z=torch.randn(b, d, l, device=device, generator=g).to(bf),
        B=torch.randn(b, 1, n, l, device=device, generator=g).to(bf),
        C=torch.randn(b, 1, n, l, device=device, generator=g).to(bf),
        A=-torch.arange(1, n + 1, device=device, dtype=torch.float32).repeat(d, 1),
        D=1 + 0.1 * torch.randn(d, device=device, generator=g),
        delta_bias=torch.log(torch.expm1(torch.rand(d, device=device, generator=g) * 0.099 + 1e-3)),
    )
    dout = torch.randn(b, d, l, device=device, generator=g).to(bf)
    return t, dout


class ClockSampler:
    """nvidia-smi clock / throttle sampling around the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return None
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("swp", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        loaded = [r for r in rows if r["power"] > 300] or rows
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(loaded)}


CPU_SAMPLE_DIM = 64  # channels of the fixed CPU sample: batch 1 x 64 x seqlen, seed 0


def cpu_threads():
    """Host threads this process may run on (its CPU affinity, not the machine's core count:
    oversubscribing the affinity set slows the oracle's per-step loop several-fold)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def _cpu_scan_seconds(dim_s):
    """Seconds for the oracle restatement of selective_scan_ref (fwd + autograd bwd) on
    batch 1 x dim_s channels x the workload's seqlen (bf16 inputs, fp32 math), seed 0."""
    from oracle import ssm_oracle as O
    l, n = CFG["seqlen"], CFG["dstate"]
    g = torch.Generator().manual_seed(0)
    inp = dict(u=torch.randn(1, dim_s, l, generator=g).bfloat16(),
               delta=torch.randn(1, dim_s, l, generator=g).bfloat16(),
               A=-torch.arange(1, n + 1, dtype=torch.float32).repeat(dim_s, 1),
               B=torch.randn(1, n, l, generator=g).bfloat16(), C=torch.randn(1, n, l, generator=g).bfloat16(),
               D=torch.ones(dim_s), z=torch.randn(1, dim_s, l, generator=g).bfloat16(),
               delta_bias=torch.full((dim_s,), -4.0))
    dout = torch.randn(1, dim_s, l, generator=g).bfloat16()
    t0 = time.perf_counter()
    O.scan_with_grads(inp, dout, True)
    return time.perf_counter() - t0


def _cpu_record(dim_s, dt, threads, n_samples):
    l, n = CFG["seqlen"], CFG["dstate"]
    f, b = algo_bytes(1, dim_s, l, n)
    return dict(value=(f + b) / dt / 1e9, unit="GB/s", cores=threads, kind="port",
                m_elements_per_s=dim_s * l / dt / 1e6,
                sample=f"selective_scan_ref fwd + autograd bwd (oracle restatement), fixed sample batch 1 x {dim_s} "
                       f"channels x seqlen {l}, n {n}, seed 0, bf16 inputs, fp32 math, {threads} threads: fastest "
                       f"{dt:.2f} s of {n_samples} timed samples after 1 warm-up (host cores are shared with other "
                       f"jobs; the fastest sample is the least disturbed) ({dim_s * l / dt / 1e6:.4f} M "
                       f"elements/s); GB/s = the sample's algorithmic bytes (the metric's formula at batch 1 x "
                       f"{dim_s} channels) / its time, i.e. the same per-element rate applied to the full workload")


def cpu_baseline_sample(n_timed=3):
    """The repo arm's cpu_baseline: the same fixed sample and thread count as the reference arm."""
    threads = cpu_threads()
    torch.set_num_threads(threads)
    _cpu_scan_seconds(CPU_SAMPLE_DIM)  # warm-up (first-call costs)
    ts = [_cpu_scan_seconds(CPU_SAMPLE_DIM) for _ in range(n_timed)]
    dt = min(ts)
    return _cpu_record(CPU_SAMPLE_DIM, dt, threads, n_timed), dt


def run_reference(args, budget_s=200.0):
    """The reference arm: the oracle port of the reference's CPU path on all host threads of this
    process, one fixed sample per step.  One warm-up sample, then up to --steps timed samples;
    sampling stops early once ~budget_s seconds have been spent so the run stays within a few
    minutes at any --steps (the line says how many samples were timed)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = cpu_threads()
    torch.set_num_threads(threads)
    t_start = time.perf_counter()
    _cpu_scan_seconds(CPU_SAMPLE_DIM)
    times = []
    for i in range(args.steps):
        times.append(_cpu_scan_seconds(CPU_SAMPLE_DIM))
        if time.perf_counter() - t_start > budget_s:
            break
    dt = min(times)
    cb = _cpu_record(CPU_SAMPLE_DIM, dt, threads, len(times))
    v = cb["value"]
    fwd_b, bwd_b = algo_bytes(**CFG)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "samples_timed": len(times),
            "ms_per_step": (fwd_b + bwd_b) / (v * 1e9) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": {"workload": "selective scan fwd+bwd, BASELINE config 4 at seqlen 4096 "
                                                        "(32 x 3072 x 4096, n 16, bf16 I/O)",
                                            "batch": CFG["batch"], "d_inner": CFG["dim"],
                                            "seqlen": CFG["seqlen"], "d_state": CFG["dstate"]},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="scan workload: skip the config-2 prefill sub-record")
    ap.add_argument("--no-sweep", action="store_true",
                    help="scan workload: skip the config-4 sub-records at seqlen 1024 and 16384")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the per-GPU batch (profiling a smaller case of the same kernels)")
    ap.add_argument("--seqlen", type=int, default=None, help="override the sequence length")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="prefill workload: override the global batch (e.g. 2 = one GPU's share at 8 GPUs)")
    ap.add_argument("--no-decode", action="store_true", help="prefill workload: skip the decode measurement")
    ap.add_argument("--breakdown", action="store_true",
                    help="prefill / tp workloads: add the per-kernel device time of one eager prefill (torch profiler)")
    ap.add_argument("--tp-chunks", type=int, default=1,
                    help="tp workload: sequence chunks whose out_proj all-reduces overlap the next chunk's compute")
    ap.add_argument("--once", action="store_true", help="kernels workload: run each kernel twice (ncu capture)")
    ap.add_argument("--quick", action="store_true", help="refkernel workload: config 4 at seqlen 1024 only")
    ap.add_argument("--workload", default="scan", choices=["scan", "prefill", "tp", "pq", "kernels", "refkernel"],
                    help="scan: selective scan fwd+bwd, config 4 (default); prefill: 24-layer config-2 stack, "
                         "prefill tok/s (global batch 16 x 4096, strong scaling) plus greedy decode tok/s; "
                         "tp: 64-layer config-3 stack, prefill 1 x 32768 with d_inner sharded over the GPUs; "
                         "pq: the motif P/Q-coupled scan fwd+bwd at a config-1 block's shape; "
                         "kernels: conv1d / add+RMSNorm / decode kernels' GB/s; "
                         "refkernel: our scan kernels timed beside the reference's CUDA extension")
    args = ap.parse_args()
    if args.batch:
        CFG["batch"] = args.batch
    if args.global_batch:
        PREFILL["global_batch"] = args.global_batch
    if args.seqlen:
        CFG["seqlen"] = args.seqlen
    args.warmup = max(args.warmup, 3)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "tp":
        return run_tp(args)
    if args.workload == "pq":
        return run_pq(args)
    if args.workload == "kernels":
        return run_kernels(args)
    if args.workload == "refkernel":
        return run_refkernel(args)
    if args.impl == "reference":
        return run_reference(args)

    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    from motif_ssm import selective_scan_cuda as ssc, selective_scan_fn

    t, dout = make_inputs(dev, seed=1234 + rank)
    fwd_b, bwd_b = algo_bytes(**CFG)
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        out, x, out_z = ssc.fwd(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"],
                                delta_bias=t["delta_bias"], delta_softplus=True)
        if ev is not None:
            ev[1].record(stream)
        grads = ssc.bwd(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"], delta_bias=t["delta_bias"],
                        dout=dout, x=x, out=out, dz=None, delta_softplus=True, recompute_out_z=False)
        if ev is not None:
            ev[2].record(stream)
        return out_z, grads

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            step(evs[i])
        end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = start.elapsed_time(end)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    tt = torch.tensor([total_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms_per_step = tt.item() / args.steps
    value = (fwd_b + bwd_b) * world / (ms_per_step * 1e-3) / 1e9
    launches_per_step = (2 if ssc_needs_split() else 1) + 3  # fwd (+carry) ; bwd main + 2 dB/dC converts

    # ---- end to end through the public API: host (pinned) inputs in, gradients out ----
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(t, dout, dev, stream, world, selective_scan_fn, fwd_b + bwd_b, max(3, args.steps // 4),
                      dist if world > 1 else None)

    # ---- config 4 at the sweep's other sequence lengths (same kernels, same timing) ----
    sweep = None
    if not args.no_sweep:
        sweep = scan_sweep(dev, rank, world, stream, dist if world > 1 else None)

    # ---- config-2 prefill (strong scaling over the ranks) and, at world > 1, the TP parity check ----
    prefill = None
    if not args.no_prefill:
        del t, dout
        torch.cuda.empty_cache()
        pre_args = argparse.Namespace(steps=max(3, min(args.steps, 10)), warmup=args.warmup)
        prefill, pre_clocks = measure_prefill(pre_args, world, rank, local, dev, with_decode=False, with_e2e=False)
        prefill["clocks"] = pre_clocks
    tpc = tp_check(world, rank, dev) if world > 1 else None

    peak, peak_kind = hbm_peak()
    dom_ms, dom_bytes, dom_name = (bwd_ms, bwd_b, "ss_bwd") if bwd_ms >= fwd_ms else (fwd_ms, fwd_b, "ss_fwd")
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    traffic = ncu_traffic(dom_name)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu, _ = cpu_baseline_sample()
    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "selective scan fwd+bwd, BASELINE config 4 at seqlen 4096 "
                                   "(32 x 3072 x 4096 per GPU, n 16, bf16 I/O, fp32 state, z, D, delta_bias, softplus)",
                       "batch_per_gpu": CFG["batch"], "d_inner": CFG["dim"], "seqlen": CFG["seqlen"],
                       "d_state": CFG["dstate"], "l2": "inputs larger than L2 (0.8 GB per tensor), no flush",
                       "algorithmic_bytes_per_step": fwd_b + bwd_b},
            "kernels": {"ss_fwd": {"ms": fwd_ms, "GB/s": fwd_b / (fwd_ms * 1e-3) / 1e9,
                                   "frac_of_hbm": fwd_b / (fwd_ms * 1e-3) / 1e9 / peak},
                        "ss_bwd": {"ms": bwd_ms, "GB/s": bwd_b / (bwd_ms * 1e-3) / 1e9,
                                   "frac_of_hbm": bwd_b / (bwd_ms * 1e-3) / 1e9 / peak}},
            "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6650 GB/s", "traffic": traffic,
                         "issue": issue_ceiling(dom_name, dom_ms, clocks)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "seqlen_sweep": sweep,
            "prefill": prefill,
            "tp_check": tpc,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def tp_check(world, rank, dev, seqlen=1024, n_layer=2, n_chunks=2):
    """Parity of the channel-sharded TP path at this world size: a config-3-shaped stack
    (d_model 2560, d_inner 5120, n 16, dt_rank 160; 2 layers, vocab 512), bf16 random init
    with the same seed on every rank, 1 x 1024 random ids.  Rank 0 runs the unsharded model
    first; then every rank shards it and runs tp_prefill (the sequence in 2 chunks, x_proj
    partial sums all-reduced in fp32, out_proj partial sums in bf16 over NCCL, asynchronously).
    The logits of all tokens are compared on rank 0 with the bound used for sums throughout
    the tests, |a - e| <= 2e-2 max(1, max|e|) + 2e-2 |e| (logits are 2560-term dot products);
    the count of elements outside the plain elementwise bound 2e-2 + 2e-2 |e| is reported too."""
    import torch.distributed as dist
    from motif_ssm.modules import MambaConfig, MambaLMHeadModel, shard_model_tp, tp_prefill
    torch.manual_seed(0)
    model = MambaLMHeadModel(MambaConfig(d_model=2560, n_layer=n_layer, vocab_size=512, ssm_cfg={"d_state": 16}),
                             device=dev, dtype=torch.bfloat16)
    model.eval()
    ids = torch.randint(0, 512, (1, seqlen), device=dev, generator=torch.Generator(device=dev).manual_seed(7))
    ref = None
    with torch.no_grad():
        if rank == 0:
            ref = model(ids).float()
        shard_model_tp(model, rank, world)
        out = tp_prefill(model, ids, n_chunks=n_chunks, num_last_tokens=0).float()
    torch.cuda.synchronize()
    res = None
    if rank == 0:
        err = (out - ref).abs()
        scale = max(1.0, ref.abs().max().item())
        res = {"world": world, "layers": n_layer, "tokens": seqlen, "chunks": n_chunks,
               "max_abs_err": err.max().item(), "max_ref": ref.abs().max().item(),
               "plain_bound_violations": int((err > 2e-2 + 2e-2 * ref.abs()).sum().item()),
               "pass": bool((err <= 2e-2 * scale + 2e-2 * ref.abs()).all().item())}
    del model
    torch.cuda.empty_cache()
    dist.barrier()
    return res


def scan_sweep(dev, rank, world, stream, dist, seqlens=(1024, 16384), steps=5, warmup=3):
    """BASELINE config 4 at its other sequence lengths: batch 32 x 3072 channels per GPU, bf16,
    fwd + bwd per step as in the headline, CUDA events on the launching stream, max over ranks.
    Inputs are larger than L2 at every length (0.2 GB per tensor at 1024), so no flush."""
    from motif_ssm import selective_scan_cuda as ssc
    saved, res = CFG["seqlen"], {}
    try:
        for L in seqlens:
            CFG["seqlen"] = L
            t, dout = make_inputs(dev, seed=4321 + rank)
            fb, bb = algo_bytes(**CFG)
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]

            def step(ev=None):
                if ev is not None:
                    ev[0].record(stream)
                out, x, _ = ssc.fwd(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"],
                                    delta_bias=t["delta_bias"], delta_softplus=True)
                if ev is not None:
                    ev[1].record(stream)
                ssc.bwd(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"], delta_bias=t["delta_bias"],
                        dout=dout, x=x, out=out, dz=None, delta_softplus=True, recompute_out_z=False)
                if ev is not None:
                    ev[2].record(stream)

            for _ in range(warmup):
                step()
            torch.cuda.synchronize()
            if dist is not None:
                dist.barrier()
            for i in range(steps):
                step(evs[i])
            torch.cuda.synchronize()
            tt = torch.tensor([sum(e[0].elapsed_time(e[2]) for e in evs) / steps], device=dev, dtype=torch.float64)
            if dist is not None:
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
            bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
            peak = hbm_peak()[0]
            res[str(L)] = {"shape": f"{CFG['batch']} x {CFG['dim']} x {L} per GPU", "steps": steps, "warmup": warmup,
                           "ms_per_step": tt.item(), "GB/s": (fb + bb) * world / (tt.item() * 1e-3) / 1e9,
                           "ss_fwd": {"ms": fwd_ms, "frac_of_hbm": fb / (fwd_ms * 1e-3) / 1e9 / peak},
                           "ss_bwd": {"ms": bwd_ms, "frac_of_hbm": bb / (bwd_ms * 1e-3) / 1e9 / peak}}
            del t, dout
            torch.cuda.empty_cache()
    finally:
        CFG["seqlen"] = saved
    return res


def ssc_needs_split():
    import ctypes
    from motif_ssm import _lib
    a = _lib.SsFwdArgs()
    a.batch, a.dim, a.seqlen, a.dstate, a.n_groups, a.itype = (CFG["batch"], CFG["dim"], CFG["seqlen"],
                                                               CFG["dstate"], 1, _lib.MSS_BF16)
    nb = ctypes.c_int64(0)
    _lib.check(_lib.lib.ss_fwd_workspace_size(ctypes.byref(a), ctypes.byref(nb)))
    return nb.value > 0


def issue_ceiling(kernel, ms, clocks):
    """The ceiling that binds these kernels: warp-instruction issue.  Instructions per launch
    come from the committed ncu capture (scaled with seqlen like the traffic); the peak is
    4 warp-instructions per SM per clock (one per scheduler) x 148 SMs at the SM clock
    sampled under load during the timed region."""
    inst = ncu_inst(kernel)
    if inst is None:
        return None
    mhz = (clocks or {}).get("sm_mhz") or 1965.0
    achieved = inst / (ms * 1e-3) / 1e9
    peak = 4 * 148 * mhz * 1e6 / 1e9
    return {"warp_inst_per_launch": inst, "achieved": achieved, "peak": peak, "unit": "G warp-inst/s",
            "frac": achieved / peak}


def host_link_probe(dev, stream, dist, nbytes=1 << 30, reps=3):
    """Pinned host <-> device copy bandwidth of this rank, measured with all ranks copying at
    the same time (as in the e2e step): one 1 GiB buffer each way, host-to-device alone,
    device-to-host alone, then both at once on two streams; best of `reps`.  Also records the
    CPU affinity of this process and the GPU's NUMA node, which decide whose memory controller
    and PCIe root the pinned buffers cross.  Returns a dict (GB/s)."""
    hbuf = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    hbuf2 = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dbuf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dbuf2 = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    s2 = torch.cuda.Stream(dev)

    def timed(fn):
        best = float("inf")
        for _ in range(reps):
            if dist is not None:
                dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            best = min(best, a.elapsed_time(b))
        return nbytes / (best * 1e-3) / 1e9

    def both():
        s2.wait_stream(stream)
        dbuf.copy_(hbuf, non_blocking=True)
        with torch.cuda.stream(s2):
            hbuf2.copy_(dbuf2, non_blocking=True)
        stream.wait_stream(s2)

    rec = {"h2d_gbs": timed(lambda: dbuf.copy_(hbuf, non_blocking=True)),
           "d2h_gbs": timed(lambda: hbuf2.copy_(dbuf2, non_blocking=True)),
           "both_each_way_gbs": timed(both)}
    try:
        rec["cpu_affinity"] = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        pass
    try:  # NUMA node of this GPU's PCI device (sysfs, via the bus id NVML reports)
        import pynvml  # nvidia_ml_py
        pynvml.nvmlInit()
        bus = pynvml.nvmlDeviceGetPciInfo(pynvml.nvmlDeviceGetHandleByIndex(dev.index)).busId
        bus = (bus.decode() if isinstance(bus, bytes) else bus)[-12:].lower()
        rec["gpu_pci"] = bus
        rec["gpu_numa_node"] = int(open(f"/sys/bus/pci/devices/{bus}/numa_node").read().strip())
    except Exception:
        pass
    del hbuf, hbuf2, dbuf, dbuf2
    return rec


def run_e2e(t, dout, dev, stream, world, selective_scan_fn, algo, steps, dist, n_sub=16):
    """selective_scan_fn (autograd) per step with host buffers: pinned host inputs ->
    device, forward, backward, all 8 gradients -> pinned host, timed with CUDA events
    around the whole step, max over ranks.

    The batch is processed as ``n_sub`` sub-batches through the same public call (the scan
    is independent across batch rows), pipelined over three streams: the host-to-device
    copy of sub-batch i+1 and the device-to-host copy of sub-batch i-1's gradients overlap
    sub-batch i's forward + backward.  dA, dD and ddelta_bias (sums over the batch) are
    accumulated on the device across the sub-batches and copied once per step."""
    keys = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
    per_row = ("u", "delta", "B", "C", "z")
    shared = ("A", "D", "delta_bias")
    host = {k: t[k].cpu().pin_memory() for k in keys}
    host_dout = dout.cpu().pin_memory()
    dev_bufs = {k: torch.empty_like(t[k]) for k in keys}
    dev_dout = torch.empty_like(dout)
    host_grads = {k: torch.empty(t[k].shape, dtype=t[k].dtype).pin_memory() for k in keys}
    dev_shared_grads = {k: torch.empty_like(t[k]) for k in shared}
    h2d = sum(v.numel() * v.element_size() for v in host.values()) + host_dout.numel() * host_dout.element_size()
    d2h = sum(v.numel() * v.element_size() for v in host_grads.values())
    batch = t["u"].shape[0]
    n_sub = max(1, min(n_sub, batch))
    bounds = [(i * batch // n_sub, (i + 1) * batch // n_sub) for i in range(n_sub)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    done = [torch.cuda.Event() for _ in range(n_sub)]  # compute of sub-batch i finished (inputs free)
    for e in done:
        e.record(stream)

    def one():
        with torch.cuda.stream(s_in):
            s_in.wait_event(done[-1])  # the previous step's last sub-batch no longer reads A, D, bias
            for k in shared:
                dev_bufs[k].copy_(host[k], non_blocking=True)
        for i, (b0, b1) in enumerate(bounds):
            ready = torch.cuda.Event()
            with torch.cuda.stream(s_in):
                s_in.wait_event(done[i])  # the previous step's compute of this slice is over
                for k in per_row:
                    dev_bufs[k][b0:b1].copy_(host[k][b0:b1], non_blocking=True)
                dev_dout[b0:b1].copy_(host_dout[b0:b1], non_blocking=True)
                ready.record(s_in)
            stream.wait_event(ready)
            leaves = {k: (dev_bufs[k][b0:b1] if k in per_row else dev_bufs[k]).detach().requires_grad_(True)
                      for k in keys}
            out = selective_scan_fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                    leaves["D"], z=leaves["z"], delta_bias=leaves["delta_bias"], delta_softplus=True)
            out.backward(dev_dout[b0:b1])
            for k in shared:
                if i == 0:
                    dev_shared_grads[k].copy_(leaves[k].grad)
                else:
                    dev_shared_grads[k].add_(leaves[k].grad)
            done[i].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done[i])
                for k in per_row:
                    g = leaves[k].grad
                    g.record_stream(s_out)
                    host_grads[k][b0:b1].copy_(g, non_blocking=True)
        with torch.cuda.stream(s_out):
            for k in shared:
                host_grads[k].copy_(dev_shared_grads[k], non_blocking=True)
        stream.wait_stream(s_out)

    for _ in range(2):
        one()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    s_in.wait_stream(stream)
    for _ in range(steps):
        one()
    e.record(stream)
    torch.cuda.synchronize()
    tt = torch.tensor([s.elapsed_time(e)], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = tt.item() / steps
    link = host_link_probe(dev, stream, dist)
    links = [link]
    if dist is not None:
        links = [None] * world
        dist.all_gather_object(links, link)
    return {"value": algo * world / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms, "steps": steps,
            "host_links_per_rank": links,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": f"motif_ssm.selective_scan_fn forward + autograd backward on {n_sub} sub-batches, pinned host "
                   "buffers, host-to-device / compute / device-to-host pipelined on three streams"}


PREFILL = dict(n_layer=24, d_model=768, vocab=512, d_state=16, global_batch=16, seqlen=4096,
               decode_batch=64, decode_steps=256, prompt=128)


def _cpu_prefill_tok_s(threads, seqlen=512):
    """The reference's CPU path for one layer of the stack (oracle restatement of the
    mixer: conv, x_proj, dt_proj, selective_scan_ref, out_proj, fp32), extrapolated
    to 24 layers: tok/s = tokens / (24 * seconds per layer)."""
    from oracle import ssm_oracle as O
    torch.set_num_threads(threads)
    d, di, n, r = PREFILL["d_model"], 2 * PREFILL["d_model"], PREFILL["d_state"], 48
    g = torch.Generator().manual_seed(0)
    xz = torch.randn(1, 2 * di, seqlen, generator=g)
    w = [0.02 * torch.randn(di, 1, 4, generator=g), 0.02 * torch.randn(di, generator=g),
         0.02 * torch.randn(r + 2 * n, di, generator=g), 0.1 * torch.randn(di, r, generator=g),
         0.02 * torch.randn(d, di, generator=g)]
    A = -torch.arange(1, n + 1, dtype=torch.float32).repeat(di, 1)
    t0 = time.perf_counter()
    with torch.no_grad():
        O.mamba_inner_ref(xz, *w, None, A, None, None, torch.ones(di), delta_bias=torch.full((di,), -4.0))
    dt = time.perf_counter() - t0
    return dict(value=seqlen / (dt * PREFILL["n_layer"]), unit="tok/s", cores=threads, kind="port",
                sample=f"one mixer layer (d_model 768, d_inner 1536) at batch 1 x {seqlen} tokens through the "
                       f"oracle restatement of mamba_inner_ref in fp32: {dt:.2f} s, extrapolated to 24 layers")


def _kernel_breakdown(fn):
    """Device time per kernel of one call of ``fn`` (run eagerly, not graphed), from the torch
    profiler's CUDA activity records: launch counts, time and share per kernel, and the share of
    NCCL kernels (whose device time includes waiting for the other ranks).  Every rank must
    call this together when ``fn`` issues collectives."""
    from torch.profiler import ProfilerActivity, profile
    with torch.no_grad():
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
    ev = [(k.key, k.device_time_total, k.count) for k in prof.key_averages() if k.device_time_total > 0]
    tot = sum(t for _, t, _ in ev)
    nccl = sum(t for k, t, _ in ev if "nccl" in k.lower())
    ev.sort(key=lambda e: -e[1])
    return {"total_ms": tot / 1e3, "nccl_ms": nccl / 1e3, "nccl_share": round(nccl / tot, 4) if tot else 0.0,
            "kernels": [{"kernel": k[:120], "launches": c, "us_per_launch": round(t / c, 2),
                         "total_ms": round(t / 1e3, 4), "share": round(t / tot, 4)} for k, t, c in ev]}


def measure_prefill(args, world, rank, local, dev, with_decode=True, with_e2e=True):
    """Config 2: 24-layer MotifMamba stack, bf16 random init, vocab 512 random ids.  Prefill of
    a fixed global batch of 16 x 4096 split over ranks (strong scaling; no collective: each rank
    runs its own rows), timed with CUDA events, max over ranks; optionally 256 greedy decode
    steps at global batch 64 through the cache and an end-to-end number (host ids in, last-token
    logits out).  Returns the record (every rank), the clock samples of the timed region."""
    import torch.distributed as dist
    from motif_ssm.modules import GraphedForward, InferenceParams, MambaConfig, MambaLMHeadModel
    P = PREFILL
    torch.manual_seed(0)
    model = MambaLMHeadModel(MambaConfig(d_model=P["d_model"], n_layer=P["n_layer"], vocab_size=P["vocab"],
                                         ssm_cfg={"d_state": P["d_state"]}), device=dev, dtype=torch.bfloat16)
    model.eval()
    bl = max(1, P["global_batch"] // world)
    g = torch.Generator(device=dev).manual_seed(rank)
    ids = torch.randint(0, P["vocab"], (bl, P["seqlen"]), device=dev, generator=g)
    stream = torch.cuda.current_stream(dev)
    graphed = GraphedForward(model, bl, P["seqlen"])  # the whole prefill as one CUDA graph

    for _ in range(args.warmup):
        graphed(ids)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        s.record(stream)
        for _ in range(args.steps):
            graphed(ids)
        e.record(stream)
        torch.cuda.synchronize()
    tt = torch.tensor([s.elapsed_time(e) / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = tt.item()
    rec = {"metric": "MotifMamba prefill tok/s (config 2)", "value": bl * world * P["seqlen"] / (ms * 1e-3),
           "unit": "tok/s", "ms_per_step": ms, "n_gpus": world, "scaling": "strong",
           "config": {"workload": "24-layer MotifMamba stack (d_model 768, d_inner 1536, n 16, RMSNorm, vocab 512), "
                                  "bf16 random init, prefill of global batch 16 x 4096 random ids, last-token logits",
                      "global_batch": bl * world, "batch_per_gpu": bl, "seqlen": P["seqlen"],
                      "parallelism": f"batch-sharded x{world}", "cuda_graph": True}}
    clocks = clk.summary()

    if with_decode:  # greedy decode through the cache
        db = max(1, P["decode_batch"] // world)
        prompt = torch.randint(0, P["vocab"], (db, P["prompt"]), device=dev, generator=g)
        with torch.no_grad():
            params = InferenceParams(max_seqlen=P["prompt"] + P["decode_steps"], max_batch_size=db)
            tok = model(prompt, inference_params=params, num_last_tokens=1).argmax(-1)
            params.seqlen_offset = P["prompt"]
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            from motif_ssm.modules import GraphedDecoder
            dec = GraphedDecoder(model, params, db)   # whole decode step as one CUDA graph
            s.record(stream)
            for _ in range(P["decode_steps"]):
                tok = dec.step(tok).argmax(-1)
            e.record(stream)
            torch.cuda.synchronize()
        td = torch.tensor([s.elapsed_time(e)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(td, op=dist.ReduceOp.MAX)
        rec["decode_tok_s"] = db * world * P["decode_steps"] / (td.item() * 1e-3)
        rec["decode"] = {"global_batch": db * world, "steps": P["decode_steps"], "prompt": P["prompt"],
                         "cuda_graph": True}

    if getattr(args, "breakdown", False) and rank == 0:
        rec["kernel_breakdown"] = _kernel_breakdown(lambda: model(ids, num_last_tokens=1))

    if with_e2e:  # end to end: host ids in, last-token logits out
        host_ids = ids.cpu().pin_memory()
        dev_ids = torch.empty_like(ids)
        out_host = torch.empty((bl, 1, model.lm_head.weight.shape[0]), dtype=torch.bfloat16).pin_memory()
        s.record(stream)
        for _ in range(args.steps):
            dev_ids.copy_(host_ids, non_blocking=True)
            lg = graphed(dev_ids)
            out_host.copy_(lg, non_blocking=True)
        e.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([s.elapsed_time(e) / args.steps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        rec["e2e"] = {"value": bl * world * P["seqlen"] / (te.item() * 1e-3), "unit": "tok/s",
                      "h2d_bytes_per_step": host_ids.numel() * 8, "d2h_bytes_per_step": out_host.numel() * 2}
    del graphed, model
    torch.cuda.empty_cache()
    return rec, clocks


def run_prefill(args):
    """--workload prefill: the config-2 prefill record as the headline line."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            cb = _cpu_prefill_tok_s(cpu_threads())
            print(json.dumps({"impl": "reference", "metric": "MotifMamba prefill tok/s (config 2)", "value": cb["value"],
                              "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
                              "data": "synthetic", "config": {"workload": "24-layer config-2 prefill"},
                              "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "tok/s",
                                                          "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    rec, clocks = measure_prefill(args, world, rank, local, dev, with_decode=not args.no_decode)
    cpu = _cpu_prefill_tok_s(cpu_threads()) if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    if rank == 0:
        line = dict(rec)
        line.update({"steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "vs_baseline": None,
                     "dtype": "bf16", "data": "synthetic", "gpu_launches": None, "clocks": clocks,
                     "cpu_baseline": cpu})
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


PQ = dict(batch=8, dim=1536, seqlen=2048, dstate=16, rank=4)


def _pq_inputs(b, d, l, n, r, device, seed, dtype=torch.bfloat16):
    g = torch.Generator(device=device).manual_seed(seed)
    rn = lambda *sh: torch.randn(*sh, device=device, generator=g)
    t = dict(u=rn(b, d, l).to(dtype), delta=rn(b, d, l).to(dtype), z=rn(b, d, l).to(dtype),
             B=rn(b, 1, n, l).to(dtype), C=rn(b, 1, n, l).to(dtype),
             A=-torch.arange(1, n + 1, device=device, dtype=torch.float32).repeat(d, 1),
             D=1 + 0.1 * rn(d), delta_bias=torch.log(torch.expm1(torch.rand(d, device=device, generator=g) * 0.099 + 1e-3)),
             P=0.1 * rn(n, r), Q=0.1 * rn(r, n))
    return t, rn(b, d, l).to(dtype)


def _cpu_pq_record(threads, budget_s):
    """The reference's CPU path for the P/Q scan (oracle restatement of selective_scan_ref with
    P / Q, fwd + autograd bwd) on batch 1 x a channel slice x the full sequence."""
    from oracle import ssm_oracle as O
    torch.set_num_threads(threads)
    l, n, r = PQ["seqlen"], PQ["dstate"], PQ["rank"]

    def run(dim_s):
        t, dout = _pq_inputs(1, dim_s, l, n, r, "cpu", 0)
        t = {k: v for k, v in t.items()}
        t["B"], t["C"] = t["B"][:, 0], t["C"][:, 0]
        t0 = time.perf_counter()
        O.scan_with_grads(t, dout, True)
        return time.perf_counter() - t0

    probe = 8
    run(probe)  # warm-up (first-call costs would skew the extrapolation)
    tp = run(probe)
    dim_s = int(max(probe, min(PQ["dim"], probe * budget_s / max(tp, 1e-3))))
    dt = run(dim_s)
    if dt < 0.5 * budget_s and dim_s < PQ["dim"]:  # per-step overheads do not scale with channels
        dim_s = int(min(PQ["dim"], dim_s * budget_s / dt))
        dt = run(dim_s)
    el = dim_s * l * n
    return dict(value=el / dt / 1e9, unit="G element-states/s", cores=threads, kind="port",
                sample=f"selective_scan_ref with P / Q (rank {r}, shared), fwd + autograd bwd, batch 1 x {dim_s} "
                       f"channels x seqlen {l}, n {n}, bf16 inputs, fp32 math: {dt:.2f} s")


def run_pq(args):
    """The motif P/Q-coupled scan, fwd + bwd (all gradients incl. dP, dQ), at a config-1 block's
    shape (batch 8, d_inner 1536, seqlen 2048, n 16, rank 4 shared, bf16, z), per GPU (weak
    scaling; no collective).  Metric: element-states (batch x d_inner x seqlen x dstate) per
    second of fwd+bwd."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric = "P/Q selective-scan fwd+bwd element-states/s"
    cfg = {"workload": "motif P/Q scan fwd+bwd, 8 x 1536 x 2048 per GPU, n 16, rank 4 shared P/Q, bf16 I/O, z, "
                       "D, delta_bias, softplus", **PQ,
           "l2": "working set per step ~0.45 GB (9 tensors of 50 MB) > 126 MB L2, no flush"}
    if args.impl == "reference":
        if rank == 0:
            cb = _cpu_pq_record(cpu_threads(), 20.0)
            print(json.dumps({"impl": "reference", "metric": metric, "value": cb["value"], "unit": cb["unit"],
                              "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                              "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                              "config": cfg, "cpu_baseline": cb,
                              "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                                      "d2h_bytes_per_step": 0}}))
        return 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from motif_ssm import selective_scan_cuda as ssc
    b, d, l, n, r = PQ["batch"], PQ["dim"], PQ["seqlen"], PQ["dstate"], PQ["rank"]
    t, dout = _pq_inputs(b, d, l, n, r, dev, 77 + rank)
    stream = torch.cuda.current_stream(dev)
    dP, dQ = torch.empty_like(t["P"]), torch.empty_like(t["Q"])

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        out, x, out_z = ssc.fwd(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"],
                                delta_bias=t["delta_bias"], P=t["P"], Q=t["Q"], delta_softplus=True)
        if ev is not None:
            ev[1].record(stream)
        ssc.bwd(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"], delta_bias=t["delta_bias"],
                P=t["P"], Q=t["Q"], dout=dout, x=x, out=out, dz=None, dP_out=dP, dQ_out=dQ, delta_softplus=True,
                recompute_out_z=False)
        if ev is not None:
            ev[2].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        s.record(stream)
        for i in range(args.steps):
            step(evs[i])
        e.record(stream)
        torch.cuda.synchronize()
    tt = torch.tensor([s.elapsed_time(e) / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = tt.item()
    fwd_ms = statistics.median(a.elapsed_time(bq) for a, bq, _ in evs)
    bwd_ms = statistics.median(bq.elapsed_time(c) for _, bq, c in evs)
    el = b * d * l * n
    cpu = _cpu_pq_record(cpu_threads(), 15.0) if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    if rank == 0:
        print(json.dumps({"metric": metric, "value": el * world / (ms * 1e-3) / 1e9, "unit": "G element-states/s",
                          "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                          "data": "synthetic", "config": cfg,
                          "kernels": {"ss_pq_fwd": {"ms": fwd_ms}, "ss_pq_bwd": {"ms": bwd_ms}},
                          "gpu_launches": 4 * args.steps, "clocks": clk.summary(), "e2e": None, "cpu_baseline": cpu}))
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_tp(args):
    """Config 3: 64-layer stack (d_model 2560, d_inner 5120, n 16, dt_rank 160), bf16 random
    init, prefill of 1 x 32768 tokens with d_inner channel-sharded over the ranks and two
    NCCL all-reduces per layer (x_dbl partial sums, out_proj partial sums)."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the tp workload has no CPU reference run; "
                              "use the default scan workload for the reference arm"}))
        return 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from motif_ssm.modules import MambaConfig, MambaLMHeadModel, shard_model_tp, tp_prefill
    L = args.seqlen or 32768
    n_layer = 64
    torch.manual_seed(0)
    model = MambaLMHeadModel(MambaConfig(d_model=2560, n_layer=n_layer, vocab_size=50277,
                                         ssm_cfg={"d_state": 16}), device=dev, dtype=torch.bfloat16)
    if world > 1:
        shard_model_tp(model, rank, world, group)
    torch.cuda.empty_cache()
    ids = torch.randint(0, 50277, (1, L), device=dev, generator=torch.Generator(device=dev).manual_seed(0))
    stream = torch.cuda.current_stream(dev)

    chunks = max(1, args.tp_chunks) if world > 1 else 1

    def run():
        if world == 1:  # one GPU: the unsharded model's own prefill path
            with torch.no_grad():
                return model(ids, num_last_tokens=1)
        return tp_prefill(model, ids, n_chunks=chunks, num_last_tokens=1)

    step = run
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        s.record(stream)
        for _ in range(args.steps):
            step()
        e.record(stream)
        torch.cuda.synchronize()
    tt = torch.tensor([s.elapsed_time(e) / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    breakdown = _kernel_breakdown(step) if args.breakdown else None  # every rank (collectives)
    if rank == 0:
        print(json.dumps({
            "kernel_breakdown": breakdown,
            "metric": "MotifMamba TP prefill tok/s (config 3)", "value": L / (tt.item() * 1e-3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": tt.item(),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "64-layer stack d_model 2560 d_inner 5120 n 16 dt_rank 160, bf16 random init, "
                                   "prefill 1 x %d, last-token logits" % L, "parallelism": f"tp{world}",
                       "seq_chunks": chunks,
                       "overlap": "with seq_chunks > 1: out_proj all-reduce of chunk i issued asynchronously "
                                  "while chunk i+1 computes"},
            "clocks": clk.summary(), "e2e": None, "cpu_baseline": None}), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def _median_ms(fn, warmup=3, iters=10, reps=10):
    """Median over ``iters`` of the mean time of ``reps`` back-to-back calls (the host's
    launch overhead overlaps the queued kernels instead of adding idle gaps)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e) / reps)
    return statistics.median(ts)


def _nbytes(*ts):
    return sum(t.numel() * t.element_size() for t in ts if t is not None)


def run_kernels(args):
    """Achieved HBM bandwidth of the kernels around the scan: causal conv1d forward / backward,
    the fused residual add + RMSNorm, and the two decode kernels (conv1d update and the SSM state
    update); one JSON line per kernel (CUDA-event medians).  ``--once`` runs each kernel twice
    instead, for an ncu launch capture.

    Shapes: the conv and the norm at BASELINE config 2's prefill (16 x 4096 tokens, d_inner 1536,
    d_model 768, bf16; every tensor > 126 MB L2 except the conv weights), the decode kernels at
    its decode step (batch 64, d_inner 1536, d_state 16), whose few MB stay in L2: those two are
    launch- and latency-bound and their GB/s says so.  Bytes are the algorithmic ones: every
    input read once, every output written once."""
    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "the kernels workload has no CPU reference run; "
                          "use the default scan workload for the reference arm"}))
        return 0
    from motif_ssm import causal_conv1d as cc
    from motif_ssm.norm import add_rms_norm
    from motif_ssm.selective_state_update import selective_state_update
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    r = lambda *s, dt=torch.bfloat16: torch.randn(*s, device=dev, generator=g).to(dt)
    b, d, l, dm = 16, 1536, 4096, 768
    x, dout = r(b, d, l), r(b, d, l)
    w, bias = r(d, 4), r(d)
    xs, res, nw = r(b * l, dm), r(b * l, dm, dt=torch.float32), r(dm)
    db, n = 64, 16
    state, conv_state = r(db, d, n), r(db, d, 4)
    xd, dtd, zd = r(db, d), r(db, d), r(db, d)
    A = -torch.arange(1, n + 1, device=dev, dtype=torch.float32).repeat(d, 1)
    Bd, Cd = r(db, n), r(db, n)
    D, dt_bias = r(d, dt=torch.float32), r(d, dt=torch.float32)
    work = [
        ("conv1d_fwd", "16 x 1536 x 4096 bf16, SiLU",
         lambda: cc.causal_conv1d_fwd_function(x, w, bias, None, None, None, True),
         2 * _nbytes(x) + _nbytes(w, bias)),
        ("conv1d_bwd", "16 x 1536 x 4096 bf16, SiLU",
         lambda: cc.causal_conv1d_bwd_function(x, w, bias, dout, None, None, None, None, False, True),
         3 * _nbytes(x) + _nbytes(w, bias) + 4 * (w.numel() + bias.numel())),
        ("add_rms_norm", "65536 x 768, bf16 x / out, fp32 residual in / out",
         lambda: add_rms_norm(xs, res, nw, 1e-5, True),
         2 * _nbytes(xs) + 2 * _nbytes(res) + _nbytes(nw)),
        ("conv1d_update", "decode, 64 x 1536, width 4, bf16",
         lambda: cc.causal_conv1d_update_function(xd, conv_state, w, bias, True, None, None),
         2 * _nbytes(xd) + 2 * _nbytes(conv_state) + _nbytes(w, bias)),
        ("ssm_state_update", "decode, 64 x 1536 x 16, bf16 state, z, D, dt_bias",
         lambda: selective_state_update(state, xd, dtd, A, Bd, Cd, D, z=zd, dt_bias=dt_bias, dt_softplus=True),
         2 * _nbytes(state) + 4 * _nbytes(xd) + _nbytes(A, Bd, Cd, D, dt_bias)),
    ]
    peak, _ = hbm_peak()
    for name, shape, fn, nbytes in work:
        if args.once:
            fn()
            fn()
            torch.cuda.synchronize()
            continue
        ms = _median_ms(fn)
        print(json.dumps({"kernel": name, "shape": shape, "ms": round(ms, 5), "bytes": nbytes,
                          "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
                          "frac_of_hbm": round(nbytes / (ms * 1e-3) / 1e9 / peak, 3)}), flush=True)
    return 0


def _time_median(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    return statistics.median(ts)


def _refk_inputs(b, d, l, n, dtype, z=True, pq_rank=0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g)
    t = dict(u=r(b, d, l).to(dtype), delta=r(b, d, l).to(dtype), z=r(b, d, l).to(dtype) if z else None,
             B=r(b, 1, n, l).to(dtype), C=r(b, 1, n, l).to(dtype),
             A=-torch.arange(1, n + 1, device="cuda", dtype=torch.float32).repeat(d, 1),
             D=1 + 0.1 * r(d), delta_bias=torch.log(torch.expm1(torch.rand(d, device="cuda", generator=g) * 0.099 + 1e-3)),
             dout=r(b, d, l).to(dtype))
    if pq_rank:
        t["P"], t["Q"] = 0.1 * r(n, pq_rank), 0.1 * r(pq_rank, n)
    return t


def _refk_bench(mod, t, pq, warmup, iters, do_bwd=True):
    kw = dict(D=t["D"], z=t["z"], delta_bias=t["delta_bias"])
    if pq:
        kw.update(P=t["P"], Q=t["Q"])
    args = (t["u"], t["delta"], t["A"], t["B"], t["C"])
    fwd = lambda: mod.fwd(*args, delta_softplus=True, **kw)
    ms_f = _time_median(fwd, warmup, iters)
    ms_b = None
    if do_bwd:
        out, x, *_ = fwd()
        dP = torch.zeros_like(t["P"]) if pq else None
        dQ = torch.zeros_like(t["Q"]) if pq else None
        bwd = lambda: mod.bwd(*args, dout=t["dout"], x=x, out=out if t["z"] is not None else None, dz=None,
                              dP_out=dP, dQ_out=dQ, delta_softplus=True, recompute_out_z=False, **kw)
        ms_b = _time_median(bwd, warmup, iters)
    return ms_f, ms_b


def run_refkernel(args):
    """This library's selective-scan kernels beside the reference's own CUDA extension (built
    from the reference's sources for sm_100a into oracle/_ref/ by oracle/build_ref_scan.py) on
    the same device inputs; one JSON line per workload with both times and the ratio.

    Workloads: BASELINE config 4 (32 x 3072 x L, n 16, bf16 I/O, z, D, delta_bias, softplus) at
    L = 1024 and 4096 (``--quick``: 1024 only), fwd and bwd separately; the module's d_state 32
    and 64 size presets at 8 x d_inner x 2048; the motif P/Q path (rank 4, shared P/Q, no z,
    since the reference's P/Q backward has none) at sizes the reference's one-thread-per-row
    kernels (forward O(L), backward O(L^2)) finish in seconds.  CUDA-event medians after
    warm-up on the current stream; config-4 inputs are > 126 MB L2."""
    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "refkernel already times the reference kernel "
                          "beside ours in one run"}))
        return 0
    from oracle import build_ref_scan
    ref = build_ref_scan.load()
    if ref is None:
        print(json.dumps({"unavailable": "reference extension not built (MOTIF_REF=... python oracle/build_ref_scan.py)"}))
        return 0
    from motif_ssm import selective_scan_cuda as ours
    work = [("config4", 32, 3072, L, 16, torch.bfloat16, True, 0, True) for L in ((1024,) if args.quick else (1024, 4096))]
    if not args.quick:
        # the module's larger size presets (d_state 32 / 64, mamba_simplemotif.py:32-36), z on
        work += [("small_n32", 8, 1024, 2048, 32, torch.bfloat16, True, 0, True),
                 ("base_n64", 8, 1536, 2048, 64, torch.bfloat16, True, 0, True)]
        work += [("pq_fwd", 8, 1536, 2048, 16, torch.bfloat16, False, 4, False),
                 ("pq_fwd_bwd", 2, 1536, 256, 16, torch.bfloat16, False, 4, True)]
    for name, b, d, l, n, dtype, z, r, do_bwd in work:
        t = _refk_inputs(b, d, l, n, dtype, z=z, pq_rank=r)
        iters = 3 if r else 10
        of, ob = _refk_bench(ours, t, r > 0, 3, iters, do_bwd)
        rf, rb = _refk_bench(ref, t, r > 0, 1 if r else 3, iters, do_bwd)
        line = {"workload": name, "batch": b, "d_inner": d, "seqlen": l, "d_state": n, "dtype": str(dtype)[6:],
                "z": z, "pq_rank": r, "ours_fwd_ms": of, "ref_fwd_ms": rf, "fwd_speedup": rf / of}
        if do_bwd:
            line.update(ours_bwd_ms=ob, ref_bwd_ms=rb, bwd_speedup=rb / ob)
        print(json.dumps(line), flush=True)
        del t
        torch.cuda.empty_cache()
    return 0


if __name__ == "__main__":
    sys.exit(main())
