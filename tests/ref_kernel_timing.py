"""Time this library's selective-scan kernels beside the reference's own CUDA extension on the
same device inputs (B200).  Test infrastructure, not a pytest module: run it directly.

    python oracle/build_ref_scan.py            # once, in a container that has the reference
    python tests/ref_kernel_timing.py [--quick]

Workloads: BASELINE config 4 (32 x 3072 x L, n 16, bf16 I/O, z, D, delta_bias, softplus) at
L = 1024 and 4096 (fwd and bwd separately), the module's d_state 32 and 64 size presets at
8 x d_inner x 2048, and the motif P/Q path (rank 4, shared P/Q, no z
since the reference's P/Q backward has none) at sizes the reference's one-thread-per-row kernels
(forward O(L), backward O(L^2)) finish in seconds.  Each line: CUDA-event median over the timed
calls after warm-up on the current stream; inputs are > 126 MB L2 for config 4.  Prints one
JSON line per workload with both times and the ratio.
"""
import argparse
import json
import os
import statistics
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "motif-mamba_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402


def _time(fn, warmup, iters):
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


def _inputs(b, d, l, n, dtype, z=True, pq_rank=0, seed=0):
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


def _bench(mod, t, pq, warmup, iters, do_bwd=True):
    kw = dict(D=t["D"], z=t["z"], delta_bias=t["delta_bias"])
    if pq:
        kw.update(P=t["P"], Q=t["Q"])
    args = (t["u"], t["delta"], t["A"], t["B"], t["C"])
    fwd = lambda: mod.fwd(*args, delta_softplus=True, **kw)
    ms_f = _time(fwd, warmup, iters)
    ms_b = None
    if do_bwd:
        out, x, *_ = fwd()
        dP = torch.zeros_like(t["P"]) if pq else None
        dQ = torch.zeros_like(t["Q"]) if pq else None
        bwd = lambda: mod.bwd(*args, dout=t["dout"], x=x, out=out if t["z"] is not None else None, dz=None,
                              dP_out=dP, dQ_out=dQ, delta_softplus=True, recompute_out_z=False, **kw)
        ms_b = _time(bwd, warmup, iters)
    return ms_f, ms_b


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true", help="config 4 at L=1024 only")
    a = ap.parse_args()
    from oracle import build_ref_scan
    ref = build_ref_scan.load()
    if ref is None:
        print(json.dumps({"unavailable": "reference extension not built (python oracle/build_ref_scan.py)"}))
        return 0
    from motif_ssm import selective_scan_cuda as ours
    work = [("config4", 32, 3072, L, 16, torch.bfloat16, True, 0, True) for L in ((1024,) if a.quick else (1024, 4096))]
    if not a.quick:
        # the module's larger size presets (d_state 32 / 64, mamba_simplemotif.py:32-36), z on
        work += [("small_n32", 8, 1024, 2048, 32, torch.bfloat16, True, 0, True),
                 ("base_n64", 8, 1536, 2048, 64, torch.bfloat16, True, 0, True)]
        work += [("pq_fwd", 8, 1536, 2048, 16, torch.bfloat16, False, 4, False),
                 ("pq_fwd_bwd", 2, 1536, 256, 16, torch.bfloat16, False, 4, True)]
    for name, b, d, l, n, dtype, z, r, do_bwd in work:
        t = _inputs(b, d, l, n, dtype, z=z, pq_rank=r)
        iters = 3 if r else 10
        of, ob = _bench(ours, t, r > 0, 3, iters, do_bwd)
        rf, rb = _bench(ref, t, r > 0, 1 if r else 3, iters, do_bwd)
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
