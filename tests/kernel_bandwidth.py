"""Achieved HBM bandwidth of the kernels around the scan: causal conv1d forward / backward,
the fused residual add + RMSNorm, and the two decode kernels (conv1d update and the SSM state
update).  Test infrastructure, not a pytest module: run it directly on a B200.

    python tests/kernel_bandwidth.py            # CUDA-event medians, one JSON line per kernel
    python tests/kernel_bandwidth.py --once     # each kernel twice, for an ncu launch capture

Shapes: the conv and the norm at BASELINE config 2's prefill (16 x 4096 tokens, d_inner 1536,
d_model 768, bf16; every tensor > 126 MB L2 except the conv weights), the decode kernels at
its decode step (batch 64, d_inner 1536, d_state 16), whose few MB stay in L2: those two are
launch- and latency-bound and their GB/s says so.  Bytes are the algorithmic ones: every input
read once, every output written once.
"""
import argparse
import json
import os
import statistics
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "motif-mamba_b200"))

import torch  # noqa: E402


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--once", action="store_true")
    args = ap.parse_args()
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
    for name, shape, fn, nbytes in work:
        if args.once:
            fn()
            fn()
            torch.cuda.synchronize()
            continue
        ms = _median_ms(fn)
        print(json.dumps({"kernel": name, "shape": shape, "ms": round(ms, 5), "bytes": nbytes,
                          "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1)}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
