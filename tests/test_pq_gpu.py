"""Parity of the motif low-rank coupling path (``selective_scan_fn(..., P=, Q=)``, the
``ss_pq`` kernels behind the C ABI) with the CPU oracle, which follows the reference's
``selective_scan_ref`` P/Q recurrence (selective_scan_interface.py:402-433) and is pinned by
the golden fixtures ``scan_pq*.pt`` that test_scan_gpu.py replays.

Tolerances as for the plain scan: 1e-3 for fp32 I/O, 2e-2 for bf16/fp16 I/O, elementwise
for out, last_state, du, ddelta, dz; sums (dA, dB, dC, dD, ddelta_bias and dP / dQ, fp32 sums
over batch, steps and, when shared, channels) relative to the tensor's magnitude."""
import pytest
import torch

from oracle import ssm_oracle as O
from ssm_cases import SUM_GRADS, assert_close, make_scan_inputs, oracle_fp32_math, tol

pytestmark = pytest.mark.gpu
DEV = "cuda"
KEYS = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias", "P", "Q")


def _run(inp, dout, softplus):
    from motif_ssm import selective_scan_fn
    leaves = {k: (v.detach().to(DEV).clone().requires_grad_(True) if v is not None else None)
              for k, v in inp.items()}
    out, last = selective_scan_fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                  leaves["D"], z=leaves["z"], delta_bias=leaves["delta_bias"],
                                  delta_softplus=softplus, return_last_state=True, P=leaves["P"], Q=leaves["Q"])
    out.backward(dout.to(DEV))
    torch.cuda.synchronize()
    return out, last, {k: (v.grad if v is not None else None) for k, v in leaves.items()}


def _check(inp, dout, softplus, dtype, what):
    ref_out, ref_last, ref_grads = oracle_fp32_math(inp, dout, softplus)
    out, last, grads = _run(inp, dout, softplus)
    t = tol(dtype)
    assert out.dtype == dtype
    assert_close(out, ref_out, t, t, f"{what} out")
    assert_close(last, ref_last, t, t, f"{what} last_state")
    for k in KEYS:
        if ref_grads.get(k) is None:
            assert grads.get(k) is None, k
            continue
        assert_close(grads[k], ref_grads[k], t, t, f"{what} d{k}", scaled=k in SUM_GRADS)


CASES = [
    # batch, dim, seqlen, dstate, dtype, rank, per_dim, groups, z, D, bias, softplus
    (2, 8, 1, 16, torch.float32, 2, False, 0, True, True, True, True),
    (1, 33, 17, 16, torch.float32, 1, True, 0, True, False, True, True),    # partial tile, ragged L
    (2, 70, 300, 16, torch.bfloat16, 4, False, 0, True, True, True, True),
    (1, 40, 530, 8, torch.float16, 8, True, 0, False, True, True, True),
    (2, 64, 257, 4, torch.float32, 3, False, 2, True, True, True, True),    # 2 groups of B / C
    (1, 16, 1030, 16, torch.float32, 2, True, 0, True, True, False, False),
    (3, 96, 64, 13, torch.float32, 5, False, 0, False, False, False, True),
    (2, 40, 300, 32, torch.bfloat16, 4, False, 0, True, True, True, True),    # 8 lanes per channel
    (1, 24, 530, 20, torch.float32, 3, True, 0, True, True, True, True),
    (2, 20, 200, 64, torch.float32, 2, False, 2, True, True, True, True),     # 16 lanes per channel
    (1, 12, 77, 40, torch.float16, 8, True, 0, False, True, True, True),
    (3, 40, 150, 16, torch.float32, 4, True, 0, True, True, True, True),     # per-channel P / Q, batch 3
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}d{}l{}n{}-{}-r{}{}-g{}{}{}{}{}".format(
    c[0], c[1], c[2], c[3], str(c[4])[6:], c[5], "pd" * c[6], c[7], "z" * c[8], "D" * c[9], "b" * c[10],
    "sp" * c[11]))
def test_pq_scan_matches_oracle(case):
    batch, dim, seqlen, dstate, dtype, r, per_dim, groups, z, D, bias, sp = case
    inp, dout = make_scan_inputs(batch, dim, seqlen, dstate, dtype, groups, z, D, bias, sp, seed=seqlen + r,
                                 pq_rank=r, pq_per_dim=per_dim, pq_scale=0.3)
    _check(inp, dout, sp, dtype, str(case))


def test_pq_scan_long_sequence():
    """2048 steps (eight 256-step chunks of x, 128 backward segments) on 96 channels."""
    inp, dout = make_scan_inputs(2, 96, 2048, 16, torch.bfloat16, seed=5, pq_rank=4, pq_scale=0.15)
    _check(inp, dout, True, torch.bfloat16, "long")


def test_pq_zero_coupling_equals_plain_scan():
    """P = 0 reduces the recurrence to the plain scan: both kernels agree (out, grads)."""
    from motif_ssm import selective_scan_fn
    inp, dout = make_scan_inputs(2, 48, 600, 16, torch.float32, seed=9, pq_rank=2)
    dev = {k: v.to(DEV) for k, v in inp.items() if v is not None}
    P0 = torch.zeros_like(dev["P"])
    a = selective_scan_fn(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], dev["D"], z=dev["z"],
                          delta_bias=dev["delta_bias"], delta_softplus=True, P=P0, Q=dev["Q"])
    b = selective_scan_fn(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], dev["D"], z=dev["z"],
                          delta_bias=dev["delta_bias"], delta_softplus=True)
    assert_close(a, b, 1e-4, 1e-4, "P=0 vs plain")


def test_pq_bwd_writes_caller_dP_dQ():
    """``selective_scan_cuda.bwd(dP_out=, dQ_out=)`` fills the caller's fp32 buffers
    (selective_scan.cpp:579-590); the return list is the reference's seven (+dz)."""
    from motif_ssm import selective_scan_cuda
    inp, dout = make_scan_inputs(1, 32, 100, 16, torch.float32, has_z=False, seed=3, pq_rank=2, pq_per_dim=True)
    d = {k: (v.to(DEV) if v is not None else None) for k, v in inp.items()}
    B, C = d["B"].unsqueeze(1), d["C"].unsqueeze(1)
    out, x = selective_scan_cuda.fwd(d["u"], d["delta"], d["A"], B, C, D=d["D"], delta_bias=d["delta_bias"],
                                     P=d["P"], Q=d["Q"], delta_softplus=True)
    dP = torch.full_like(d["P"], 7.0)
    dQ = torch.full_like(d["Q"], 7.0)
    res = selective_scan_cuda.bwd(d["u"], d["delta"], d["A"], B, C, D=d["D"], delta_bias=d["delta_bias"],
                                  P=d["P"], Q=d["Q"], dout=dout.to(DEV), x=x, dP_out=dP, dQ_out=dQ,
                                  delta_softplus=True)
    assert len(res) == 7
    _, _, ref_grads = O.scan_with_grads(inp, dout, True)
    assert_close(dP, ref_grads["P"], 1e-3, 1e-3, "dP_out")
    assert_close(dQ, ref_grads["Q"], 1e-3, 1e-3, "dQ_out")


def test_pq_argument_errors():
    from motif_ssm import selective_scan_fn
    inp, _ = make_scan_inputs(1, 8, 16, 80, torch.float32, seed=1, pq_rank=2)
    d = {k: (v.to(DEV) if v is not None else None) for k, v in inp.items()}
    args = (d["u"], d["delta"], d["A"], d["B"], d["C"])
    with pytest.raises(NotImplementedError):      # dstate 80 > 64 with the coupling
        selective_scan_fn(*args, P=d["P"], Q=d["Q"])
    inp, _ = make_scan_inputs(1, 8, 16, 16, torch.float32, seed=1, pq_rank=2)
    d = {k: (v.to(DEV) if v is not None else None) for k, v in inp.items()}
    args = (d["u"], d["delta"], d["A"], d["B"], d["C"])
    with pytest.raises(ValueError):
        selective_scan_fn(*args, P=d["P"])
    with pytest.raises(RuntimeError):             # rank 9 > 8
        selective_scan_fn(*args, P=torch.zeros(16, 9, device=DEV), Q=torch.zeros(9, 16, device=DEV))
    with pytest.raises(RuntimeError):             # P / Q shapes disagree
        selective_scan_fn(*args, P=torch.zeros(16, 2, device=DEV), Q=torch.zeros(3, 16, device=DEV))


def test_pq_partial_tile_repeatable():
    """A CTA's padding channels (dim not a multiple of 32) must not touch real channels'
    rows: repeated backward calls on a 16-channel problem give the same gradients (bit for
    bit where no float atomics are involved; per-channel dP / dQ sum the batch rows with
    atomics, so those are compared at 1e-6)."""
    inp, dout = make_scan_inputs(2, 16, 1030, 16, torch.float32, seed=12, pq_rank=3, pq_per_dim=True, pq_scale=0.3)
    runs = [_run(inp, dout, True) for _ in range(3)]
    for out, last, grads in runs[1:]:
        assert torch.equal(out, runs[0][0])
        for k in KEYS:
            if grads[k] is None:
                continue
            if k in ("P", "Q"):
                assert_close(grads[k], runs[0][2][k], 1e-6, 1e-6, k)
            else:
                assert torch.equal(grads[k], runs[0][2][k]), k


def test_full_matrix_entry_point_equals_selective_scan_fn():
    """selective_scan_full_matrix_cuda (the reference's per-step P/Q path, here on the kernels)
    gives selective_scan_fn's P/Q results and gradients; its argument checks raise as there."""
    from motif_ssm.selective_scan_interface import selective_scan_full_matrix_cuda
    from motif_ssm import selective_scan_fn
    inp, dout = make_scan_inputs(2, 24, 150, 16, torch.float32, seed=21, pq_rank=2)
    res = []
    for fn in (selective_scan_full_matrix_cuda, selective_scan_fn):
        leaves = {k: v.to(DEV).clone().requires_grad_(True) for k, v in inp.items() if v is not None}
        out, last = fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], leaves["D"],
                       z=leaves["z"], delta_bias=leaves["delta_bias"], delta_softplus=True, return_last_state=True,
                       P=leaves["P"], Q=leaves["Q"])
        out.backward(dout.to(DEV))
        res.append((out, last, {k: v.grad for k, v in leaves.items()}))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])
    for k in res[0][2]:
        assert_close(res[0][2][k], res[1][2][k], 1e-6, 1e-6, k)
    with pytest.raises(ValueError):
        selective_scan_full_matrix_cuda(res[0][0], res[0][0], inp["A"].to(DEV), inp["B"].to(DEV),
                                        inp["C"].to(DEV), P=None, Q=inp["Q"].to(DEV))
