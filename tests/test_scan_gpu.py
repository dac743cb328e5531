"""Parity of the sm_100a selective scan (through the C ABI) with the CPU oracle and
with the golden fixtures produced by the reference's own code.

Tolerances (north star): outputs, last_state and the 8 gradients within 1e-3 for fp32
I/O and 2e-2 for bf16/fp16 I/O, elementwise (|a - e| <= atol + rtol |e|) for
outputs, last_state, du, ddelta and dz; sums over channels / batch (dA, dB, dC, dD,
ddelta_bias) relative to the tensor's magnitude (see ``ssm_cases.assert_close``)."""
import glob
import os

import pytest
import torch

from oracle import ssm_oracle as O
from ssm_cases import SUM_GRADS, assert_close, make_scan_inputs, oracle_fp32_math, tol

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"
GRAD_KEYS = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")


def run_kernel(inputs, dout, softplus, backward=True):
    from motif_ssm import selective_scan_fn
    leaves = {k: (v.detach().to(DEV).clone().requires_grad_(backward) if v is not None else None)
              for k, v in inputs.items()}
    out, last = selective_scan_fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                  leaves["D"], z=leaves["z"], delta_bias=leaves["delta_bias"],
                                  delta_softplus=softplus, return_last_state=True,
                                  P=leaves.get("P"), Q=leaves.get("Q"))
    grads = None
    if backward:
        out.backward(dout.to(DEV))
        grads = {k: (v.grad if v is not None else None) for k, v in leaves.items()}
    torch.cuda.synchronize()
    return out, last, grads


def compare(out, last, grads, ref_out, ref_last, ref_grads, dtype, what=""):
    t = tol(dtype)
    assert out.dtype == ref_out.dtype
    assert_close(out, ref_out, t, t, f"{what} out")
    assert_close(last, ref_last, t, t, f"{what} last_state")
    if grads is not None:
        for k in GRAD_KEYS + tuple(k for k in ("P", "Q") if ref_grads.get(k) is not None):
            if ref_grads.get(k) is None:
                assert grads[k] is None, k
                continue
            assert grads[k] is not None, k
            assert_close(grads[k], ref_grads[k], t, t, f"{what} d{k}", scaled=k in SUM_GRADS)


def oracle(inputs, dout, softplus):
    return oracle_fp32_math(inputs, dout, softplus)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "scan_*.pt"))),
                         ids=lambda p: os.path.basename(p)[5:-3])
def test_scan_matches_reference_golden(path):
    rec = torch.load(path, weights_only=False)
    inp = rec["inputs"]
    out, last, grads = run_kernel(inp, rec["dout"], rec["softplus"])
    compare(out, last, grads, rec["out"], rec["last_state"], rec["grads"], inp["u"].dtype, rec["name"])


CASES = [
    # batch, dim, seqlen, dstate, dtype, groups, z, D, bias, softplus
    (2, 8, 1, 16, torch.float32, 0, True, True, True, True),
    (2, 8, 7, 16, torch.float32, 0, False, True, False, True),
    (1, 24, 255, 16, torch.float32, 0, True, False, True, True),
    (1, 24, 257, 16, torch.bfloat16, 0, True, True, True, True),
    (2, 40, 513, 16, torch.float32, 0, True, True, True, False),
    (1, 16, 1000, 8, torch.float16, 0, True, True, True, True),
    (2, 32, 300, 4, torch.float32, 2, True, True, True, True),
    (1, 4, 2049, 16, torch.bfloat16, 0, True, True, True, True),   # time-split forward
    (1, 8, 9000, 16, torch.float32, 0, True, True, True, True),    # 113 segments
    (1, 8, 1088, 16, torch.float32, 0, True, True, True, True),    # 17 segments: 16 carries, 2 whole batches
    (1, 8, 1088, 64, torch.float32, 0, True, True, True, True),    # the same, a row's states over 2 warps
    (3, 130, 130, 16, torch.float32, 0, True, True, True, True),   # partial channel tiles
    (1, 8, 70, 1, torch.float32, 0, True, True, True, True),
    (1, 8, 70, 13, torch.float32, 0, True, True, True, True),
    (2, 24, 300, 32, torch.bfloat16, 0, True, True, True, True),   # state blocks of 16
    (1, 16, 530, 64, torch.float32, 0, True, True, True, True),
    (1, 8, 90, 20, torch.float32, 2, False, True, False, True),
    # rows split over 2 / 4 threads (dstate 32 / 64), with time split and partial channel tiles
    (1, 70, 1100, 32, torch.bfloat16, 0, True, True, True, True),
    (2, 33, 700, 64, torch.float32, 0, True, True, True, True),
    (1, 40, 300, 48, torch.float16, 2, False, True, True, True),
    # a wave of rows or more: dstate 32 / 64 rows in one thread each
    (38, 1000, 20, 32, torch.bfloat16, 0, True, True, True, True),
    (40, 1000, 17, 64, torch.float32, 0, False, True, True, True),
    # dstate above 64 (up to the reference's 256): 8 / 16 lanes of 16 states per row, 16-state blocks
    (1, 16, 300, 100, torch.float32, 0, True, True, True, True),
    (2, 12, 270, 128, torch.bfloat16, 0, True, True, True, True),
    (1, 8, 600, 256, torch.float32, 2, True, True, True, True),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}d{}l{}n{}-{}-g{}{}{}{}{}".format(
    c[0], c[1], c[2], c[3], str(c[4])[6:], c[5], "z" * c[6], "D" * c[7], "b" * c[8], "sp" * c[9]))
def test_scan_matches_oracle(case):
    batch, dim, seqlen, dstate, dtype, groups, z, D, bias, sp = case
    inp, dout = make_scan_inputs(batch, dim, seqlen, dstate, dtype, groups, z, D, bias, sp, seed=seqlen)
    ref_out, ref_last, ref_grads = oracle(inp, dout, sp)
    out, last, grads = run_kernel(inp, dout, sp)
    compare(out, last, grads, ref_out, ref_last, ref_grads, dtype, str(case))


def test_scan_strided_views_like_mamba_inner():
    """x / z as halves of one (b, 2d, l) tensor and delta as a transposed GEMM output --
    the layouts mamba_inner_fn hands the scan (selective_scan_interface.py:480-489)."""
    from motif_ssm import selective_scan_cuda
    batch, dim, seqlen, n = 2, 48, 96, 16
    inp, dout = make_scan_inputs(batch, dim, seqlen, n, torch.bfloat16, seed=11)
    xz = torch.cat([inp["u"], inp["z"]], dim=1).to(DEV)
    u, z = xz.chunk(2, dim=1)
    delta = inp["delta"].transpose(0, 1).contiguous().transpose(0, 1).to(DEV)  # strides (l, b*l, 1)
    assert not u.is_contiguous() and not delta.is_contiguous()
    B = inp["B"].unsqueeze(1).to(DEV)
    C = inp["C"].unsqueeze(1).to(DEV)
    args = (inp["A"].to(DEV), B, C)
    out, x, out_z = selective_scan_cuda.fwd(u, delta, *args, D=inp["D"].to(DEV), z=z,
                                            delta_bias=inp["delta_bias"].to(DEV), delta_softplus=True)
    ref = O.selective_scan_ref(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], inp["D"], z=inp["z"],
                               delta_bias=inp["delta_bias"], delta_softplus=True)
    assert_close(out_z, ref, 2e-2, 2e-2, "strided out_z")


@pytest.mark.parametrize("seqlen", [1024, 4096, 16384])
def test_scan_full_size_rows_and_linearity(seqlen):
    """BASELINE config 4 (32 x 3072 x {1024, 4096, 16384}, bf16): the full-size forward agrees
    with the oracle on sampled rows, and dout confined to a few channels gives gradients the
    oracle reproduces exactly from those channels alone (dB/dC sums included)."""
    from motif_ssm import selective_scan_fn
    batch, dim, n = 32, 3072, 16
    g = torch.Generator(device=DEV).manual_seed(0)
    u = torch.randn(batch, dim, seqlen, device=DEV, generator=g).bfloat16()
    delta = torch.randn(batch, dim, seqlen, device=DEV, generator=g).bfloat16()
    z = torch.randn(batch, dim, seqlen, device=DEV, generator=g).bfloat16()
    B = torch.randn(batch, n, seqlen, device=DEV, generator=g).bfloat16()
    C = torch.randn(batch, n, seqlen, device=DEV, generator=g).bfloat16()
    A = -torch.arange(1, n + 1, device=DEV, dtype=torch.float32).repeat(dim, 1)
    D = 1 + 0.1 * torch.randn(dim, device=DEV, generator=g)
    bias = torch.log(torch.expm1(torch.rand(dim, device=DEV, generator=g) * 0.099 + 1e-3))
    leaves = [t.clone().requires_grad_(True) for t in (u, delta, A, B, C, D, z, bias)]
    out, last = selective_scan_fn(leaves[0], leaves[1], leaves[2], leaves[3], leaves[4], leaves[5],
                                  z=leaves[6], delta_bias=leaves[7], delta_softplus=True, return_last_state=True)
    bsel, dsel = 5, torch.tensor([0, 1, 777, 1500, 3071])
    dout = torch.zeros_like(out)
    dout[bsel, dsel] = torch.randn(len(dsel), seqlen, device=DEV, generator=g).bfloat16()
    out.backward(dout)
    torch.cuda.synchronize()
    cpu = lambda t: t.detach().cpu()
    sub = dict(u=cpu(u[bsel:bsel + 1, dsel]), delta=cpu(delta[bsel:bsel + 1, dsel]), A=cpu(A[dsel]),
               B=cpu(B[bsel:bsel + 1]), C=cpu(C[bsel:bsel + 1]), D=cpu(D[dsel]), z=cpu(z[bsel:bsel + 1, dsel]),
               delta_bias=cpu(bias[dsel]))
    r_out, r_last, r_g = oracle_fp32_math(sub, cpu(dout[bsel:bsel + 1, dsel]), True)
    t = 2e-2
    assert_close(out[bsel:bsel + 1, dsel], r_out, t, t, "full-size out rows")
    assert_close(last[bsel:bsel + 1, dsel], r_last, t, t, "full-size last_state rows")
    gu, gdelta, gA, gB, gC, gD, gz, gbias = (l.grad for l in leaves)
    assert_close(gu[bsel:bsel + 1, dsel], r_g["u"], t, t, "du rows")
    assert_close(gdelta[bsel:bsel + 1, dsel], r_g["delta"], t, t, "ddelta rows")
    assert_close(gz[bsel:bsel + 1, dsel], r_g["z"], t, t, "dz rows")
    assert_close(gA[dsel], r_g["A"], t, t, "dA rows", scaled=True)
    assert_close(gD[dsel], r_g["D"], t, t, "dD rows", scaled=True)
    assert_close(gbias[dsel], r_g["delta_bias"], t, t, "ddelta_bias rows", scaled=True)
    assert_close(gB[bsel:bsel + 1], r_g["B"], t, t, "dB (sum over channels)", scaled=True)
    assert_close(gC[bsel:bsel + 1], r_g["C"], t, t, "dC (sum over channels)", scaled=True)
    # every other row got no gradient
    mask = torch.ones(batch, dim, dtype=torch.bool, device=DEV)
    mask[bsel, dsel] = False
    assert gu[mask].abs().max().item() == 0.0
    assert gB[torch.arange(batch, device=DEV) != bsel].abs().max().item() == 0.0
    del leaves, out, last, dout, gu, gdelta, gA, gB, gC, gD, gz, gbias, u, delta, z, B, C
    torch.cuda.empty_cache()


def test_fwd_is_deterministic_and_x_layout():
    from motif_ssm import selective_scan_cuda
    inp, _ = make_scan_inputs(2, 64, 600, 16, torch.bfloat16, seed=3, device=DEV)
    B, C = inp["B"].unsqueeze(1), inp["C"].unsqueeze(1)
    r1 = selective_scan_cuda.fwd(inp["u"], inp["delta"], inp["A"], B, C, D=inp["D"], z=inp["z"],
                                 delta_bias=inp["delta_bias"], delta_softplus=True)
    r2 = selective_scan_cuda.fwd(inp["u"], inp["delta"], inp["A"], B, C, D=inp["D"], z=inp["z"],
                                 delta_bias=inp["delta_bias"], delta_softplus=True)
    for a, b in zip(r1, r2):
        assert torch.equal(a, b)
    out, x, out_z = r1
    assert x.shape == (2, 64, 3, 32) and x.dtype == torch.float32
    # x[..., 0::2] is the cumulative decay exp(A * sum(dt)): in (0, 1] and non-increasing over chunks
    dec = x[..., 0::2]
    assert (dec > 0).all() or (dec >= 0).all()
    assert (dec[:, :, 1:] <= dec[:, :, :-1] * (1 + 1e-6)).all()


def test_bwd_accepts_preallocated_dz_in_place():
    from motif_ssm import selective_scan_cuda
    inp, dout = make_scan_inputs(2, 16, 100, 16, torch.float32, seed=5, device=DEV)
    B, C = inp["B"].unsqueeze(1), inp["C"].unsqueeze(1)
    out, x, out_z = selective_scan_cuda.fwd(inp["u"], inp["delta"], inp["A"], B, C, D=inp["D"], z=inp["z"],
                                            delta_bias=inp["delta_bias"], delta_softplus=True)
    buf = torch.full((2, 32, 100), 7.0, device=DEV)
    dz_view = buf[:, 16:]
    res = selective_scan_cuda.bwd(inp["u"], inp["delta"], inp["A"], B, C, D=inp["D"], z=inp["z"],
                                  delta_bias=inp["delta_bias"], dout=dout, x=x, out=out, dz=dz_view,
                                  delta_softplus=True, recompute_out_z=True)
    assert res[7].data_ptr() == dz_view.data_ptr()
    assert (buf[:, :16] == 7.0).all()
    assert_close(res[8], out_z, 1e-5, 1e-5, "recomputed out_z")


def test_scan_extreme_delta_and_z():
    """delta + bias spanning the softplus threshold (-30 .. 30) and large |z| (sigmoid tails)."""
    inp, dout = make_scan_inputs(2, 32, 200, 16, torch.float32, seed=9)
    inp["delta"] = inp["delta"] * 12.0
    inp["z"] = inp["z"] * 15.0
    ref_out, ref_last, ref_grads = oracle(inp, dout, True)
    out, last, grads = run_kernel(inp, dout, True)
    compare(out, last, grads, ref_out, ref_last, ref_grads, torch.float32, "extreme delta/z")


@pytest.mark.parametrize("dtype,seqlen,dstate", [(torch.float32, 300, 16), (torch.bfloat16, 700, 16),
                                                 (torch.float32, 2049, 16), (torch.float32, 2049, 32),
                                                 (torch.bfloat16, 700, 64)])
def test_scan_unstructured_A(dtype, seqlen, dstate):
    """A without the S4D-real (n+1) A_0 structure takes the per-state exp path."""
    inp, dout = make_scan_inputs(2, 40, seqlen, dstate, dtype, seed=seqlen + 1, random_A=True)
    ref_out, ref_last, ref_grads = oracle(inp, dout, True)
    out, last, grads = run_kernel(inp, dout, True)
    compare(out, last, grads, ref_out, ref_last, ref_grads, dtype, "random A")


@pytest.mark.parametrize("dstate", [16, 64])
def test_scan_mixed_structure_in_one_cta(dstate):
    """Channels with and without the structure side by side in one CTA (with 64 states, only
    the last of a row's four threads sees the break)."""
    inp, dout = make_scan_inputs(1, 64, 400, dstate, torch.float32, seed=77)
    if dstate == 16:
        inp["A"][5] = -torch.exp(torch.randn(16))
    else:
        inp["A"][5, 60] *= 1.5
    ref_out, ref_last, ref_grads = oracle(inp, dout, True)
    out, last, grads = run_kernel(inp, dout, True)
    compare(out, last, grads, ref_out, ref_last, ref_grads, torch.float32, "mixed A")


@pytest.mark.parametrize("batch,dim,seqlen,dtype", [(2, 64, 1000, torch.float32), (1, 40, 4100, torch.float32),
                                                    (2, 96, 2000, torch.bfloat16)])
def test_initial_state_chains_sequence_pieces(batch, dim, seqlen, dtype):
    """fwd(..., initial_state=h): scanning a sequence in pieces, each started from the previous
    piece's final state x[:, :, -1, 1::2], gives the full scan's outputs and final state (the
    second shape runs with the time split, whose carry scan composes h in front of segment 0)."""
    from motif_ssm import selective_scan_cuda as ssc
    inp, _ = make_scan_inputs(batch, dim, seqlen, 16, dtype, seed=31, device=DEV)
    B, C = inp["B"].unsqueeze(1), inp["C"].unsqueeze(1)
    kw = dict(D=inp["D"], delta_bias=inp["delta_bias"], delta_softplus=True)
    out, x, out_z = ssc.fwd(inp["u"], inp["delta"], inp["A"], B, C, z=inp["z"], **kw)
    cuts = [0, 300, 700, seqlen]
    h, pieces, pieces_z = None, [], []
    for t0, t1 in zip(cuts[:-1], cuts[1:]):
        sl = lambda t: t[..., t0:t1]
        o, xp, oz = ssc.fwd(sl(inp["u"]), sl(inp["delta"]), inp["A"], sl(B), sl(C), z=sl(inp["z"]), initial_state=h,
                            **kw)
        pieces.append(o)
        pieces_z.append(oz)
        h = xp[:, :, -1, 1::2].contiguous()
    t = 1e-5 if dtype == torch.float32 else tol(dtype)
    assert_close(torch.cat(pieces, -1), out, t, t, "out from pieces")
    assert_close(torch.cat(pieces_z, -1), out_z, t, t, "out_z from pieces")
    assert_close(h, x[:, :, -1, 1::2], 1e-5, 1e-5, "final state from pieces")
    with pytest.raises(RuntimeError):
        ssc.fwd(inp["u"], inp["delta"], inp["A"], B, C, z=inp["z"], initial_state=h[:, :1], **kw)
