"""This library against the reference's own CUDA extension (``selective_scan_cuda`` built from
the reference's sources for sm_100a by ``oracle/build_ref_scan.py`` into ``oracle/_ref/``).

Both implementations get identical device inputs through the same call signature
(``fwd`` / ``bwd`` of ``selective_scan.cpp:620-637``); outputs and gradients must agree within
the north-star tolerances (1e-3 fp32 I/O, 2e-2 bf16/fp16 I/O, relative to the tensor's
magnitude).  Skipped when the reference extension has not been built."""
import pytest
import torch

from ssm_cases import assert_close, make_scan_inputs, tol

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ref():
    from oracle import build_ref_scan
    mod = build_ref_scan.load()
    if mod is None:
        pytest.skip("reference extension not built (python oracle/build_ref_scan.py)")
    return mod


def _dev(inp):
    d = {k: (v.to(DEV) if v is not None else None) for k, v in inp.items()}
    for k in ("B", "C"):
        if d[k].dim() == 3:
            d[k] = d[k].unsqueeze(1)
    return d


def _both(ref, d, dout, softplus, pq=False):
    from motif_ssm import selective_scan_cuda as ours
    res = {}
    for name, mod in (("ours", ours), ("ref", ref)):
        kw = dict(D=d["D"], z=d["z"], delta_bias=d["delta_bias"])
        if pq:
            kw.update(P=d["P"], Q=d["Q"])
        out, x, *rest = mod.fwd(d["u"], d["delta"], d["A"], d["B"], d["C"], delta_softplus=softplus, **kw)
        dP = torch.zeros_like(d["P"]) if pq else None
        dQ = torch.zeros_like(d["Q"]) if pq else None
        grads = mod.bwd(d["u"], d["delta"], d["A"], d["B"], d["C"], dout=dout, x=x,
                        out=out if d["z"] is not None else None, dz=None, dP_out=dP, dQ_out=dQ,
                        delta_softplus=softplus, recompute_out_z=False, **kw)
        torch.cuda.synchronize()
        res[name] = dict(out=out, last=x[:, :, -1, 1::2], out_z=rest[0] if rest else None,
                         grads=grads, dP=dP, dQ=dQ)
    return res["ours"], res["ref"]


def _compare(a, b, dtype, what):
    t = tol(dtype)
    assert_close(a["out"], b["out"], t, t, f"{what} out")
    assert_close(a["last"], b["last"], t, t, f"{what} last_state")
    if b["out_z"] is not None:
        assert_close(a["out_z"], b["out_z"], t, t, f"{what} out_z")
    names = ("du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias", "dz")
    for n, ga, gb in zip(names, a["grads"], b["grads"]):
        if gb is None or not gb.numel():
            continue
        assert_close(ga, gb, t, t, f"{what} {n}")
    if b["dP"] is not None:
        assert_close(a["dP"], b["dP"], t, t, f"{what} dP")
        assert_close(a["dQ"], b["dQ"], t, t, f"{what} dQ")


CASES = [
    # batch, dim, seqlen, dstate, dtype, groups, z, D, bias, softplus
    (2, 256, 4100, 16, torch.bfloat16, 0, True, True, True, True),     # config-4 shape, 3 reference chunks
    (2, 64, 300, 16, torch.float32, 0, True, True, True, True),
    (1, 48, 777, 8, torch.float16, 2, False, True, False, True),
    (2, 40, 513, 32, torch.bfloat16, 0, True, True, True, False),
    (1, 24, 130, 64, torch.float32, 0, True, False, True, True),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}d{}l{}n{}-{}-g{}".format(*c[:4], str(c[4])[6:], c[5]))
def test_scan_matches_reference_kernel(ref, case):
    batch, dim, seqlen, dstate, dtype, groups, z, D, bias, sp = case
    inp, dout = make_scan_inputs(batch, dim, seqlen, dstate, dtype, groups, z, D, bias, sp, seed=seqlen)
    a, b = _both(ref, _dev(inp), dout.to(DEV), sp)
    _compare(a, b, dtype, str(case))


PQ_CASES = [
    # batch, dim, seqlen, dstate, dtype, rank, per_dim  (the reference P/Q backward has no z)
    (2, 32, 96, 16, torch.float32, 2, False),
    (1, 40, 64, 8, torch.bfloat16, 4, True),
]


@pytest.mark.parametrize("case", PQ_CASES, ids=lambda c: "b{}d{}l{}n{}-{}-r{}{}".format(
    *c[:4], str(c[4])[6:], c[5], "pd" * c[6]))
def test_pq_scan_matches_reference_kernel(ref, case):
    batch, dim, seqlen, dstate, dtype, r, per_dim = case
    inp, dout = make_scan_inputs(batch, dim, seqlen, dstate, dtype, has_z=False, seed=seqlen + r,
                                 pq_rank=r, pq_per_dim=per_dim, pq_scale=0.3)
    a, b = _both(ref, _dev(inp), dout.to(DEV), True, pq=True)
    _compare(a, b, dtype, str(case))
