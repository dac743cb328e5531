"""ss_bwd_noalloc: the backward for callers that may not allocate device memory (their
memory belongs to another allocator, or their runtime forbids cudaMalloc once running).
It takes its scratch from a static array inside the library instead of a workspace.

Called through the C ABI and compared with ss_bwd (which gets a torch-allocated
workspace) on the same inputs, twice in a row, since every call reuses the same array.
This file is collected last so a failure here leaves every other test already run."""
import ctypes

import pytest
import torch

from ssm_cases import assert_close, make_scan_inputs, tol

pytestmark = pytest.mark.gpu
SUM_NAMES = {"dA", "dB", "dC", "dD", "ddelta_bias", "dP", "dQ"}
DEV = "cuda"


def _noalloc_bwd(inp, x, out, dout, softplus):
    """Fill ss_bwd_args exactly as selective_scan_cuda.bwd does, allocate the outputs here,
    and call ss_bwd_noalloc (no workspace passed).  Returns the 8 gradients (plus dP, dQ
    when the inputs carry the motif coupling)."""
    from motif_ssm import _lib
    from motif_ssm import selective_scan_cuda as ssc
    u, delta, A, B, C, D, z, bias = (inp[k] for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias"))
    P, Q = inp.get("P"), inp.get("Q")
    sizes = ssc._check_common(u, delta, A, B, C, D, z, bias, P, Q, None)
    a = _lib.SsBwdArgs()
    ssc._fill_common(a, u, delta, A, B, C, D, z, bias, sizes, softplus)
    ssc._fill_pq(a, P, Q)
    dP = dQ = None
    if P is not None:
        dP, dQ = torch.empty_like(P), torch.empty_like(Q)
        a.dP, a.dQ = dP.data_ptr(), dQ.data_ptr()
    du, ddelta, dz = torch.empty_like(u), torch.empty_like(delta), torch.empty_like(z)
    dA, dB, dC = torch.empty_like(A), torch.empty_like(B), torch.empty_like(C)
    dD, dbias = torch.empty_like(D), torch.empty_like(bias)
    a.out, a.out_bs, a.out_ds = out.data_ptr(), out.stride(0), out.stride(1)
    a.dz, a.dz_bs, a.dz_ds = dz.data_ptr(), dz.stride(0), dz.stride(1)
    a.x = x.data_ptr()
    a.dout, a.dout_bs, a.dout_ds = dout.data_ptr(), dout.stride(0), dout.stride(1)
    a.du, a.du_bs, a.du_ds = du.data_ptr(), du.stride(0), du.stride(1)
    a.ddelta, a.ddelta_bs, a.ddelta_ds = ddelta.data_ptr(), ddelta.stride(0), ddelta.stride(1)
    a.dA, a.dB, a.dC, a.dD, a.ddelta_bias = (t.data_ptr() for t in (dA, dB, dC, dD, dbias))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(_lib.lib.ss_bwd_noalloc(ctypes.byref(a), stream))
    torch.cuda.synchronize()
    res = [du, ddelta, dA, dB, dC, dD, dbias, dz]
    return res + ([dP, dQ] if P is not None else [])


def _check_against_ss_bwd(inp, dout, dtype):
    """ss_bwd (torch-allocated workspace) is the reference; ss_bwd_noalloc must match it on
    two calls in a row (the second sees the first call's leftovers in the shared array)."""
    from motif_ssm import selective_scan_cuda as ssc
    inp["B"], inp["C"] = inp["B"].unsqueeze(1), inp["C"].unsqueeze(1)
    P, Q = inp.get("P"), inp.get("Q")
    out, x, _ = ssc.fwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], D=inp["D"], z=inp["z"],
                        delta_bias=inp["delta_bias"], P=P, Q=Q, delta_softplus=True)
    dP, dQ = (torch.empty_like(P), torch.empty_like(Q)) if P is not None else (None, None)
    ref = ssc.bwd(inp["u"], inp["delta"], inp["A"], inp["B"], inp["C"], D=inp["D"], z=inp["z"],
                  delta_bias=inp["delta_bias"], P=P, Q=Q, dout=dout, x=x, out=out, dz=None, dP_out=dP,
                  dQ_out=dQ, delta_softplus=True, recompute_out_z=False)
    if P is not None:
        ref = ref + [dP, dQ]
    torch.cuda.synchronize()
    names = ["du", "ddelta", "dA", "dB", "dC", "dD", "ddelta_bias", "dz", "dP", "dQ"]
    t = tol(dtype)
    for call in range(2):
        got = _noalloc_bwd(inp, x, out, dout, True)
        assert len(got) == len(ref)
        for name, g, r in zip(names, got, ref):
            assert_close(g, r, t, t, f"call {call} {name}", scaled=name in SUM_NAMES)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_bwd_matches_ss_bwd_twice(dtype):
    inp, dout = make_scan_inputs(4, 96, 700, 16, dtype, seed=21, device=DEV)
    _check_against_ss_bwd(inp, dout, dtype)


def test_noalloc_bwd_dstate32_uses_the_per_step_scratch():
    """dstate 32 runs two 16-state blocks that carry per-step sums through the scratch
    array's second region; these sizes fit in the array."""
    inp, dout = make_scan_inputs(2, 64, 600, 32, torch.bfloat16, seed=22, device=DEV)
    _check_against_ss_bwd(inp, dout, torch.bfloat16)


def test_noalloc_bwd_motif_pq_uses_the_checkpoint_region():
    """The motif P/Q backward keeps state checkpoints in the scratch array."""
    inp, dout = make_scan_inputs(2, 64, 520, 16, torch.float32, seed=23, device=DEV, pq_rank=4,
                                 pq_per_dim=True, pq_scale=0.3)
    _check_against_ss_bwd(inp, dout, torch.float32)


def test_noalloc_bwd_dstate32_beyond_the_array_is_rejected():
    """dstate > 16 needs scratch growing with batch x dim x seqlen: a call that exceeds the
    array fails with MSS_ERR_WORKSPACE instead of running."""
    from motif_ssm import _lib
    a = _lib.SsBwdArgs()
    a.batch, a.dim, a.seqlen, a.dstate, a.n_groups, a.itype = 8, 2048, 2048, 32, 1, _lib.MSS_BF16
    rc = _lib.lib.ss_bwd_noalloc(ctypes.byref(a), None)
    assert rc == _lib.MSS_ERR_WORKSPACE


def test_noalloc_bwd_rejects_sizes_beyond_its_array():
    from motif_ssm import _lib
    a = _lib.SsBwdArgs()
    a.batch, a.dim, a.seqlen, a.dstate, a.n_groups, a.itype = 64, 8, 1 << 16, 16, 1, _lib.MSS_BF16
    rc = _lib.lib.ss_bwd_noalloc(ctypes.byref(a), None)
    assert rc == _lib.MSS_ERR_WORKSPACE
    assert b"static array" in _lib.lib.ss_last_error()
