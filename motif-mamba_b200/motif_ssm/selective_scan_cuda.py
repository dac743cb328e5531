"""Drop-in for the reference's ``selective_scan_cuda`` extension (``fwd`` / ``bwd``).

Same argument names, defaults, checks and return lists as the reference binding
(``csrc/selective_scan/selective_scan.cpp:270-413`` forward, ``:415-618`` backward,
``:620-637`` signatures).  Outputs are allocated here with torch (the C side never
allocates) and the work runs in ``libmotif_ssm.so`` on the current CUDA stream.

Differences from the reference, all raising instead of silently diverging:
* complex ``A`` and constant (2-D) ``B`` / ``C`` raise ``NotImplementedError``;
* ``P`` / ``Q`` (the motif low-rank coupling, ``:342-369``) must be contiguous fp32 with
  ``dstate <= 64`` (the reference allows 256); ``gamma`` is checked and, as in the
  reference's dense P/Q kernels, not used;
* ``dstate`` up to ``MAX_DSTATE`` (256, the reference's limit; above 64 a row's states are
  spread over 8 or 16 lanes in the forward and the backward runs blocks of 16 states);
* ``x`` holds one (decay, state) pair per ``CHUNK_LEN`` = 256 steps instead of 2048;
  ``x[:, :, -1, 1::2]`` is still the final state and ``bwd`` expects this ``x``.
"""
import ctypes

import torch

from . import _lib
from ._lib import lib, check

CHUNK_LEN = _lib.CHUNK_LEN

_ITYPE = {torch.float32: _lib.MSS_F32, torch.float16: _lib.MSS_F16, torch.bfloat16: _lib.MSS_BF16}


def _itype(dtype):
    try:
        return _ITYPE[dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from None


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _req(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _check_shape(t, *shape, name="tensor"):
    _req(tuple(t.shape) == tuple(shape), f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")


def _check_pq(P, Q, gamma, dim, dstate):
    """Shape rules of the reference binding (``selective_scan.cpp:342-369``)."""
    _req(P is None or Q is not None, "Q must be provided when P is provided")
    _req(Q is None or P is not None, "P must be provided when Q is provided")
    if P is not None:
        _req(P.is_cuda and Q.is_cuda, "P and Q must be CUDA tensors")
        _req(P.dim() == Q.dim() and P.dim() in (2, 3), "P/Q must be 2D or 3D with same rank")
        if P.dim() == 2:
            _req(P.size(0) == dstate and Q.size(1) == dstate and P.size(1) == Q.size(0),
                 "Expect P(dstate, r), Q(r, dstate)")
        else:
            _req(P.size(0) == dim and Q.size(0) == dim, "P/Q dim mismatch")
            _req(P.size(1) == dstate and Q.size(2) == dstate and P.size(2) == Q.size(1),
                 "Expect P(dim, dstate, r), Q(dim, r, dstate)")
        _req(P.size(-1) <= 8, "Current dense CUDA forward supports pq_rank <= 8")
        _req(P.dtype == torch.float32 and Q.dtype == torch.float32, "P and Q must be float32")
        _req(P.is_contiguous() and Q.is_contiguous(), "P and Q must be contiguous")
        if dstate > 64:
            raise NotImplementedError("selective_scan_cuda: the P/Q coupling supports dstate <= 64 in this library")
    if gamma is not None:
        _req(gamma.is_cuda, "gamma must be CUDA tensor")
        _req(gamma.dim() in (1, 2), "gamma must be 1D or 2D")
        if gamma.dim() == 1:
            _req(gamma.size(0) == dstate, "gamma(1D) shape must be (dstate,)")
        else:
            _req(gamma.size(0) == dim and gamma.size(1) == dstate, "gamma(2D) shape must be (dim, dstate)")


def _fill_pq(a, P, Q):
    if P is not None:
        a.P, a.Q = _ptr(P), _ptr(Q)
        a.pq_rank = P.size(-1)
        a.pq_per_dim = 1 if P.dim() == 3 else 0


def _check_common(u, delta, A, B, C, D, z, delta_bias, P, Q, gamma):
    if A.is_complex():
        raise NotImplementedError("selective_scan_cuda: complex A is not supported by this library")
    _req(u.dtype in _ITYPE, "u must be float32, float16 or bfloat16")
    _req(A.dtype == torch.float32, "A must be float32")
    if B.dim() < 3 or C.dim() < 3:
        raise NotImplementedError("selective_scan_cuda: constant (2-D) B / C are not supported by this library")
    _req(delta.dtype == u.dtype, "delta must have the dtype of u")
    _req(B.dtype == u.dtype and C.dtype == u.dtype, "variable B / C must have the dtype of u")
    for name, t in (("u", u), ("delta", delta), ("A", A), ("B", B), ("C", C)):
        _req(t.is_cuda, f"{name} must be a CUDA tensor")
    _req(u.stride(-1) == 1 or u.size(-1) == 1, "u must have unit stride in the last dimension")
    _req(delta.stride(-1) == 1 or delta.size(-1) == 1, "delta must have unit stride in the last dimension")
    batch, dim, seqlen = u.shape
    dstate = A.size(1)
    n_groups = B.size(1)
    _req(dstate <= 256, "selective_scan only supports state dimension <= 256")
    _check_shape(u, batch, dim, seqlen, name="u")
    _check_shape(delta, batch, dim, seqlen, name="delta")
    _check_shape(A, dim, dstate, name="A")
    _check_shape(B, batch, n_groups, dstate, seqlen, name="B")
    _check_shape(C, batch, n_groups, dstate, seqlen, name="C")
    _req(B.stride(-1) == 1 or B.size(-1) == 1, "B must have unit stride in the last dimension")
    _req(C.stride(-1) == 1 or C.size(-1) == 1, "C must have unit stride in the last dimension")
    for name, t in (("D", D), ("delta_bias", delta_bias)):
        if t is not None:
            _req(t.dtype == torch.float32, f"{name} must be float32")
            _req(t.is_cuda, f"{name} must be a CUDA tensor")
            _req(t.stride(-1) == 1 or t.size(-1) == 1, f"{name} must have unit stride")
            _check_shape(t, dim, name=name)
    if z is not None:
        _req(z.dtype == u.dtype, "z must have the dtype of u")
        _req(z.is_cuda, "z must be a CUDA tensor")
        _req(z.stride(-1) == 1 or z.size(-1) == 1, "z must have unit stride in the last dimension")
        _check_shape(z, batch, dim, seqlen, name="z")
    _check_pq(P, Q, gamma, dim, dstate)
    return batch, dim, seqlen, dstate, n_groups


def _fill_common(a, u, delta, A, B, C, D, z, delta_bias, sizes, softplus):
    batch, dim, seqlen, dstate, n_groups = sizes
    a.batch, a.dim, a.seqlen, a.dstate, a.n_groups = batch, dim, seqlen, dstate, n_groups
    a.itype = _itype(u.dtype)
    a.delta_softplus = 1 if softplus else 0
    a.u, a.u_bs, a.u_ds = _ptr(u), u.stride(0), u.stride(1)
    a.delta, a.delta_bs, a.delta_ds = _ptr(delta), delta.stride(0), delta.stride(1)
    a.A, a.A_ds, a.A_ns = _ptr(A), A.stride(0), A.stride(1)
    a.B, a.B_bs, a.B_gs, a.B_ns = _ptr(B), B.stride(0), B.stride(1), B.stride(2)
    a.C, a.C_bs, a.C_gs, a.C_ns = _ptr(C), C.stride(0), C.stride(1), C.stride(2)
    if D is not None:
        a.D, a.D_s = _ptr(D), D.stride(0)
    if delta_bias is not None:
        a.delta_bias, a.delta_bias_s = _ptr(delta_bias), delta_bias.stride(0)
    if z is not None:
        a.z, a.z_bs, a.z_ds = _ptr(z), z.stride(0), z.stride(1)


def n_chunks(seqlen):
    return (seqlen + CHUNK_LEN - 1) // CHUNK_LEN


def fwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, P=None, Q=None, gamma=None,
        delta_softplus=False, initial_state=None):
    """Selective-scan forward.  Returns ``[out, x]`` plus ``out_z`` when ``z`` is given.

    ``initial_state`` (an addition of this library; the reference always starts from zero):
    fp32 contiguous (batch, dim, dstate), the state before the first step, so that a sequence
    can be scanned in pieces -- ``x[:, :, -1, 1::2]`` of one piece starts the next.  Forward
    only (``bwd`` assumes a zero initial state) and not with P / Q."""
    sizes = _check_common(u, delta, A, B, C, D, z, delta_bias, P, Q, gamma)
    batch, dim, seqlen, dstate, n_groups = sizes
    if initial_state is not None:
        _req(P is None, "initial_state is not supported with P / Q")
        _req(initial_state.dtype == torch.float32 and initial_state.is_cuda and initial_state.is_contiguous(),
             "initial_state must be a contiguous float32 CUDA tensor")
        _check_shape(initial_state, batch, dim, dstate, name="initial_state")
    out = torch.empty_like(delta)
    x = torch.empty(batch, dim, n_chunks(seqlen), 2 * dstate, device=u.device, dtype=torch.float32)
    out_z = torch.empty_like(z) if z is not None else None
    a = _lib.SsFwdArgs()
    _fill_common(a, u, delta, A, B, C, D, z, delta_bias, sizes, delta_softplus)
    _fill_pq(a, P, Q)
    a.out, a.out_bs, a.out_ds = _ptr(out), out.stride(0), out.stride(1)
    if z is not None:
        a.out_z, a.out_z_bs, a.out_z_ds = _ptr(out_z), out_z.stride(0), out_z.stride(1)
    a.x = _ptr(x)
    a.h0 = _ptr(initial_state)
    ws_bytes = ctypes.c_int64(0)
    check(lib.ss_fwd_workspace_size(ctypes.byref(a), ctypes.byref(ws_bytes)))
    ws = None
    if ws_bytes.value > 0:
        ws = torch.empty(ws_bytes.value, device=u.device, dtype=torch.uint8)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws_bytes.value
    with torch.cuda.device(u.device):
        check(lib.ss_fwd(ctypes.byref(a), _stream(u.device)))
    return [out, x] + ([out_z] if z is not None else [])


def bwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, P=None, Q=None, gamma=None,
        dout=None, x=None, out=None, dz=None, dP_out=None, dQ_out=None, delta_softplus=False,
        recompute_out_z=False):
    """Selective-scan backward.

    Returns ``[du, ddelta, dA, dB, dC, dD, ddelta_bias]`` plus ``dz`` when ``z`` is
    given plus ``out_z`` when ``recompute_out_z``.  A caller-provided ``dz`` is written
    in place (``selective_scan_interface.py:593-603`` passes a view into ``dxz``).  With
    ``P`` / ``Q`` the gradients of the coupling go to ``dP_out`` / ``dQ_out`` (fp32, the
    shapes of P and Q, overwritten; allocated and dropped when not given), as in
    ``selective_scan.cpp:579-590``.
    """
    sizes = _check_common(u, delta, A, B, C, D, z, delta_bias, P, Q, gamma)
    batch, dim, seqlen, dstate, n_groups = sizes
    _req(dout is not None, "dout must be given")
    _req(dout.dtype == u.dtype and dout.is_cuda, "dout must be a CUDA tensor with the dtype of u")
    _req(dout.stride(-1) == 1 or dout.size(-1) == 1, "dout must have unit stride in the last dimension")
    _check_shape(dout, batch, dim, seqlen, name="dout")
    nc = n_chunks(seqlen)
    if x is not None:
        _req(x.dtype == torch.float32 and x.is_cuda and x.is_contiguous(), "x must be a contiguous float32 CUDA tensor")
        _req(tuple(x.shape) == (batch, dim, nc, 2 * dstate),
             f"x must have shape {(batch, dim, nc, 2 * dstate)} (chunk length {CHUNK_LEN}), got {tuple(x.shape)}")
    else:
        _req(nc <= 1 or P is not None, "x (the forward's chunk states) is required when seqlen > %d" % CHUNK_LEN)
    if z is not None:
        _req(out is not None, "out must be given with z")
        _req(out.dtype == u.dtype and out.is_cuda, "out must be a CUDA tensor with the dtype of u")
        _req(out.stride(-1) == 1 or out.size(-1) == 1, "out must have unit stride in the last dimension")
        _check_shape(out, batch, dim, seqlen, name="out")
        if dz is not None:
            _req(dz.dtype == u.dtype and dz.is_cuda, "dz must be a CUDA tensor with the dtype of u")
            _req(dz.stride(-1) == 1 or dz.size(-1) == 1, "dz must have unit stride in the last dimension")
            _check_shape(dz, batch, dim, seqlen, name="dz")
        else:
            dz = torch.empty_like(z)
    du = torch.empty_like(u)
    ddelta = torch.empty_like(delta)
    dA = torch.empty_like(A)
    dB = torch.empty(B.shape, device=B.device, dtype=B.dtype)
    dC = torch.empty(C.shape, device=C.device, dtype=C.dtype)
    dD = torch.empty_like(D) if D is not None else None
    ddelta_bias = torch.empty_like(delta_bias) if delta_bias is not None else None
    out_z = torch.empty_like(out) if (recompute_out_z and z is not None) else None
    if P is not None:
        dP_out = torch.empty_like(P) if dP_out is None else dP_out
        dQ_out = torch.empty_like(Q) if dQ_out is None else dQ_out
        _req(dP_out.is_cuda and dQ_out.is_cuda, "dP_out and dQ_out must be CUDA tensors")
        _req(dP_out.dtype == torch.float32 and dQ_out.dtype == torch.float32, "dP_out and dQ_out must be float32")
        _req(dP_out.shape == P.shape, "dP_out shape mismatch")
        _req(dQ_out.shape == Q.shape, "dQ_out shape mismatch")
        _req(dP_out.is_contiguous() and dQ_out.is_contiguous(), "dP_out and dQ_out must be contiguous")

    a = _lib.SsBwdArgs()
    _fill_common(a, u, delta, A, B, C, D, z, delta_bias, sizes, delta_softplus)
    a.recompute_out_z = 1 if out_z is not None else 0
    _fill_pq(a, P, Q)
    if P is not None:
        a.dP, a.dQ = _ptr(dP_out), _ptr(dQ_out)
    if z is not None:
        a.out, a.out_bs, a.out_ds = _ptr(out), out.stride(0), out.stride(1)
        a.dz, a.dz_bs, a.dz_ds = _ptr(dz), dz.stride(0), dz.stride(1)
    if out_z is not None:
        a.out_z, a.out_z_bs, a.out_z_ds = _ptr(out_z), out_z.stride(0), out_z.stride(1)
    a.x = _ptr(x) if x is not None else _ptr(u)  # never read when seqlen <= CHUNK_LEN or with P
    a.dout, a.dout_bs, a.dout_ds = _ptr(dout), dout.stride(0), dout.stride(1)
    a.du, a.du_bs, a.du_ds = _ptr(du), du.stride(0), du.stride(1)
    a.ddelta, a.ddelta_bs, a.ddelta_ds = _ptr(ddelta), ddelta.stride(0), ddelta.stride(1)
    a.dA, a.dB, a.dC = _ptr(dA), _ptr(dB), _ptr(dC)
    a.dD, a.ddelta_bias = _ptr(dD), _ptr(ddelta_bias)
    ws_bytes = ctypes.c_int64(0)
    check(lib.ss_bwd_workspace_size(ctypes.byref(a), ctypes.byref(ws_bytes)))
    ws = None
    if ws_bytes.value > 0:
        ws = torch.empty(ws_bytes.value, device=u.device, dtype=torch.uint8)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws_bytes.value
    with torch.cuda.device(u.device):
        check(lib.ss_bwd(ctypes.byref(a), _stream(u.device)))
    res = [du, ddelta, dA, dB, dC, dD, ddelta_bias]
    if z is not None:
        res.append(dz)
    if out_z is not None:
        res.append(out_z)
    return res
