"""Drop-in for ``mamba_ssm.ops.triton.selective_state_update.selective_state_update``
(called at ``mamba_ssm/modules/mamba_simplemotif.py:396-399``), on ``libmotif_ssm.so``.

state (batch, dim, dstate) is updated in place; returns out (batch, dim).
"""
import ctypes

import torch

from . import _lib
from ._lib import lib, check
from .selective_scan_cuda import _itype, _ptr, _stream, _req


def selective_state_update(state, x, dt, A, B, C, D=None, z=None, dt_bias=None, dt_softplus=False,
                           state_batch_indices=None):
    """state_batch_indices (batch,): batch row b reads and updates state row
    state_batch_indices[b] (continuous batching); a negative index marks a padding row,
    whose state is untouched and whose output is zero."""
    a, out = _state_args(state, x, dt, A, B, C, D, z, dt_bias, dt_softplus, state_batch_indices)
    with torch.cuda.device(x.device):
        check(lib.ssm_state_update(ctypes.byref(a), _stream(x.device)))
    return out


def dtproj_supported(state, x, dt_in, dt_proj_weight):
    """Whether ``selective_state_update_dtproj`` takes these tensors."""
    r = dt_proj_weight.shape[-1]
    return (state.dim() == 3 and state.shape[-1] == 16 and state.is_contiguous() and r % 8 == 0 and r <= 256
            and dt_proj_weight.is_contiguous() and dt_proj_weight.dtype == x.dtype == dt_in.dtype
            and dt_in.stride(-1) == 1 and (dt_in.stride(0) * dt_in.element_size()) % 16 == 0
            and dt_in.data_ptr() % 16 == 0 and dt_proj_weight.data_ptr() % 16 == 0)


def selective_state_update_dtproj(state, x, dt_in, dt_proj_weight, A, B, C, D=None, z=None, dt_bias=None,
                                  dt_softplus=False):
    """``selective_state_update(state, x, F.linear(dt_in, dt_proj_weight), ...)`` in one kernel
    (the decode step's dt_proj GEMM folded into the state update; dt is rounded to x's dtype
    as the GEMM output is).  dt_in (batch, dt_rank), dt_proj_weight (dim, dt_rank)."""
    batch = x.shape[0]
    dim, rank = dt_proj_weight.shape
    _req(dt_in.shape == (batch, rank), "dt_in must be (batch, dt_rank)")
    a, out = _state_args(state, x, None, A, B, C, D, z, dt_bias, dt_softplus)
    p = _lib.DtProjArgs()
    p.dt_in, p.dt_in_bs, p.weight, p.rank = _ptr(dt_in), dt_in.stride(0), _ptr(dt_proj_weight), rank
    with torch.cuda.device(x.device):
        check(lib.ssm_state_update_dtproj(ctypes.byref(a), ctypes.byref(p), _stream(x.device)))
    return out


def _state_args(state, x, dt, A, B, C, D, z, dt_bias, dt_softplus, state_batch_indices=None):
    if state.dim() != 3:
        raise NotImplementedError("selective_state_update: only the (batch, dim, dstate) layout is supported")
    state_batch, dim, dstate = state.shape
    batch = x.shape[0]
    if state_batch_indices is None:
        _req(state_batch == batch, "state and x must have the same batch size")
    else:
        _req(state_batch_indices.shape == (batch,) and state_batch_indices.is_cuda,
             "state_batch_indices must be a (batch,) CUDA tensor")
        state_batch_indices = state_batch_indices.to(torch.int32).contiguous()
    _req(x.shape == (batch, dim) and (dt is None or dt.shape == (batch, dim)), "x and dt must be (batch, dim)")
    _req(dt is None or x.dtype == dt.dtype, "x and dt must share a dtype")
    _req(A.shape == (dim, dstate) and A.dtype == torch.float32, "A must be float32 (dim, dstate)")
    if B.dim() == 2:
        B = B.unsqueeze(1)
    if C.dim() == 2:
        C = C.unsqueeze(1)
    n_groups = B.shape[1]
    _req(B.shape == (batch, n_groups, dstate) and C.shape == (batch, n_groups, dstate),
         "B and C must be (batch, dstate) or (batch, n_groups, dstate)")
    if B.dtype != x.dtype:
        B = B.to(x.dtype)
    if C.dtype != x.dtype:
        C = C.to(x.dtype)
    if B.stride(-1) != 1:
        B = B.contiguous()
    if C.stride(-1) != 1:
        C = C.contiguous()
    for t in (x, dt):
        _req(t is None or t.stride(-1) == 1, "x and dt must have unit stride in the last dimension")
    if D is not None:
        D = D.float().contiguous()
        _req(D.shape == (dim,), "D must be (dim,)")
    if dt_bias is not None:
        dt_bias = dt_bias.float().contiguous()
        _req(dt_bias.shape == (dim,), "dt_bias must be (dim,)")
    if z is not None:
        _req(z.shape == (batch, dim) and z.stride(-1) == 1, "z must be (batch, dim), unit stride")
        if z.dtype != x.dtype:
            z = z.to(x.dtype)
    out = torch.empty_like(x)
    a = _lib.StateUpdateArgs()
    a.batch, a.dim, a.dstate, a.n_groups = batch, dim, dstate, n_groups
    a.itype, a.stype, a.dt_softplus = _itype(x.dtype), _itype(state.dtype), 1 if dt_softplus else 0
    a.state, a.st_bs, a.st_ds, a.st_ns = _ptr(state), state.stride(0), state.stride(1), state.stride(2)
    a.x, a.x_bs = _ptr(x), x.stride(0)
    if dt is not None:
        a.dt, a.dt_bs = _ptr(dt), dt.stride(0)
    a.A, a.A_ds, a.A_ns = _ptr(A), A.stride(0), A.stride(1)
    a.B, a.B_bs, a.B_gs = _ptr(B), B.stride(0), B.stride(1)
    a.C, a.C_bs, a.C_gs = _ptr(C), C.stride(0), C.stride(1)
    a.D = _ptr(D)
    if z is not None:
        a.z, a.z_bs = _ptr(z), z.stride(0)
    a.dt_bias = _ptr(dt_bias)
    a.out, a.out_bs = _ptr(out), out.stride(0)
    if state_batch_indices is not None:
        a.state_batch_indices, a.state_batch = _ptr(state_batch_indices), state_batch
        a._keep = state_batch_indices  # alive until the launch is queued
    return a, out
