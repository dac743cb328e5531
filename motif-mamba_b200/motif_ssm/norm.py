"""Fused residual add + RMSNorm of the pre-norm stack on ``libmotif_ssm.so``.

The reference runs Add -> Norm as one fused call (``layer_norm_fn(..., residual=residual,
prenorm=True, residual_in_fp32=...)``, ``mamba_ssm/models/mixer_seq_simple.py:190-211``):

    residual = x + residual        (fp32 when residual_in_fp32)
    out      = residual * rsqrt(mean(residual^2) + eps) * weight       (x's dtype)

``add_rms_norm`` does both in one kernel.  Its backward is plain torch (fp32): it runs once
per layer per training step and is not on the scan's hot path.
"""
import ctypes

import torch

from . import _lib
from ._lib import lib, check
from .selective_scan_cuda import _itype, _ptr, _stream


def supported(x, residual, weight):
    """Whether the kernel takes these tensors (else use the torch expression)."""
    D = x.shape[-1]
    ok = (x.is_cuda and D % 8 == 0 and D <= 4096 and x.stride(-1) == 1 and weight.is_contiguous()
          and weight.dtype in (torch.float32, x.dtype) and x.dtype in (torch.float32, torch.float16, torch.bfloat16))
    if residual is not None:
        ok = ok and residual.shape == x.shape and residual.stride(-1) == 1 and residual.dtype in (torch.float32, x.dtype)
    return ok


def _launch(x2, r2, weight, eps, rdtype):
    rows, D = x2.shape
    out = torch.empty_like(x2)
    rout = torch.empty(rows, D, dtype=rdtype, device=x2.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x2.device)
    a = _lib.AddRmsNormArgs()
    a.rows, a.dim = rows, D
    a.itype = _itype(x2.dtype)
    a.rin_type = _itype(r2.dtype) if r2 is not None else a.itype
    a.rout_type, a.wtype = _itype(rdtype), _itype(weight.dtype)
    a.x, a.x_rs = _ptr(x2), x2.stride(0)
    if r2 is not None:
        a.residual_in, a.rin_rs = _ptr(r2), r2.stride(0)
    a.residual_out, a.rout_rs = _ptr(rout), rout.stride(0)
    a.weight = _ptr(weight)
    a.out, a.out_rs = _ptr(out), out.stride(0)
    a.rstd = _ptr(rstd)
    a.eps = float(eps)
    with torch.cuda.device(x2.device):
        check(lib.add_rms_norm(ctypes.byref(a), _stream(x2.device)))
    return out, rout, rstd


class AddRmsNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, residual, weight, eps, residual_in_fp32):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        r2 = residual.reshape(-1, shape[-1]) if residual is not None else None
        rdtype = torch.float32 if residual_in_fp32 else (residual.dtype if residual is not None else x.dtype)
        out, rout, rstd = _launch(x2, r2, weight, eps, rdtype)
        ctx.save_for_backward(rout, rstd, weight)
        ctx.has_res, ctx.x_dtype = residual is not None, x.dtype
        ctx.res_dtype = residual.dtype if residual is not None else None
        return out.view(shape), rout.view(shape)

    @staticmethod
    def backward(ctx, dout, dres):
        rout, rstd, weight = ctx.saved_tensors
        D = rout.shape[-1]
        r = rout.reshape(-1, D).float()
        rs = rstd.unsqueeze(-1)
        gw = dout.reshape(-1, D).float() * weight.float()
        dr = rs * gw - r * rs.pow(3) * (r * gw).mean(-1, keepdim=True)
        if dres is not None:
            dr = dr + dres.reshape(-1, D).float()
        dw = (dout.reshape(-1, D).float() * r * rs).sum(0).to(weight.dtype)
        dx = dr.to(ctx.x_dtype).view(dout.shape)
        dresid = dr.to(ctx.res_dtype).view(dout.shape) if ctx.has_res else None
        return dx, dresid, dw, None, None


def add_rms_norm(x, residual, weight, eps=1e-5, residual_in_fp32=True):
    """Returns (normed, new_residual).  ``residual`` may be None (first layer)."""
    return AddRmsNormFn.apply(x, residual, weight, eps, residual_in_fp32)
