"""``selective_scan_fn`` and ``mamba_inner_fn`` on the sm_100a kernels.

Same call signatures and autograd contract as the reference's
``mamba_ssm/ops/selective_scan_interface.py`` (``selective_scan_fn`` :237-259,
``SelectiveScanFn`` :24-91, ``mamba_inner_fn`` :648-656, ``MambaInnerFn`` :454-645):

* ``selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None,
  delta_softplus=False, return_last_state=False)`` returns ``out`` (z-gated when z is
  given) and optionally ``last_state`` (batch, dim, dstate) fp32, which carries no
  gradient;
* ``mamba_inner_fn(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight,
  out_proj_weight, out_proj_bias, A, B=None, C=None, D=None, delta_bias=None,
  B_proj_bias=None, C_proj_bias=None, delta_softplus=True, checkpoint_lvl=1)`` fuses
  conv1d+SiLU -> x_proj -> dt_proj -> scan -> out_proj; with ``checkpoint_lvl=1`` the
  backward recomputes the conv output and delta instead of saving them.

The GEMMs (x_proj, dt_proj, out_proj and their gradients) are cuBLAS calls through
torch; the conv, the scan and its backward are this library's kernels.
"""
import torch
import torch.nn.functional as F

from . import selective_scan_cuda
from .causal_conv1d import causal_conv1d_bwd_function, causal_conv1d_fwd_function


def _last_dim_contig(t):
    return t if (t is None or t.stride(-1) == 1) else t.contiguous()


class SelectiveScanFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                return_last_state=False):
        u, delta, B, C, z = (_last_dim_contig(t) for t in (u, delta, B, C, z))
        if D is not None:
            D = D.contiguous()
        ctx.squeeze_B = B.dim() == 3
        ctx.squeeze_C = C.dim() == 3
        if ctx.squeeze_B:
            B = B.unsqueeze(1)
        if ctx.squeeze_C:
            C = C.unsqueeze(1)
        out, x, *rest = selective_scan_cuda.fwd(u, delta, A, B, C, D=D, z=z, delta_bias=delta_bias,
                                                delta_softplus=delta_softplus)
        ctx.delta_softplus = delta_softplus
        ctx.has_z = z is not None
        last_state = x[:, :, -1, 1::2]
        if ctx.has_z:
            ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, x, out)
            result = rest[0]
        else:
            ctx.save_for_backward(u, delta, A, B, C, D, delta_bias, x)
            result = out
        ctx.mark_non_differentiable(last_state)
        return (result, last_state) if return_last_state else result

    @staticmethod
    def backward(ctx, dout, *unused):
        if ctx.has_z:
            u, delta, A, B, C, D, z, delta_bias, x, out = ctx.saved_tensors
        else:
            u, delta, A, B, C, D, delta_bias, x = ctx.saved_tensors
            z = out = None
        dout = _last_dim_contig(dout)
        du, ddelta, dA, dB, dC, dD, ddelta_bias, *rest = selective_scan_cuda.bwd(
            u, delta, A, B, C, D=D, z=z, delta_bias=delta_bias, dout=dout, x=x, out=out, dz=None,
            delta_softplus=ctx.delta_softplus, recompute_out_z=False)
        dz = rest[0] if ctx.has_z else None
        if ctx.squeeze_B:
            dB = dB.squeeze(1)
        if ctx.squeeze_C:
            dC = dC.squeeze(1)
        return (du, ddelta, dA, dB, dC, dD if D is not None else None, dz,
                ddelta_bias if delta_bias is not None else None, None, None)


class SelectiveScanPQFn(torch.autograd.Function):
    """The scan with the motif low-rank coupling ``h += dt * P (Q h_prev)``
    (``selective_scan_interface.py:94-219``).  Unlike the reference's dense kernel this one
    also takes ``z`` (the reference sends that case to its per-step torch loop,
    ``:262-350``), and ``dP`` / ``dQ`` are the exact gradients from the backward kernel (the
    reference's default recomputes them by autograd through that loop).  ``gamma`` is
    accepted and unused, as in the reference's forward."""

    @staticmethod
    def forward(ctx, u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                return_last_state=False, P=None, Q=None, gamma=None):
        if A.is_complex():
            raise NotImplementedError("P/Q path supports real A only")
        if P is None or Q is None:
            raise ValueError("P and Q must both be provided")
        if gamma is not None and gamma.requires_grad:
            raise NotImplementedError("the P/Q backward does not return dgamma")
        u, delta, B, C, z = (_last_dim_contig(t) for t in (u, delta, B, C, z))
        if D is not None:
            D = D.contiguous()
        ctx.squeeze_B = B.dim() == 3
        ctx.squeeze_C = C.dim() == 3
        if ctx.squeeze_B:
            B = B.unsqueeze(1)
        if ctx.squeeze_C:
            C = C.unsqueeze(1)
        ctx.P_dtype, ctx.Q_dtype = P.dtype, Q.dtype
        P32 = P.detach().float().contiguous()
        Q32 = Q.detach().float().contiguous()
        out, x, *rest = selective_scan_cuda.fwd(u, delta, A, B, C, D=D, z=z, delta_bias=delta_bias,
                                                P=P32, Q=Q32, gamma=gamma, delta_softplus=delta_softplus)
        ctx.delta_softplus = delta_softplus
        ctx.has_z = z is not None
        ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, P32, Q32, out if ctx.has_z else None)
        last_state = x[:, :, -1, 1::2]
        ctx.mark_non_differentiable(last_state)
        result = rest[0] if ctx.has_z else out
        return (result, last_state) if return_last_state else result

    @staticmethod
    def backward(ctx, dout, *unused):
        u, delta, A, B, C, D, z, delta_bias, P32, Q32, out = ctx.saved_tensors
        dout = _last_dim_contig(dout)
        dP = torch.empty_like(P32)
        dQ = torch.empty_like(Q32)
        du, ddelta, dA, dB, dC, dD, ddelta_bias, *rest = selective_scan_cuda.bwd(
            u, delta, A, B, C, D=D, z=z, delta_bias=delta_bias, P=P32, Q=Q32, dout=dout, x=None, out=out,
            dz=None, dP_out=dP, dQ_out=dQ, delta_softplus=ctx.delta_softplus, recompute_out_z=False)
        dz = rest[0] if ctx.has_z else None
        if ctx.squeeze_B:
            dB = dB.squeeze(1)
        if ctx.squeeze_C:
            dC = dC.squeeze(1)
        return (du, ddelta, dA, dB, dC, dD if D is not None else None, dz,
                ddelta_bias if delta_bias is not None else None, None, None,
                dP.to(ctx.P_dtype), dQ.to(ctx.Q_dtype), None)


def selective_scan_fn(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                      return_last_state=False, P=None, Q=None, gamma=None):
    """If ``return_last_state`` is True returns ``(out, last_state)``; ``last_state`` is
    (batch, dim, dstate) and receives no gradient.  ``P`` / ``Q`` switch on the motif
    low-rank coupling (``selective_scan_interface.py:237-259``)."""
    if P is not None or Q is not None or gamma is not None:
        return SelectiveScanPQFn.apply(u, delta, A, B, C, D, z, delta_bias, delta_softplus, return_last_state,
                                       P, Q, gamma)
    return SelectiveScanFn.apply(u, delta, A, B, C, D, z, delta_bias, delta_softplus, return_last_state)


def _rms_along(t, weight, eps, dim):
    """RMSNorm of ``t`` along ``dim`` (fp32 math, output in t's dtype, contiguous):
    t * rsqrt(mean(t^2) + eps) * weight -- the reference's ``rms_norm_forward`` over the rows
    it rearranges to (``selective_scan_interface.py:217-234, 521-532``)."""
    tf = t.float()
    shape = [1] * t.dim()
    shape[dim] = -1
    y = tf * torch.rsqrt(tf.pow(2).mean(dim=dim, keepdim=True) + eps) * weight.float().view(shape)
    return y.to(t.dtype).contiguous()


def selective_scan_full_matrix_cuda(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                                   return_last_state=False, P=None, Q=None, gamma=None):
    """The reference's full-matrix P/Q entry point (``selective_scan_interface.py:262-350``):
    same arguments, checks and results, computed by the P/Q kernels instead of a per-step
    torch loop (gradients included, ``gamma`` unused as there)."""
    if P is None or Q is None:
        raise ValueError("P and Q must both be provided for full-matrix path")
    if A.is_complex():
        raise NotImplementedError("Full-matrix P/Q path currently supports real A only")
    if not all(t.is_cuda for t in (u, delta, A, B, C, P, Q)):
        raise ValueError("Full-matrix path requires CUDA tensors")
    return SelectiveScanPQFn.apply(u, delta, A, B, C, D, z, delta_bias, delta_softplus, return_last_state, P, Q,
                                   gamma)


def rms_norm_forward(x, weight, bias, eps=1e-6, is_rms_norm=True):
    """The reference's helper (``selective_scan_interface.py:217-234``): normalises the last
    dimension of x (no autograd through it, as there)."""
    from .layer_norm import _layer_norm_fwd
    x = x if x.stride(-1) == 1 else x.contiguous()
    return _layer_norm_fwd(x, weight.contiguous(), bias.contiguous() if bias is not None else None, eps, None,
                           residual_dtype=None, is_rms_norm=is_rms_norm)[0]


def _bcast(w, batch):
    """A weight matrix as a (batch, m, k) operand of a batched product (batch stride 0, no copy)."""
    return w.unsqueeze(0).expand(batch, -1, -1)


class MambaInnerFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight, out_proj_weight,
                out_proj_bias, A, B=None, C=None, D=None, delta_bias=None, B_proj_bias=None,
                C_proj_bias=None, delta_softplus=True, checkpoint_lvl=1, b_rms_weight=None, c_rms_weight=None,
                dt_rms_weight=None, b_c_dt_rms_eps=1e-6):
        assert checkpoint_lvl in (0, 1)
        if A.is_complex():
            raise NotImplementedError("mamba_inner_fn: complex A is not supported by this library")
        L = xz.shape[-1]
        rank = delta_proj_weight.shape[1]
        d_state = A.shape[-1]
        if torch.is_autocast_enabled():
            dt = torch.get_autocast_dtype("cuda")
            x_proj_weight = x_proj_weight.to(dt)
            delta_proj_weight = delta_proj_weight.to(dt)
            out_proj_weight = out_proj_weight.to(dt)
            out_proj_bias = out_proj_bias.to(dt) if out_proj_bias is not None else None
        xz = _last_dim_contig(xz)
        w_conv = conv1d_weight.reshape(conv1d_weight.shape[0], conv1d_weight.shape[-1])
        x, z = xz.chunk(2, dim=1)
        conv1d_bias = conv1d_bias.contiguous() if conv1d_bias is not None else None
        conv_out = causal_conv1d_fwd_function(x, w_conv, conv1d_bias, None, None, None, True)
        # x_proj as a batched product in the scan's (b, d, l) layout: x_dbl is (b, dt_rank + 2n, l),
        # so delta (dt_proj), B and C come out with l unit-stride and need no transpose copies
        # (B / C are strided views of x_dbl's rows).
        x_dbl = torch.bmm(_bcast(x_proj_weight, conv_out.shape[0]), conv_out)
        delta = torch.bmm(_bcast(delta_proj_weight, conv_out.shape[0]), x_dbl[:, :rank])
        ctx.is_variable_B = B is None
        ctx.is_variable_C = C is None
        ctx.B_proj_bias_is_None = B_proj_bias is None
        ctx.C_proj_bias_is_None = C_proj_bias is None
        if B is None:
            B = x_dbl[:, rank:rank + d_state]
            if B_proj_bias is not None:
                B = B + B_proj_bias.to(B.dtype).unsqueeze(-1)
            B = B.unsqueeze(1)
        else:
            B = _last_dim_contig(B)
        if C is None:
            C = x_dbl[:, rank + d_state:rank + 2 * d_state]
            if C_proj_bias is not None:
                C = C + C_proj_bias.to(C.dtype).unsqueeze(-1)
            C = C.unsqueeze(1)
        else:
            C = _last_dim_contig(C)
        if D is not None:
            D = D.contiguous()
        # optional RMSNorm of B / C over dstate and of delta over channels, applied to the scan
        # inputs as the reference does (selective_scan_interface.py:521-532)
        if b_rms_weight is not None:
            B = _rms_along(B, b_rms_weight, b_c_dt_rms_eps, dim=2)
        if c_rms_weight is not None:
            C = _rms_along(C, c_rms_weight, b_c_dt_rms_eps, dim=2)
        if dt_rms_weight is not None:
            delta = _rms_along(delta, dt_rms_weight, b_c_dt_rms_eps, dim=1)
        ctx.rms = (b_rms_weight, c_rms_weight, dt_rms_weight, b_c_dt_rms_eps)
        out, scan_x, out_z = selective_scan_cuda.fwd(conv_out, delta, A, B, C, D=D, z=z, delta_bias=delta_bias,
                                                     delta_softplus=delta_softplus)
        ctx.delta_softplus = delta_softplus
        ctx.out_proj_bias_is_None = out_proj_bias is None
        ctx.checkpoint_lvl = checkpoint_lvl
        if checkpoint_lvl >= 1:
            conv_out, delta = None, None
        ctx.save_for_backward(xz, w_conv, conv1d_bias, x_dbl, x_proj_weight, delta_proj_weight, out_proj_weight,
                              conv_out, delta, A, B, C, D, delta_bias, scan_x, out)
        return F.linear(out_z.transpose(1, 2), out_proj_weight, out_proj_bias)

    @staticmethod
    def backward(ctx, dout):
        (xz, w_conv, conv1d_bias, x_dbl, x_proj_weight, delta_proj_weight, out_proj_weight, conv_out, delta,
         A, B, C, D, delta_bias, scan_x, out) = ctx.saved_tensors
        L = xz.shape[-1]
        batch = xz.shape[0]
        rank = delta_proj_weight.shape[1]
        d_state = A.shape[-1]
        x, z = xz.chunk(2, dim=1)
        dout = _last_dim_contig(dout)
        if ctx.checkpoint_lvl == 1:
            conv_out = causal_conv1d_fwd_function(x, w_conv, conv1d_bias, None, None, None, True)
            delta = torch.bmm(_bcast(delta_proj_weight, batch), x_dbl[:, :rank])
            # the reference's recompute (selective_scan_interface.py:572-589): delta is normalised
            # again from the projection, and the SAVED (already normalised) B / C are normalised
            # a second time; both are kept so that the gradients equal the reference's
            b_rms, c_rms, dt_rms, eps = ctx.rms
            if dt_rms is not None:
                delta = _rms_along(delta, dt_rms, eps, dim=1)
            if b_rms is not None:
                B = _rms_along(B, b_rms, eps, dim=2)
            if c_rms is not None:
                C = _rms_along(C, c_rms, eps, dim=2)
        dxz = torch.empty_like(xz)
        dx, dz = dxz.chunk(2, dim=1)
        dout2 = dout.reshape(-1, dout.shape[-1]).t()              # (e, b*l)
        dout_y = (out_proj_weight.t() @ dout2).view(-1, batch, L).transpose(0, 1)
        dconv_out, ddelta, dA, dB, dC, dD, ddelta_bias, dz, out_z = selective_scan_cuda.bwd(
            conv_out, delta, A, B, C, D=D, z=z, delta_bias=delta_bias, dout=dout_y, x=scan_x, out=out, dz=dz,
            delta_softplus=ctx.delta_softplus, recompute_out_z=True)
        out_z_rows = out_z.transpose(0, 1).reshape(out_z.shape[1], -1)  # (d, b*l)
        dout_proj_weight = dout2 @ out_z_rows.t()
        dout_proj_bias = dout.sum(dim=(0, 1)) if not ctx.out_proj_bias_is_None else None
        # x_dbl is (b, dt_rank + 2n, l): dB / dC are its gradient rows as they come from the scan
        dx_dbl = torch.empty_like(x_dbl)
        dB_proj_bias = dC_proj_bias = None
        if ctx.is_variable_B:
            dB_proj_bias = dB.sum(dim=(0, 1, 3)) if not ctx.B_proj_bias_is_None else None
            dx_dbl[:, rank:rank + d_state] = dB.squeeze(1)
            dB = None
        if ctx.is_variable_C:
            dC_proj_bias = dC.sum(dim=(0, 1, 3)) if not ctx.C_proj_bias_is_None else None
            dx_dbl[:, rank + d_state:rank + 2 * d_state] = dC.squeeze(1)
            dC = None
        ddelta_proj_weight = torch.bmm(ddelta, x_dbl[:, :rank].transpose(1, 2)).sum(0)
        torch.bmm(_bcast(delta_proj_weight.t(), batch), ddelta, out=dx_dbl[:, :rank])
        dx_proj_weight = torch.bmm(dx_dbl, conv_out.transpose(1, 2)).sum(0)
        dconv_out = torch.baddbmm(dconv_out, _bcast(x_proj_weight.t(), batch), dx_dbl)
        dx, dconv_w, dconv_b, _ = causal_conv1d_bwd_function(x, w_conv, conv1d_bias, dconv_out, None, None, None,
                                                             dx, False, True)
        dconv_b = dconv_b if conv1d_bias is not None else None
        dconv_w = dconv_w.unsqueeze(1)
        return (dxz, dconv_w, dconv_b, dx_proj_weight, ddelta_proj_weight, dout_proj_weight, dout_proj_bias,
                dA, dB, dC, dD, ddelta_bias if delta_bias is not None else None, dB_proj_bias, dC_proj_bias,
                None, None, None, None, None, None)


def mamba_inner_fn(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight, out_proj_weight,
                   out_proj_bias, A, B=None, C=None, D=None, delta_bias=None, B_proj_bias=None,
                   C_proj_bias=None, delta_softplus=True, checkpoint_lvl=1, b_rms_weight=None,
                   c_rms_weight=None, dt_rms_weight=None, b_c_dt_rms_eps=1e-6):
    """With ``b_rms_weight`` / ``c_rms_weight`` / ``dt_rms_weight`` the scan's B, C (over
    dstate) and delta (over channels) are RMS-normalised first.  As in the reference's
    backward (``selective_scan_interface.py:597-645``), the gradients of B, C and delta pass
    to x_proj / dt_proj as if the normalisation were the identity, and the norm weights get
    no gradient."""
    return MambaInnerFn.apply(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight, out_proj_weight,
                              out_proj_bias, A, B, C, D, delta_bias, B_proj_bias, C_proj_bias, delta_softplus,
                              checkpoint_lvl, b_rms_weight, c_rms_weight, dt_rms_weight, b_c_dt_rms_eps)
