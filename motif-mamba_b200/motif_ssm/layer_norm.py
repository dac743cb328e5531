"""Stand-in for ``mamba_ssm.ops.triton.layer_norm`` (a Triton module the reference imports,
``selective_scan_interface.py:19``, ``mixer_seq_simple.py``, whose source the export lacks).

RMSNorm (with or without a residual add) runs on this library's fused ``add_rms_norm``
kernel; LayerNorm, a bias, and shapes the kernel does not take use the equivalent torch
expression.  Dropout, rowscale and the second (x1) branch of the upstream API are not
supported and raise.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

from .norm import add_rms_norm, supported


def _plain(x, weight, bias, eps, residual, residual_in_fp32, is_rms_norm):
    r = x if residual is None else x + residual
    if residual_in_fp32:
        r = r.float()
    if is_rms_norm:
        rf = r.float()
        y = rf * torch.rsqrt(rf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
        if bias is not None:
            y = y + bias.float()
        y = y.to(x.dtype)
    else:
        y = F.layer_norm(r.to(weight.dtype), (x.shape[-1],), weight, bias, eps).to(x.dtype)
    return y, r


def layer_norm_fn(x, weight, bias, residual=None, x1=None, weight1=None, bias1=None, eps=1e-6, dropout_p=0.0,
                  rowscale=None, prenorm=False, residual_in_fp32=False, is_rms_norm=False,
                  return_dropout_mask=False):
    """y = norm(x + residual); returns y, or (y, new_residual) when ``prenorm``."""
    if x1 is not None or weight1 is not None or dropout_p or rowscale is not None or return_dropout_mask:
        raise NotImplementedError("layer_norm_fn: x1 / weight1 / dropout / rowscale are not supported")
    if is_rms_norm and bias is None and supported(x, residual, weight):
        y, r = add_rms_norm(x, residual, weight, eps, residual_in_fp32)
        if not residual_in_fp32 and residual is None:
            r = r.to(x.dtype)
    else:
        y, r = _plain(x, weight, bias, eps, residual, residual_in_fp32, is_rms_norm)
    return (y, r) if prenorm else y


def rms_norm_fn(x, weight, bias, residual=None, x1=None, weight1=None, bias1=None, eps=1e-6, dropout_p=0.0,
                rowscale=None, prenorm=False, residual_in_fp32=False, return_dropout_mask=False):
    return layer_norm_fn(x, weight, bias, residual, x1, weight1, bias1, eps, dropout_p, rowscale, prenorm,
                         residual_in_fp32, True, return_dropout_mask)


def _layer_norm_fwd(x, weight, bias, eps, residual=None, x1=None, weight1=None, bias1=None, dropout_p=0.0,
                    rowscale=None, out_dtype=None, residual_dtype=None, zero_centered_weight=False,
                    is_rms_norm=False, return_dropout_mask=False, out=None, residual_out=None):
    """Forward only (no autograd); returns (y, mean, rstd, residual_out) with mean None."""
    with torch.no_grad():
        y, r = layer_norm_fn(x, weight, bias, residual=residual, x1=x1, weight1=weight1, bias1=bias1, eps=eps,
                             dropout_p=dropout_p, rowscale=rowscale, prenorm=True,
                             residual_in_fp32=residual_dtype == torch.float32, is_rms_norm=is_rms_norm)
        if out_dtype is not None:
            y = y.to(out_dtype)
        rf = r.float()
        rstd = torch.rsqrt(rf.pow(2).mean(-1) + eps) if is_rms_norm else \
            torch.rsqrt(rf.var(-1, unbiased=False) + eps)
    return y, None, rstd, r


class RMSNorm(nn.Module):
    def __init__(self, hidden_size, eps=1e-5, dropout_p=0.0, device=None, dtype=None):
        super().__init__()
        if dropout_p:
            raise NotImplementedError("RMSNorm: dropout is not supported")
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size, device=device, dtype=dtype))
        self.register_parameter("bias", None)

    def forward(self, x, residual=None, prenorm=False, residual_in_fp32=False):
        return rms_norm_fn(x, self.weight, self.bias, residual=residual, eps=self.eps, prenorm=prenorm,
                           residual_in_fp32=residual_in_fp32)
