"""Drop-in for the external ``causal_conv1d`` package the reference imports
(``mamba_ssm/ops/selective_scan_interface.py:10-17``,
``mamba_ssm/modules/mamba_simplemotif.py:15-18``), running on ``libmotif_ssm.so``.

Provides ``causal_conv1d_fn``, ``causal_conv1d_update`` and, as
``cpp_functions``, ``causal_conv1d_fwd_function`` / ``causal_conv1d_bwd_function`` /
``causal_conv1d_update_function`` with the argument order the reference uses.
Sequence-index packing, initial / final states and cache indices are not built and
raise ``NotImplementedError`` (no call site of the reference passes them).
"""
import ctypes
import types

import torch

from . import _lib
from ._lib import lib, check
from .selective_scan_cuda import _itype, _ptr, _stream, _req


def _not_built(**kw):
    for k, v in kw.items():
        if v is not None and v is not False:
            raise NotImplementedError(f"causal_conv1d: {k} is not supported by this library")


def _silu_flag(activation):
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, 'silu' or 'swish'")
    return activation in ("silu", "swish")


def _conv_args(x, weight, bias, silu):
    _req(x.is_cuda and weight.is_cuda, "x and weight must be CUDA tensors")
    _req(x.dim() == 3, "x must be (batch, dim, seqlen)")
    batch, dim, seqlen = x.shape
    _req(weight.dim() == 2 and weight.shape[0] == dim, "weight must be (dim, width)")
    _req(x.stride(-1) == 1 or seqlen == 1, "x must have unit stride in the last dimension")
    if bias is not None:
        _req(bias.is_cuda and bias.shape == (dim,) and bias.dtype == weight.dtype and bias.is_contiguous(),
             "bias must be a contiguous (dim,) CUDA tensor with the dtype of weight")
    a = _lib.Conv1dArgs()
    a.batch, a.dim, a.seqlen, a.width = batch, dim, seqlen, weight.shape[1]
    a.itype, a.wtype, a.silu = _itype(x.dtype), _itype(weight.dtype), 1 if silu else 0
    a.x, a.x_bs, a.x_ds = _ptr(x), x.stride(0), x.stride(1)
    a.weight, a.w_ds, a.w_ks = _ptr(weight), weight.stride(0), weight.stride(1)
    a.bias = _ptr(bias)
    return a


def causal_conv1d_fwd_function(x, weight, bias, seq_idx, initial_states, final_states_out, silu_activation):
    _not_built(seq_idx=seq_idx, initial_states=initial_states, final_states_out=final_states_out)
    a = _conv_args(x, weight, bias, silu_activation)
    out = torch.empty_like(x)
    a.out, a.out_bs, a.out_ds = _ptr(out), out.stride(0), out.stride(1)
    with torch.cuda.device(x.device):
        check(lib.conv1d_fwd(ctypes.byref(a), _stream(x.device)))
    return out


def causal_conv1d_bwd_function(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx,
                               return_dinitial_states, silu_activation):
    _not_built(seq_idx=seq_idx, initial_states=initial_states, dfinal_states=dfinal_states,
               return_dinitial_states=return_dinitial_states)
    a = _conv_args(x, weight, bias, silu_activation)
    _req(dout.shape == x.shape and dout.dtype == x.dtype and dout.is_cuda, "dout must match x")
    if dout.stride(-1) != 1:
        dout = dout.contiguous()
    if dx is None:
        dx = torch.empty_like(x)
    _req(dx.shape == x.shape and dx.dtype == x.dtype and dx.stride(-1) == 1, "dx must match x")
    dweight = torch.empty(weight.shape, device=x.device, dtype=torch.float32)
    dbias = torch.empty(bias.shape, device=x.device, dtype=torch.float32) if bias is not None else None
    a.dout, a.dout_bs, a.dout_ds = _ptr(dout), dout.stride(0), dout.stride(1)
    a.dx, a.dx_bs, a.dx_ds = _ptr(dx), dx.stride(0), dx.stride(1)
    a.dweight, a.dbias = _ptr(dweight), _ptr(dbias)
    with torch.cuda.device(x.device):
        check(lib.conv1d_bwd(ctypes.byref(a), _stream(x.device)))
    dweight = dweight.to(weight.dtype)
    if dbias is not None:
        dbias = dbias.to(bias.dtype)
    return dx, dweight, dbias, None


def causal_conv1d_update_function(x, conv_state, weight, bias, silu_activation, cache_seqlens, conv_state_indices):
    _not_built(cache_seqlens=cache_seqlens, conv_state_indices=conv_state_indices)
    squeeze = x.dim() == 2
    if x.dim() == 3:
        _req(x.shape[-1] == 1, "causal_conv1d_update: only one token per call is supported")
        x = x[..., 0]
    batch, dim = x.shape
    _req(conv_state.is_cuda and conv_state.dim() == 3 and conv_state.shape[:2] == (batch, dim),
         "conv_state must be (batch, dim, state_len)")
    _req(conv_state.stride(-1) == 1, "conv_state must have unit stride in the last dimension")
    _req(x.stride(-1) == 1, "x must have unit stride in the last dimension")
    _req(weight.dim() == 2 and weight.shape[0] == dim, "weight must be (dim, width)")
    if bias is not None:
        _req(bias.shape == (dim,) and bias.dtype == weight.dtype and bias.is_contiguous(), "bad bias")
    out = torch.empty_like(x)
    a = _lib.Conv1dUpdateArgs()
    a.batch, a.dim, a.width, a.state_len = batch, dim, weight.shape[1], conv_state.shape[2]
    a.itype, a.wtype, a.stype = _itype(x.dtype), _itype(weight.dtype), _itype(conv_state.dtype)
    a.silu = 1 if silu_activation else 0
    a.x, a.x_bs = _ptr(x), x.stride(0)
    a.conv_state, a.cs_bs, a.cs_ds = _ptr(conv_state), conv_state.stride(0), conv_state.stride(1)
    a.weight, a.w_ds, a.w_ks = _ptr(weight), weight.stride(0), weight.stride(1)
    a.bias = _ptr(bias)
    a.out, a.out_bs = _ptr(out), out.stride(0)
    with torch.cuda.device(x.device):
        check(lib.conv1d_update(ctypes.byref(a), _stream(x.device)))
    return out if squeeze else out.unsqueeze(-1)


class CausalConv1dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias=None, activation=None):
        silu = _silu_flag(activation)
        if x.stride(-1) != 1:
            x = x.contiguous()
        weight = weight.contiguous()
        bias = bias.contiguous() if bias is not None else None
        ctx.save_for_backward(x, weight, bias)
        ctx.silu = silu
        return causal_conv1d_fwd_function(x, weight, bias, None, None, None, silu)

    @staticmethod
    def backward(ctx, dout):
        x, weight, bias = ctx.saved_tensors
        dx, dweight, dbias, _ = causal_conv1d_bwd_function(x, weight, bias, dout, None, None, None, None,
                                                           False, ctx.silu)
        return dx, dweight, dbias if bias is not None else None, None


def causal_conv1d_fn(x, weight, bias=None, seq_idx=None, initial_states=None, return_final_states=False,
                     final_states_out=None, activation=None):
    """x: (batch, dim, seqlen); weight: (dim, width); returns (batch, dim, seqlen)."""
    _not_built(seq_idx=seq_idx, initial_states=initial_states, return_final_states=return_final_states,
               final_states_out=final_states_out)
    return CausalConv1dFn.apply(x, weight, bias, activation)


def causal_conv1d_update(x, conv_state, weight, bias=None, activation=None, cache_seqlens=None,
                         conv_state_indices=None):
    """x: (batch, dim) or (batch, dim, 1); conv_state (batch, dim, state_len) is updated in place."""
    return causal_conv1d_update_function(x, conv_state, weight, bias, _silu_flag(activation), cache_seqlens,
                                         conv_state_indices)


cpp_functions = types.SimpleNamespace(
    causal_conv1d_fwd_function=causal_conv1d_fwd_function,
    causal_conv1d_bwd_function=causal_conv1d_bwd_function,
    causal_conv1d_update_function=causal_conv1d_update_function,
)
