"""The reference's own Python glue running on this library's module names (``shims.install()``).

Where the reference's sources are present ($MOTIF_REF names its ``motifmamba`` project
directory), its ``mamba_ssm/ops/selective_scan_interface.py`` is executed with this library
registered as ``selective_scan_cuda`` / ``causal_conv1d`` / the Triton ``layer_norm`` module.
The reference's autograd functions (``SelectiveScanFn``, ``SelectiveScanPQFn``,
``MambaInnerFn``) then call ``selective_scan_cuda.fwd/bwd`` and the causal-conv1d functions with
their own positional and keyword arguments (``selective_scan_interface.py:47-51, 76-82,
136-141, 167-175, 482-484, 534-538, 567-569, 597-603, 635-637``).  Every such call is bound
with ``inspect.signature(...).bind`` against this library's real functions (so a keyword the
reference passes that this library does not accept fails here), and then answered on the CPU
by the oracle in this library's return conventions (list lengths and order, ``x`` layout with
the final state in the last chunk's odd lanes, ``dB`` / ``dC`` in B's 4-D shape, ``dz`` written
into a caller-provided buffer, ``dP_out`` / ``dQ_out`` filled in place).  The reference's
results must equal the oracle's: that checks both the binding and that the reference's glue
(rearranges, squeezes, last_state slicing) works with what this library returns.  The kernels
themselves are checked against the oracle by the GPU tests; this file needs no GPU.
"""
import importlib.util
import inspect
import os
import sys
import types

import pytest
import torch
import torch.nn.functional as F

from oracle import ssm_oracle as O
from ssm_cases import assert_close, make_scan_inputs

REF = os.environ.get("MOTIF_REF")
SSI_PATH = os.path.join(REF, "mamba_ssm/ops/selective_scan_interface.py") if REF else None
pytestmark = pytest.mark.skipif(not (SSI_PATH and os.path.isfile(SSI_PATH)),
                                reason="reference sources not present ($MOTIF_REF unset)")


class _Recorder:
    """Binds each call against this library's function and answers it with `impl`."""

    def __init__(self, real, impl):
        self.sig = inspect.signature(real)
        self.impl = impl
        self.calls = []

    def __call__(self, *args, **kwargs):
        bound = self.sig.bind(*args, **kwargs)  # TypeError for any argument the library rejects
        bound.apply_defaults()
        self.calls.append(sorted(kwargs))
        return self.impl(**bound.arguments)


def _scan_fwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, P=None, Q=None, gamma=None,
              delta_softplus=False, initial_state=None):
    from motif_ssm import selective_scan_cuda as ssc
    assert initial_state is None  # the reference never passes this library's extra argument
    with torch.no_grad():
        out_z_or_out, last = O.selective_scan_ref(u, delta, A, B, C, D, z=z, delta_bias=delta_bias,
                                                  delta_softplus=delta_softplus, return_last_state=True, P=P, Q=Q)
        out = out_z_or_out
        if z is not None:
            out = O.selective_scan_ref(u, delta, A, B, C, D, z=None, delta_bias=delta_bias,
                                       delta_softplus=delta_softplus, P=P, Q=Q)
    b, d, l = u.shape
    n = A.shape[1]
    x = torch.zeros(b, d, ssc.n_chunks(l), 2 * n)
    x[:, :, -1, 1::2] = last
    return [out, x] + ([out_z_or_out] if z is not None else [])


def _scan_bwd(u, delta, A, B, C, D=None, z=None, delta_bias=None, P=None, Q=None, gamma=None, dout=None,
              x=None, out=None, dz=None, dP_out=None, dQ_out=None, delta_softplus=False, recompute_out_z=False):
    inp = dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z, delta_bias=delta_bias)
    if P is not None:
        inp["P"], inp["Q"] = P, Q
    with torch.enable_grad():
        _, _, g = O.scan_with_grads(inp, dout, delta_softplus)
    res = [g["u"], g["delta"], g["A"], g["B"], g["C"], g["D"], g["delta_bias"]]
    if z is not None:
        if dz is not None:
            dz.copy_(g["z"])
            res.append(dz)
        else:
            res.append(g["z"])
        if recompute_out_z:
            res.append(O.selective_scan_ref(u, delta, A, B, C, D, z=z, delta_bias=delta_bias,
                                            delta_softplus=delta_softplus))
    if P is not None:
        if dP_out is not None:
            dP_out.copy_(g["P"])
            dQ_out.copy_(g["Q"])
    return res


def _conv_fwd(x, weight, bias, seq_idx, initial_states, final_states_out, silu_activation):
    assert seq_idx is None and initial_states is None and final_states_out is None
    return O.causal_conv1d_ref(x, weight, bias, "silu" if silu_activation else None)


def _conv_bwd(x, weight, bias, dout, seq_idx, initial_states, dfinal_states, dx, return_dinitial_states,
              silu_activation):
    xl, wl = x.detach().clone().requires_grad_(True), weight.detach().clone().requires_grad_(True)
    bl = bias.detach().clone().requires_grad_(True) if bias is not None else None
    with torch.enable_grad():
        y = O.causal_conv1d_ref(xl, wl, bl, "silu" if silu_activation else None)
        y.backward(dout)
    gx = xl.grad
    if dx is not None:
        dx.copy_(gx)
        gx = dx
    return gx, wl.grad, (bl.grad if bl is not None else None), None


@pytest.fixture(scope="module")
def ref_interface():
    """Execute the reference's selective_scan_interface.py on this library's shims, with the
    scan / conv entry points wrapped by recorders."""
    from motif_ssm import causal_conv1d as cc, selective_scan_cuda as ssc, shims
    saved = {k: sys.modules.get(k) for k in ("mamba_ssm", "mamba_ssm.ops", "mamba_ssm.utils", "mamba_ssm.utils.torch",
                                             "mamba_ssm.ops.triton", "mamba_ssm.ops.triton.layer_norm",
                                             "mamba_ssm.ops.triton.selective_state_update", "selective_scan_cuda",
                                             "causal_conv1d", "causal_conv1d.cpp_functions",
                                             "mamba_ssm.ops.selective_scan_interface")}

    def stub(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        sys.modules[name] = m
        return m

    ident = lambda f=None, **kw: f if f is not None else (lambda g: g)
    stub("mamba_ssm").__path__ = []
    stub("mamba_ssm.ops").__path__ = []
    stub("mamba_ssm.utils").__path__ = []
    stub("mamba_ssm.utils.torch", custom_fwd=ident, custom_bwd=ident)  # absent from the export
    stub("mamba_ssm.ops.triton").__path__ = []
    shims.install()
    rec = {"fwd": _Recorder(ssc.fwd, _scan_fwd), "bwd": _Recorder(ssc.bwd, _scan_bwd),
           "conv_fwd": _Recorder(cc.causal_conv1d_fwd_function, _conv_fwd),
           "conv_bwd": _Recorder(cc.causal_conv1d_bwd_function, _conv_bwd)}
    spec = importlib.util.spec_from_file_location("mamba_ssm.ops.selective_scan_interface", SSI_PATH)
    ssi = importlib.util.module_from_spec(spec)
    sys.modules["mamba_ssm.ops.selective_scan_interface"] = ssi
    spec.loader.exec_module(ssi)
    assert ssi.selective_scan_cuda is ssc  # the reference imported this library under its module name
    ssi.selective_scan_cuda = types.SimpleNamespace(fwd=rec["fwd"], bwd=rec["bwd"])
    ssi.causal_conv1d_fwd_function = rec["conv_fwd"]
    ssi.causal_conv1d_bwd_function = rec["conv_bwd"]
    ssi.causal_conv1d_fn = lambda x, w, b=None, activation=None: O.causal_conv1d_ref(x, w, b, activation)
    yield ssi, rec
    for k, v in saved.items():
        if v is None:
            sys.modules.pop(k, None)
        else:
            sys.modules[k] = v


@pytest.mark.parametrize("has_z,groups", [(True, 0), (False, 0), (True, 2)])
def test_reference_selective_scan_fn_on_shims(ref_interface, has_z, groups):
    ssi, rec = ref_interface
    inp, dout = make_scan_inputs(2, 8, 300, 16, torch.float32, groups=groups, has_z=has_z, seed=5)
    leaves = {k: (v.clone().requires_grad_(True) if v is not None else None) for k, v in inp.items()}
    n_fwd, n_bwd = len(rec["fwd"].calls), len(rec["bwd"].calls)
    out, last = ssi.selective_scan_fn(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                      leaves["D"], z=leaves["z"], delta_bias=leaves["delta_bias"],
                                      delta_softplus=True, return_last_state=True)
    out.backward(dout)
    assert len(rec["fwd"].calls) == n_fwd + 1 and len(rec["bwd"].calls) == n_bwd + 1
    r_out, r_last, r_g = O.scan_with_grads(inp, dout, True)
    assert_close(out, r_out, 1e-5, 1e-5, "out")
    assert_close(last, r_last, 1e-5, 1e-5, "last_state")
    for k in ("u", "delta", "A", "B", "C", "D", "z", "delta_bias"):
        if inp[k] is None:
            continue
        assert leaves[k].grad.shape == inp[k].shape, k
        assert_close(leaves[k].grad, r_g[k], 1e-5, 1e-5, f"d{k}", scaled=True)


def test_reference_selective_scan_pq_fn_on_shims(ref_interface, monkeypatch):
    """SelectiveScanPQFn passes P, Q, gamma and dP_out / dQ_out to fwd / bwd (its fused-gradient
    mode; the default mode re-derives dP / dQ through a CUDA-only path)."""
    ssi, rec = ref_interface
    monkeypatch.setenv("MOTIFMAMBA_PQ_GRAD_MODE", "fast")
    inp, dout = make_scan_inputs(2, 8, 120, 16, torch.float32, has_z=False, seed=6, pq_rank=3, pq_scale=0.3)
    leaves = {k: (v.clone().requires_grad_(True) if v is not None else None) for k, v in inp.items()}
    out, last = ssi.SelectiveScanPQFn.apply(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                            leaves["D"], None, leaves["delta_bias"], True, True, leaves["P"],
                                            leaves["Q"], None)
    out.backward(dout)
    assert "dP_out" in rec["bwd"].calls[-1] and "P" in rec["fwd"].calls[-1]
    r_out, r_last, r_g = O.scan_with_grads(inp, dout, True)
    assert_close(out, r_out, 1e-5, 1e-5, "P/Q out")
    assert_close(last, r_last, 1e-5, 1e-5, "P/Q last_state")
    for k in ("u", "delta", "A", "B", "C", "D", "delta_bias", "P", "Q"):
        assert_close(leaves[k].grad, r_g[k], 1e-5, 1e-5, f"P/Q d{k}", scaled=True)


def test_reference_mamba_inner_fn_on_shims(ref_interface):
    """MambaInnerFn: causal_conv1d_fwd/bwd_function and selective_scan_cuda.fwd/bwd (with a
    caller-provided dz view into dxz and recompute_out_z=True) through the reference's code."""
    ssi, rec = ref_interface
    g = torch.Generator().manual_seed(8)
    d_model, d_inner, n, rank, b, l = 16, 32, 16, 4, 2, 64
    p = dict(xz=torch.randn(b, 2 * d_inner, l, generator=g),
             conv1d_weight=0.3 * torch.randn(d_inner, 1, 4, generator=g),
             conv1d_bias=0.1 * torch.randn(d_inner, generator=g),
             x_proj_weight=0.2 * torch.randn(rank + 2 * n, d_inner, generator=g),
             delta_proj_weight=0.3 * torch.randn(d_inner, rank, generator=g),
             out_proj_weight=0.2 * torch.randn(d_model, d_inner, generator=g),
             A=-torch.arange(1, n + 1, dtype=torch.float32).repeat(d_inner, 1),
             D=torch.ones(d_inner), delta_bias=torch.full((d_inner,), -3.0))
    dout = torch.randn(b, l, d_model, generator=g)
    args = ("xz", "conv1d_weight", "conv1d_bias", "x_proj_weight", "delta_proj_weight", "out_proj_weight")
    la = {k: v.clone().requires_grad_(True) for k, v in p.items()}
    out = ssi.mamba_inner_fn(*(la[k] for k in args), None, la["A"], None, None, la["D"],
                             delta_bias=la["delta_bias"], delta_softplus=True)
    out.backward(dout)
    assert rec["bwd"].calls[-1].count("dz") == 1 and "recompute_out_z" in rec["bwd"].calls[-1]
    lr = {k: v.clone().requires_grad_(True) for k, v in p.items()}
    ref = O.mamba_inner_ref(*(lr[k] for k in args), None, lr["A"], None, None, lr["D"],
                            delta_bias=lr["delta_bias"])
    ref.backward(dout)
    assert_close(out, ref, 1e-4, 1e-4, "mamba_inner_fn out")
    for k in p:
        assert_close(la[k].grad, lr[k].grad, 1e-4, 1e-4, f"mamba_inner_fn d{k}", scaled=True)
