"""CPU oracle for the selective-scan hot path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as the checker / the timed CPU reference.
The product (``motif-mamba_b200/motif_ssm``) never imports it and has no CPU
fallback.

Each function is a plain-torch restatement, in fp32 on the CPU, of the
reference's own pure-torch path (4354ce38/Motif-Mamba, a fork of mamba_ssm
2.2.6.post3; paths below are relative to the reference project):

* ``selective_scan_ref``        <- ``mamba_ssm/ops/selective_scan_interface.py:353-451``
* ``mamba_inner_ref``           <- ``mamba_ssm/ops/selective_scan_interface.py:659-694``
* ``causal_conv1d_ref``         <- ``mamba_ssm/modules/mamba_simplemotif.py:75-83, 294-295``
                                   (the module's own fallback for the external
                                   ``causal_conv1d`` package, which the reference
                                   does not vendor; causal-conv1d >= 1.2.0 per
                                   ``pyproject.toml:33-34``)
* ``causal_conv1d_update_ref``  <- ``mamba_ssm/modules/mamba_simplemotif.py:344-350``
* ``selective_state_update_ref``<- ``mamba_ssm/modules/mamba_simplemotif.py:367-376``
                                   (fallback for the missing Triton kernel)
* ``mixer_pq_prefill_ref``      <- ``mamba_ssm/modules/mamba_simplemotif.py:256-335`` (slow
                                   path with ``P_eff = pq_k * P``)
* ``mixer_pq_step_ref``         <- ``mamba_ssm/modules/mamba_simplemotif.py:337-402`` (P/Q step)
* ``rms_norm_ref``              <- x * rsqrt(mean(x^2) + eps) * w, the RMSNorm the
                                   stack uses (``mamba_ssm/models/mixer_seq_simple.py:64-66``,
                                   eps default ``:35``); the Triton source is missing.

Parity pinning: ``tests/test_oracle_golden.py`` checks every function here
against fixtures produced by running the reference's own code
(``tests/golden/make_golden.py``).
"""
import torch
import torch.nn.functional as F


def _softplus(x):
    # torch's softplus (threshold 20) is what the reference calls (selective_scan_interface.py:374).
    return F.softplus(x)


def selective_scan_ref(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False,
                       return_last_state=False, P=None, Q=None, gamma=None):
    """Sequential diagonal SSM scan, real A only.

    h_t = exp(delta_t * A) * h_{t-1} + delta_t * B_t * u_t ;  y_t = <C_t, h_t>
    out = (y + D * u) * silu(z), cast to u's dtype.

    Shapes: u, delta, z (b, d, l); A (d, n); B, C (b, n, l) or (b, g, n, l) or
    constant (d, n); D, delta_bias (d,).  Follows selective_scan_interface.py:368-451
    step for step (fp32 math, silu(z) evaluated in z's dtype as at :449).
    """
    if A.is_complex():
        raise NotImplementedError("oracle covers real A only")
    dtype_in = u.dtype
    u = u.float()
    delta = delta.float()
    if delta_bias is not None:
        delta = delta + delta_bias[..., None].float()
    if delta_softplus:
        delta = _softplus(delta)
    batch, dim, dstate = u.shape[0], A.shape[0], A.shape[1]
    var_B, var_C = B.dim() >= 3, C.dim() >= 3
    B = B.float()
    C = C.float()
    if var_B and B.dim() == 4:
        B = B.repeat_interleave(dim // B.shape[1], dim=1)       # (b, d, n, l)
    if var_C and C.dim() == 4:
        C = C.repeat_interleave(dim // C.shape[1], dim=1)
    dA = torch.exp(delta.unsqueeze(-1) * A.float().unsqueeze(1))  # (b, d, l, n)
    if not var_B:
        dBu = (delta * u).unsqueeze(-1) * B.unsqueeze(1)
    elif B.dim() == 3:
        dBu = (delta * u).unsqueeze(-1) * B.transpose(1, 2).unsqueeze(1)
    else:
        dBu = (delta * u).unsqueeze(-1) * B.permute(0, 1, 3, 2)
    h = u.new_zeros(batch, dim, dstate)
    ys = []
    use_pq = P is not None or Q is not None
    if use_pq:
        # motif low-rank coupling (selective_scan_interface.py:402-433): gamma is not used there
        if P is None or Q is None:
            raise ValueError("P and Q must be both provided")
        if P.dim() == 2:
            Pd, Qd = P.float().unsqueeze(0).expand(dim, -1, -1), Q.float().unsqueeze(0).expand(dim, -1, -1)
        else:
            Pd, Qd = P.float(), Q.float()
    for i in range(u.shape[2]):
        if use_pq:
            q = torch.einsum("drn,bdn->bdr", Qd, h)
            pq = torch.einsum("dnr,bdr->bdn", Pd, q)
            h = dA[:, :, i] * h + delta[:, :, i].unsqueeze(-1) * pq + dBu[:, :, i]
        else:
            h = dA[:, :, i] * h + dBu[:, :, i]
        if not var_C:
            y = (h * C.unsqueeze(0)).sum(-1)
        elif C.dim() == 3:
            y = (h * C[:, :, i].unsqueeze(1)).sum(-1)
        else:
            y = (h * C[:, :, :, i]).sum(-1)
        ys.append(y)
    y = torch.stack(ys, dim=2)
    out = y if D is None else y + u * D.float().unsqueeze(-1)
    if z is not None:
        out = out * F.silu(z)
    out = out.to(dtype_in)
    return (out, h) if return_last_state else out


def causal_conv1d_ref(x, weight, bias=None, activation=None):
    """Depthwise causal conv over L: y[b,c,t] = act(bias_c + sum_k w[c,k] * x[b,c,t-W+1+k]).

    The module's fallback is ``nn.Conv1d(groups=d_inner, padding=W-1)(x)[..., :L]``
    followed by SiLU (mamba_simplemotif.py:75-83, 295); math in fp32, output in x's dtype.
    """
    dtype_in = x.dtype
    w = weight.shape[-1]
    y = F.conv1d(x.float(), weight.float().unsqueeze(1),
                 bias.float() if bias is not None else None,
                 padding=w - 1, groups=x.shape[1])[..., : x.shape[-1]]
    if activation in ("silu", "swish"):
        y = F.silu(y)
    return y.to(dtype_in)


def causal_conv1d_update_ref(x, conv_state, weight, bias=None, activation=None):
    """One decode step (mamba_simplemotif.py:344-350): roll the state left, append x,
    dot with the taps, add bias, activation.  ``conv_state`` (b, d, W) is updated in place."""
    dtype = x.dtype
    conv_state.copy_(torch.roll(conv_state, shifts=-1, dims=-1))
    conv_state[:, :, -1] = x
    y = torch.sum(conv_state.float() * weight.float(), dim=-1)
    if bias is not None:
        y = y + bias.float()
    if activation in ("silu", "swish"):
        y = F.silu(y)
    return y.to(dtype)


def selective_state_update_ref(state, x, dt, A, B, C, D=None, z=None, dt_bias=None,
                               dt_softplus=False):
    """Single-token SSM update (mamba_simplemotif.py:367-376); ``state`` (b, d, n) updated in place.

    dt <- softplus(dt + dt_bias); state <- state * exp(dt*A) + x * dt * B;
    y = <state, C> + D * x; y *= silu(z).
    """
    dtype = x.dtype
    dtf = dt.float()
    if dt_bias is not None:
        dtf = dtf + dt_bias.float()
    if dt_softplus:
        dtf = _softplus(dtf)
    dA = torch.exp(dtf.unsqueeze(-1) * A.float())
    dB = dtf.unsqueeze(-1) * B.float().unsqueeze(1)
    new_state = state.float() * dA + x.float().unsqueeze(-1) * dB
    state.copy_(new_state.to(state.dtype))
    y = (state.float() * C.float().unsqueeze(1)).sum(-1)
    if D is not None:
        y = y + D.float() * x.float()
    if z is not None:
        y = y * F.silu(z.float())
    return y.to(dtype)


def _rms_straight_through(t, weight, eps, dim):
    """RMSNorm of t along ``dim`` (fp32 math, t's dtype) whose gradient is passed through
    unchanged, as the reference's ``MambaInnerFn.backward`` treats it."""
    tf = t.detach().float()
    shape = [1] * t.dim()
    shape[dim] = -1
    y = (tf * torch.rsqrt(tf.pow(2).mean(dim=dim, keepdim=True) + eps) * weight.detach().float().view(shape))
    y = y.to(t.dtype)
    return t + (y - t).detach()


def mamba_inner_ref(xz, conv1d_weight, conv1d_bias, x_proj_weight, delta_proj_weight,
                    out_proj_weight, out_proj_bias, A, B=None, C=None, D=None, delta_bias=None,
                    B_proj_bias=None, C_proj_bias=None, delta_softplus=True, b_rms_weight=None,
                    c_rms_weight=None, dt_rms_weight=None, b_c_dt_rms_eps=1e-6):
    """Mamba-1 inner block (selective_scan_interface.py:659-694): conv+SiLU -> x_proj ->
    dt_proj -> selective scan (z-gated, softplus) -> out_proj.

    The optional RMSNorm weights follow ``MambaInnerFn`` (``:521-532``): B and C are
    normalised over dstate and delta over channels before the scan.  Their backward is the
    identity (the reference's backward, ``:597-645``, passes the scan's dB / dC / ddelta
    straight to x_proj and dt_proj), so autograd through this function reproduces those
    gradients."""
    L = xz.shape[-1]
    delta_rank = delta_proj_weight.shape[1]
    d_state = A.shape[-1]
    x, z = xz.chunk(2, dim=1)
    x = causal_conv1d_ref(x, conv1d_weight.reshape(conv1d_weight.shape[0], -1), conv1d_bias,
                          activation="silu")
    x_dbl = F.linear(x.transpose(1, 2).reshape(-1, x.shape[1]), x_proj_weight)
    delta = (delta_proj_weight @ x_dbl[:, :delta_rank].t())
    delta = delta.reshape(delta.shape[0], -1, L).transpose(0, 1)
    if B is None:
        B = x_dbl[:, delta_rank:delta_rank + d_state]
        if B_proj_bias is not None:
            B = B + B_proj_bias.to(B.dtype)
        B = B.reshape(-1, L, d_state).transpose(1, 2).contiguous()
    if C is None:
        C = x_dbl[:, -d_state:]
        if C_proj_bias is not None:
            C = C + C_proj_bias.to(C.dtype)
        C = C.reshape(-1, L, d_state).transpose(1, 2).contiguous()
    if b_rms_weight is not None:
        B = _rms_straight_through(B, b_rms_weight, b_c_dt_rms_eps, -2)
    if c_rms_weight is not None:
        C = _rms_straight_through(C, c_rms_weight, b_c_dt_rms_eps, -2)
    if dt_rms_weight is not None:
        delta = _rms_straight_through(delta, dt_rms_weight, b_c_dt_rms_eps, 1)
    y = selective_scan_ref(x, delta, A, B, C, D, z=z, delta_bias=delta_bias,
                           delta_softplus=delta_softplus)
    return F.linear(y.transpose(1, 2), out_proj_weight, out_proj_bias)


def mixer_pq_prefill_ref(sd, hidden, return_last_state=False):
    """Mambamotif slow-path prefill with the P/Q coupling (mamba_simplemotif.py:256-335):
    in_proj -> causal conv + SiLU -> x_proj -> dt_proj -> scan with ``P_eff = pq_k * P`` ->
    out_proj.  ``sd`` is the module's state dict (fp32)."""
    batch, seqlen, _ = hidden.shape
    xz = torch.einsum("od,bld->bol", sd["in_proj.weight"], hidden)
    x, z = xz.chunk(2, dim=1)
    x = causal_conv1d_ref(x, sd["conv1d.weight"][:, 0, :], sd["conv1d.bias"], "silu")
    n = sd["A_log"].shape[1]
    dt_rank = sd["dt_proj.weight"].shape[1]
    x_dbl = torch.einsum("bdl,od->blo", x, sd["x_proj.weight"])
    dt, B, C = torch.split(x_dbl, [dt_rank, n, n], dim=-1)
    dt = torch.einsum("blr,dr->bdl", dt, sd["dt_proj.weight"])
    A = -torch.exp(sd["A_log"].float())
    y = selective_scan_ref(x, dt, A, B.transpose(1, 2), C.transpose(1, 2), sd["D"].float(), z=z,
                           delta_bias=sd["dt_proj.bias"].float(), delta_softplus=True,
                           return_last_state=return_last_state, P=sd["pq_k"] * sd["P"], Q=sd["Q"])
    y, last = y if return_last_state else (y, None)
    out = torch.einsum("bdl,od->blo", y, sd["out_proj.weight"])
    return (out, last) if return_last_state else out


def mixer_pq_step_ref(sd, hidden, conv_state, ssm_state):
    """Mambamotif.step with the P/Q coupling (mamba_simplemotif.py:337-395): conv update, then
    a one-step scan that starts from a zero state (the reference does not feed ``ssm_state``
    in), whose final state overwrites ``ssm_state``.  Updates the states in place."""
    xz = hidden[:, 0] @ sd["in_proj.weight"].t()
    x, z = xz.chunk(2, dim=-1)
    x = causal_conv1d_update_ref(x, conv_state, sd["conv1d.weight"][:, 0, :], sd["conv1d.bias"], "silu")
    n = sd["A_log"].shape[1]
    dt_rank = sd["dt_proj.weight"].shape[1]
    dt, B, C = torch.split(x @ sd["x_proj.weight"].t(), [dt_rank, n, n], dim=-1)
    dt = _softplus(dt @ sd["dt_proj.weight"].t() + sd["dt_proj.bias"])
    A = -torch.exp(sd["A_log"].float())
    y, last = selective_scan_ref(x[..., None], dt[..., None], A, B[..., None], C[..., None], sd["D"].float(),
                                 z=z[..., None], return_last_state=True, P=sd["pq_k"] * sd["P"], Q=sd["Q"])
    ssm_state.copy_(last)
    return (y[..., 0] @ sd["out_proj.weight"].t())[:, None]


def rms_norm_ref(x, weight, eps=1e-5):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    return y.to(x.dtype)


def scan_with_grads(inputs, dout, delta_softplus, return_last_state=True):
    """Run ``selective_scan_ref`` with autograd; returns (out, last_state, grads dict).
    ``inputs`` may carry ``P`` / ``Q`` (motif path)."""
    leaves = {k: (v.detach().clone().requires_grad_(True) if v is not None else None)
              for k, v in inputs.items()}
    out, last = selective_scan_ref(leaves["u"], leaves["delta"], leaves["A"], leaves["B"],
                                   leaves["C"], leaves["D"], z=leaves["z"],
                                   delta_bias=leaves["delta_bias"],
                                   delta_softplus=delta_softplus, return_last_state=True,
                                   P=leaves.get("P"), Q=leaves.get("Q"))
    out.backward(dout)
    grads = {k: (v.grad if v is not None else None) for k, v in leaves.items()}
    return out.detach(), last.detach(), grads
