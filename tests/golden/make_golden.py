"""Generate the golden fixtures that pin the CPU oracle to the reference itself.

This script imports the reference's own Python code (mamba_ssm 2.2.6.post3 fork,
``motifmamba/mamba_ssm``) and records its outputs on small seeded inputs.  The
reference export is incomplete, so three missing modules are replaced by stubs
before the file is executed:

* ``mamba_ssm.utils.torch``             -> identity ``custom_fwd`` / ``custom_bwd``
* ``mamba_ssm.ops.triton.layer_norm``   -> unused placeholder (only imported)
* ``selective_scan_cuda``               -> empty module (only imported; the
  fixtures use the pure-torch reference functions, never the CUDA extension)

``causal_conv1d`` is a third-party package that the export does not vendor.  For
``mamba_inner_ref`` it is replaced by the model's own torch fallback
(``nn.Conv1d(groups=d, padding=w-1)[..., :L]`` + SiLU,
``motifmamba/mamba_ssm/modules/mamba_simplemotif.py:75-83, 295``).

Run in a container that has the reference checkout (its ``motifmamba`` project directory
in ``$MOTIF_REF``, which is required).  The outputs are small
``.pt`` files next to this script; nothing at test time reads the reference.
"""
import importlib.util
import os
import sys
import types

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("MOTIF_REF")
if not REF:
    raise SystemExit("set MOTIF_REF to the reference's motifmamba project directory")


def _stub(name, **attrs):
    m = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(m, k, v)
    sys.modules[name] = m
    return m


def load_reference():
    """Exec the reference's ops and module files with the stubs described above."""
    def _identity_deco(f=None, **kw):
        return f if f is not None else (lambda g: g)

    pkg = _stub("mamba_ssm")
    pkg.__path__ = []
    ops = _stub("mamba_ssm.ops")
    ops.__path__ = []
    _stub("mamba_ssm.utils")
    _stub("mamba_ssm.utils.torch", custom_fwd=_identity_deco, custom_bwd=_identity_deco)
    _stub("mamba_ssm.ops.triton")
    _stub("mamba_ssm.ops.triton.layer_norm", _layer_norm_fwd=None)
    _stub("selective_scan_cuda")
    spec = importlib.util.spec_from_file_location(
        "mamba_ssm.ops.selective_scan_interface",
        os.path.join(REF, "mamba_ssm/ops/selective_scan_interface.py"))
    ssi = importlib.util.module_from_spec(spec)
    sys.modules["mamba_ssm.ops.selective_scan_interface"] = ssi
    spec.loader.exec_module(ssi)

    def conv_fallback(x, weight, bias=None, activation=None):
        w = weight.shape[-1]
        y = F.conv1d(x, weight.unsqueeze(1), bias, padding=w - 1, groups=x.shape[1])[..., : x.shape[-1]]
        return F.silu(y) if activation in ("silu", "swish") else y

    ssi.causal_conv1d_fn = conv_fallback
    # mamba_inner_ref calls selective_scan_fn, which dispatches to the CUDA
    # extension; on CPU it is swapped for the pure-torch reference, as the
    # reference's own CPU re-evaluation does (motif/eval_induction_checkpoints.py:61-68).
    ssi.selective_scan_fn = ssi.selective_scan_ref

    spec = importlib.util.spec_from_file_location(
        "mamba_ssm.modules.mamba_simplemotif",
        os.path.join(REF, "mamba_ssm/modules/mamba_simplemotif.py"))
    msm = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(msm)
    # Same swap the reference's own CPU re-evaluation does
    # (motif/eval_induction_checkpoints.py:61-68).
    msm.selective_scan_fn = ssi.selective_scan_ref
    return ssi, msm


def scan_case(ssi, name, *, batch, dim, seqlen, dstate, dtype=torch.float32, groups=0,
              has_z=True, has_D=True, has_bias=True, softplus=True, grads=True, seed=0, pq_rank=0,
              pq_per_dim=False):
    """Inputs distributed as BASELINE config 0: N(0,1) data, S4D-real A, bias = inv-softplus(U[1e-3, 1e-1])."""
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(batch, dim, seqlen, generator=g).to(dtype)
    if softplus:
        delta = torch.randn(batch, dim, seqlen, generator=g).to(dtype)
    else:  # without softplus, delta must already be a step size (>= 0)
        delta = (0.5 * torch.rand(batch, dim, seqlen, generator=g)).to(dtype)
    A = -torch.arange(1, dstate + 1, dtype=torch.float32).repeat(dim, 1).contiguous()
    if groups:
        B = torch.randn(batch, groups, dstate, seqlen, generator=g).to(dtype)
        C = torch.randn(batch, groups, dstate, seqlen, generator=g).to(dtype)
    else:
        B = torch.randn(batch, dstate, seqlen, generator=g).to(dtype)
        C = torch.randn(batch, dstate, seqlen, generator=g).to(dtype)
    D = (1.0 + 0.1 * torch.randn(dim, generator=g)).float() if has_D else None
    z = torch.randn(batch, dim, seqlen, generator=g).to(dtype) if has_z else None
    if has_bias:
        dt = torch.rand(dim, generator=g) * (0.1 - 1e-3) + 1e-3
        delta_bias = torch.log(torch.expm1(dt)).float()
    else:
        delta_bias = None
    dout = torch.randn(batch, dim, seqlen, generator=g).to(dtype)
    inputs = dict(u=u, delta=delta, A=A, B=B, C=C, D=D, z=z, delta_bias=delta_bias)
    if pq_rank:
        # magnitudes like a trained motif adapter: P, Q ~ N(0, 0.5) (the module scales P by pq_k)
        if pq_per_dim:
            inputs["P"] = 0.5 * torch.randn(dim, dstate, pq_rank, generator=g)
            inputs["Q"] = 0.5 * torch.randn(dim, pq_rank, dstate, generator=g)
        else:
            inputs["P"] = 0.5 * torch.randn(dstate, pq_rank, generator=g)
            inputs["Q"] = 0.5 * torch.randn(pq_rank, dstate, generator=g)
    leaves = {k: (v.clone().requires_grad_(grads) if v is not None else None) for k, v in inputs.items()}
    out, last_state = ssi.selective_scan_ref(
        leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"], leaves["D"],
        z=leaves["z"], delta_bias=leaves["delta_bias"], delta_softplus=softplus, return_last_state=True,
        P=leaves.get("P"), Q=leaves.get("Q"))
    rec = dict(name=name, kind="scan", softplus=softplus, inputs=inputs, dout=dout,
               out=out.detach(), last_state=last_state.detach())
    if grads:
        out.backward(dout)
        rec["grads"] = {k: (v.grad.detach() if v is not None else None) for k, v in leaves.items()}
    torch.save(rec, os.path.join(HERE, f"scan_{name}.pt"))
    print("wrote", name, tuple(out.shape), out.dtype)


def inner_case(ssi, name, *, batch=2, d_model=16, expand=2, dstate=8, dt_rank=4, d_conv=4,
               seqlen=40, seed=0):
    g = torch.Generator().manual_seed(seed)
    d_inner = expand * d_model
    p = dict(
        xz=torch.randn(batch, 2 * d_inner, seqlen, generator=g),
        conv1d_weight=0.3 * torch.randn(d_inner, 1, d_conv, generator=g),
        conv1d_bias=0.1 * torch.randn(d_inner, generator=g),
        x_proj_weight=0.2 * torch.randn(dt_rank + 2 * dstate, d_inner, generator=g),
        delta_proj_weight=0.3 * torch.randn(d_inner, dt_rank, generator=g),
        out_proj_weight=0.2 * torch.randn(d_model, d_inner, generator=g),
        out_proj_bias=0.1 * torch.randn(d_model, generator=g),
        A=-torch.arange(1, dstate + 1, dtype=torch.float32).repeat(d_inner, 1),
        D=torch.ones(d_inner) + 0.1 * torch.randn(d_inner, generator=g),
        delta_bias=torch.log(torch.expm1(torch.rand(d_inner, generator=g) * 0.099 + 1e-3)),
    )
    dout = torch.randn(batch, seqlen, d_model, generator=g)
    leaves = {k: v.clone().requires_grad_(True) for k, v in p.items()}
    out = ssi.mamba_inner_ref(
        leaves["xz"], leaves["conv1d_weight"], leaves["conv1d_bias"], leaves["x_proj_weight"],
        leaves["delta_proj_weight"], leaves["out_proj_weight"], leaves["out_proj_bias"],
        leaves["A"], None, None, leaves["D"], delta_bias=leaves["delta_bias"], delta_softplus=True)
    out.backward(dout)
    rec = dict(name=name, kind="inner", inputs=p, dout=dout, out=out.detach(),
               grads={k: v.grad.detach() for k, v in leaves.items()})
    torch.save(rec, os.path.join(HERE, f"inner_{name}.pt"))
    print("wrote inner", name, tuple(out.shape))


def module_case(msm, name, *, batch=2, d_model=16, d_state=8, prefill=12, steps=3, seed=0, pq_rank=0,
                pq_per_dim=False, pq_k=8.0):
    """Mambamotif prefill (slow path) + decode steps through the module's torch fallbacks.
    With ``pq_rank`` the P / Q factors and ``pq_k`` are redrawn large enough (N(0, 0.5) and ``pq_k``)
    that the coupling visibly changes the outputs."""
    torch.manual_seed(seed)
    mod = msm.Mambamotif(d_model=d_model, d_state=d_state, d_conv=4, expand=2,
                         use_fast_path=False, layer_idx=0, pq_rank=pq_rank, pq_per_dim=pq_per_dim)
    g = torch.Generator().manual_seed(seed + 1)
    pq = {}
    if pq_rank:
        with torch.no_grad():
            mod.P.copy_(0.5 * torch.randn(mod.P.shape, generator=g))
            mod.Q.copy_(0.5 * torch.randn(mod.Q.shape, generator=g))
            mod.pq_k.fill_(pq_k)
        pq = dict(P=mod.pq_k * mod.P, Q=mod.Q)
    hs = torch.randn(batch, prefill, d_model, generator=g)
    with torch.no_grad():
        y_prefill = mod(hs)
        # Build the decode state exactly as the module's prefill would with an
        # inference cache: conv_state <- last d_conv inputs, ssm_state <- last state.
        conv_state, ssm_state = mod.allocate_inference_cache(batch, prefill + steps)
        xz = torch.einsum("od,bld->bol", mod.in_proj.weight, hs)
        x, z = xz.chunk(2, dim=1)
        conv_state.copy_(F.pad(x, (mod.d_conv - x.shape[-1], 0)))
        x_act = F.silu(mod.conv1d(x)[..., :prefill])
        x_dbl = mod.x_proj(x_act.transpose(1, 2).reshape(-1, mod.d_inner))
        dt, Bm, Cm = torch.split(x_dbl, [mod.dt_rank, mod.d_state, mod.d_state], dim=-1)
        dt = (mod.dt_proj.weight @ dt.t()).reshape(mod.d_inner, batch, prefill).permute(1, 0, 2)
        Bm = Bm.reshape(batch, prefill, -1).transpose(1, 2).contiguous()
        Cm = Cm.reshape(batch, prefill, -1).transpose(1, 2).contiguous()
        A = -torch.exp(mod.A_log.float())
        _, last = msm.selective_scan_fn(x_act, dt, A, Bm, Cm, mod.D.float(), z=z,
                                        delta_bias=mod.dt_proj.bias.float(), delta_softplus=True,
                                        return_last_state=True, **pq)
        ssm_state.copy_(last)
        conv0, ssm0 = conv_state.clone(), ssm_state.clone()
        step_in, step_out = [], []
        for _ in range(steps):
            h1 = torch.randn(batch, 1, d_model, generator=g)
            o, _, _ = mod.step(h1, conv_state, ssm_state)
            step_in.append(h1)
            step_out.append(o)
    rec = dict(name=name, kind="module", config=dict(d_model=d_model, d_state=d_state, d_conv=4, expand=2,
                                                     pq_rank=pq_rank, pq_per_dim=pq_per_dim),
               state_dict={k: v.clone() for k, v in mod.state_dict().items()},
               hidden=hs, y_prefill=y_prefill, conv_state0=conv0, ssm_state0=ssm0,
               step_in=torch.stack(step_in), step_out=torch.stack(step_out),
               conv_state_final=conv_state.clone(), ssm_state_final=ssm_state.clone())
    torch.save(rec, os.path.join(HERE, f"module_{name}.pt"))
    print("wrote module", name)


def load_motif_reference():
    """The reference's ``motifRegular`` class and ``compute_model_motif_loss`` function, taken
    out of its training script (``motif/train_kpq_motif_pile_lm.py:405-466, 590-642``) by
    ``ast`` and executed alone: the script's other top-level code (argument parsing, data,
    distributed setup) is not run."""
    import ast
    path = os.path.join(REF, "motif/train_kpq_motif_pile_lm.py")
    src = open(path).read()
    tree = ast.parse(src)
    keep = [n for n in tree.body if getattr(n, "name", None) in ("motifRegular", "compute_model_motif_loss")]
    assert len(keep) == 2, "motifRegular / compute_model_motif_loss not found"
    ns = {"torch": torch}
    exec(compile(ast.Module(body=keep, type_ignores=[]), path, "exec"), ns)
    return ns


def motif_case(ns, name, *, n_mat, cc, scale, amplitude, bias, fre, loss_form="mse", loss_weights=None,
               seed=0):
    """Loss, densities and d loss / d a of the reference's motifRegular.cal, matrix by matrix."""
    g = torch.Generator().manual_seed(seed)
    mats = scale * torch.randn(n_mat, cc, cc, generator=g)
    reg = ns["motifRegular"](fre, device="cpu", cc=cc, loss_form=loss_form, loss_weights=loss_weights)
    losses, obs, grads = [], [], []
    for i in range(n_mat):
        a = mats[i].clone().requires_grad_(True)
        r, o = reg.cal(a, amplitude=amplitude, bias=bias)
        r.backward()
        losses.append(r.detach().clone())
        obs.append(o.detach().clone())
        grads.append(a.grad.detach().clone())
    rec = dict(name=name, kind="motif", mats=mats, cc=cc, amplitude=amplitude, bias=bias,
               fre=torch.tensor(fre, dtype=torch.float32), loss_form=loss_form, loss_weights=loss_weights,
               loss=torch.stack(losses), obs=torch.stack(obs), grad=torch.stack(grads))
    torch.save(rec, os.path.join(HERE, f"motif_{name}.pt"))
    print("wrote motif", name, n_mat, cc)


def main():
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    ssi, msm = load_reference()
    # BASELINE config 0 exactly (fp32, 2x64x256, n16, z, softplus, last_state, seed 0).
    scan_case(ssi, "cfg0", batch=2, dim=64, seqlen=256, dstate=16, seed=0)
    scan_case(ssi, "plain_ragged", batch=2, dim=8, seqlen=37, dstate=16, has_z=False,
              has_bias=False, softplus=False, seed=1)
    scan_case(ssi, "groups2_n8", batch=1, dim=8, seqlen=64, dstate=8, groups=2, seed=2)
    scan_case(ssi, "bf16", batch=2, dim=16, seqlen=300, dstate=16, dtype=torch.bfloat16, seed=3)
    scan_case(ssi, "n4_L1", batch=2, dim=4, seqlen=1, dstate=4, seed=4)
    scan_case(ssi, "long2100", batch=1, dim=2, seqlen=2100, dstate=16, seed=5)
    scan_case(ssi, "noD_n32", batch=1, dim=4, seqlen=70, dstate=32, has_D=False, seed=6)
    scan_case(ssi, "pq2_shared", batch=2, dim=16, seqlen=300, dstate=16, pq_rank=2, seed=7)
    scan_case(ssi, "pq4_perdim_noz", batch=1, dim=8, seqlen=70, dstate=8, pq_rank=4, pq_per_dim=True,
              has_z=False, seed=8)
    inner_case(ssi, "small")
    module_case(msm, "small")
    module_case(msm, "pq2", pq_rank=2, seed=3, pq_k=40.0)
    module_case(msm, "pq3_perdim", d_state=16, pq_rank=3, pq_per_dim=True, seed=4)
    ns = load_motif_reference()
    mavgf = [0.0455015, 0.1438295, 0.0891085, 0.053934, -1, -1, -1, -1, -1, -1, 0.065183, 0.1245175, 0.0]
    single2 = [-1.0] * 13
    single2[1] = 0.25  # --motif-class 2, the script's default
    # the script's default amplitude / bias, matrices around the threshold sqrt(bias)
    motif_case(ns, "default_class2", n_mat=6, cc=16, scale=0.01, amplitude=1e5, bias=5e-5, fre=single2, seed=11)
    motif_case(ns, "mavgf_weighted", n_mat=5, cc=16, scale=0.01, amplitude=1e5, bias=5e-5, fre=mavgf,
               loss_weights=[1.0, 2.0, 0.5, 1.0, 1, 1, 1, 1, 1, 1, 3.0, 0.25, 1], seed=12)
    motif_case(ns, "log_mse_cc8", n_mat=4, cc=8, scale=1.0, amplitude=4.0, bias=0.5, fre=mavgf,
               loss_form="log_mse", seed=13)
    motif_case(ns, "soft_cc32", n_mat=2, cc=32, scale=1.0, amplitude=2.0, bias=0.8, fre=mavgf, seed=14)


if __name__ == "__main__":
    main()
