"""Pin the CPU oracle against fixtures produced by the reference's own code."""
import glob
import os

import pytest
import torch

from oracle import ssm_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(path):
    return torch.load(path, weights_only=False)


def _tol(dtype):
    return (1e-5, 1e-5) if dtype == torch.float32 else (1e-2, 1e-2)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "scan_*.pt"))),
                         ids=lambda p: os.path.basename(p))
def test_scan_oracle_matches_reference(path):
    rec = _load(path)
    inp = rec["inputs"]
    out, last, grads = O.scan_with_grads(inp, rec["dout"], rec["softplus"])
    rtol, atol = _tol(inp["u"].dtype)
    torch.testing.assert_close(out, rec["out"], rtol=rtol, atol=atol)
    torch.testing.assert_close(last, rec["last_state"], rtol=1e-5, atol=1e-5)
    for k, g in rec["grads"].items():
        if g is None:
            assert grads[k] is None
            continue
        scale = g.float().abs().max().item() + 1e-6
        torch.testing.assert_close(grads[k].float(), g.float(), rtol=rtol, atol=atol * scale,
                                   msg=lambda m: f"grad {k}: {m}")


def test_inner_oracle_matches_reference():
    rec = _load(os.path.join(GOLD, "inner_small.pt"))
    leaves = {k: v.clone().requires_grad_(True) for k, v in rec["inputs"].items()}
    out = O.mamba_inner_ref(leaves["xz"], leaves["conv1d_weight"], leaves["conv1d_bias"],
                            leaves["x_proj_weight"], leaves["delta_proj_weight"],
                            leaves["out_proj_weight"], leaves["out_proj_bias"], leaves["A"],
                            None, None, leaves["D"], delta_bias=leaves["delta_bias"])
    torch.testing.assert_close(out, rec["out"], rtol=1e-5, atol=1e-5)
    out.backward(rec["dout"])
    for k, g in rec["grads"].items():
        torch.testing.assert_close(leaves[k].grad, g, rtol=1e-4, atol=1e-4 * (g.abs().max().item() + 1e-6))


def test_module_step_oracle_matches_reference():
    """Conv-update + state-update restatements reproduce Mambamotif.step's torch fallback."""
    rec = _load(os.path.join(GOLD, "module_small.pt"))
    sd = rec["state_dict"]
    conv_state = rec["conv_state0"].clone()
    ssm_state = rec["ssm_state0"].clone()
    W = sd["conv1d.weight"][:, 0, :]
    dt_rank = sd["dt_proj.weight"].shape[1]
    n = sd["A_log"].shape[1]
    A = -torch.exp(sd["A_log"].float())
    for i in range(rec["step_in"].shape[0]):
        hs = rec["step_in"][i][:, 0]
        xz = hs @ sd["in_proj.weight"].t()
        x, z = xz.chunk(2, dim=-1)
        x = O.causal_conv1d_update_ref(x, conv_state, W, sd["conv1d.bias"], "silu")
        x_db = x @ sd["x_proj.weight"].t()
        dt, B, C = torch.split(x_db, [dt_rank, n, n], dim=-1)
        dt = dt @ sd["dt_proj.weight"].t()
        y = O.selective_state_update_ref(ssm_state, x, dt, A, B, C, sd["D"], z=z,
                                         dt_bias=sd["dt_proj.bias"], dt_softplus=True)
        out = y @ sd["out_proj.weight"].t()
        torch.testing.assert_close(out, rec["step_out"][i][:, 0], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(conv_state, rec["conv_state_final"])
    torch.testing.assert_close(ssm_state, rec["ssm_state_final"], rtol=1e-5, atol=1e-5)


def test_module_prefill_oracle_matches_reference():
    """Block prefill (mamba_simplemotif.py:256-335, slow path) == mamba_inner_ref restatement."""
    rec = _load(os.path.join(GOLD, "module_small.pt"))
    sd = rec["state_dict"]
    hs = rec["hidden"]
    xz = torch.einsum("od,bld->bol", sd["in_proj.weight"], hs)
    A = -torch.exp(sd["A_log"].float())
    out = O.mamba_inner_ref(xz, sd["conv1d.weight"], sd["conv1d.bias"], sd["x_proj.weight"],
                            sd["dt_proj.weight"], sd["out_proj.weight"], None, A, None, None,
                            sd["D"].float(), delta_bias=sd["dt_proj.bias"].float())
    torch.testing.assert_close(out, rec["y_prefill"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["pq2", "pq3_perdim"])
def test_module_pq_oracle_matches_reference(name):
    """Mambamotif with the P/Q coupling: slow-path prefill, cache states and decode steps."""
    rec = _load(os.path.join(GOLD, f"module_{name}.pt"))
    sd = rec["state_dict"]
    out, last = O.mixer_pq_prefill_ref(sd, rec["hidden"], return_last_state=True)
    torch.testing.assert_close(out, rec["y_prefill"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(last, rec["ssm_state0"], rtol=1e-5, atol=1e-5)
    conv_state = rec["conv_state0"].clone()
    ssm_state = rec["ssm_state0"].clone()
    for i in range(rec["step_in"].shape[0]):
        o = O.mixer_pq_step_ref(sd, rec["step_in"][i], conv_state, ssm_state)
        torch.testing.assert_close(o, rec["step_out"][i], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(conv_state, rec["conv_state_final"])
    torch.testing.assert_close(ssm_state, rec["ssm_state_final"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "motif_*.pt"))),
                         ids=lambda p: os.path.basename(p))
def test_motif_oracle_matches_reference(path):
    """motif_regular_ref reproduces the reference's motifRegular.cal: loss, densities, d loss / d a."""
    from oracle import motif_oracle as MO
    rec = _load(path)
    for i in range(rec["mats"].shape[0]):
        a = rec["mats"][i].clone().requires_grad_(True)
        r, obs = MO.motif_regular_ref(a, rec["fre"], rec["amplitude"], rec["bias"], rec["loss_form"],
                                      loss_weights=rec["loss_weights"])
        r.backward()
        torch.testing.assert_close(r.detach(), rec["loss"][i], rtol=1e-5, atol=1e-7)
        torch.testing.assert_close(obs, rec["obs"][i], rtol=1e-5, atol=1e-7)
        g = rec["grad"][i]
        torch.testing.assert_close(a.grad, g, rtol=1e-4, atol=1e-5 * (g.abs().max().item() + 1e-9))
