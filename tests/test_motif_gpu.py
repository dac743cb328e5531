"""Motif regulariser kernel (motif_regular) against the reference's own outputs (golden) and
the oracle restatement: loss, densities and gradients, one matrix or whole models at once."""
import glob
import os

import pytest
import torch
import torch.nn as nn

from oracle import motif_oracle as MO

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"
# fp32 kernel vs fp32 torch: sums of cc^2 products in a different order
RTOL, ATOL = 1e-4, 1e-6


def _grad_close(got, want):
    torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-4 * (want.abs().max().item() + 1e-9))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "motif_*.pt"))),
                         ids=lambda p: os.path.basename(p))
def test_kernel_matches_reference_fixture(path):
    from motif_ssm.motif_regular import motifRegular
    rec = torch.load(path, weights_only=False)
    reg = motifRegular(rec["fre"].tolist(), device=DEV, cc=rec["cc"], loss_form=rec["loss_form"],
                       loss_weights=rec["loss_weights"])
    a = rec["mats"].to(DEV).requires_grad_(True)
    loss, obs = reg.cal_batched(a, amplitude=rec["amplitude"], bias=rec["bias"])
    torch.testing.assert_close(loss.cpu(), rec["loss"], rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(obs.cpu(), rec["obs"], rtol=RTOL, atol=ATOL)
    loss.sum().backward()
    _grad_close(a.grad.cpu(), rec["grad"])
    # the single-matrix call: same results, and obs is the regulariser's own buffer
    r, o = reg.cal(rec["mats"][-1].to(DEV), amplitude=rec["amplitude"], bias=rec["bias"])
    assert o is reg.obs
    torch.testing.assert_close(r.cpu(), rec["loss"][-1], rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(o.cpu(), rec["obs"][-1], rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("cc", [3, 5, 16, 17, 31, 32])
@pytest.mark.parametrize("loss_form", ["mse", "log_mse"])
def test_batched_kernel_matches_oracle(cc, loss_form):
    from motif_ssm.motif_regular import motif_regular_batched
    g = torch.Generator().manual_seed(cc)
    mats = torch.randn(7, cc, cc, generator=g)
    fre = torch.rand(13, generator=g) * 0.3
    fre[[2, 5, 9]] = -1.0
    fre[7] = 0.0  # zero targets are skipped, as negative ones
    wts = torch.rand(13, generator=g) + 0.5
    amp, bias = 3.0, 0.6
    a = mats.to(DEV).requires_grad_(True)
    loss, obs = motif_regular_batched(a, fre, amp, bias, weight=wts, loss_form=loss_form)
    dl = torch.randn(7, generator=g)
    (loss * dl.to(DEV)).sum().backward()
    for i in range(7):
        ai = mats[i].clone().requires_grad_(True)
        r, o = MO.motif_regular_ref(ai, fre, amp, bias, loss_form, loss_weights=wts)
        (r * dl[i]).backward()
        torch.testing.assert_close(loss[i].detach().cpu(), r.detach(), rtol=RTOL, atol=ATOL)
        torch.testing.assert_close(obs[i].cpu(), o, rtol=RTOL, atol=ATOL)
        _grad_close(a.grad[i].cpu(), ai.grad)


def test_batched_kernel_many_matrices_and_strided_view():
    """A large batch (every channel of a 24-layer 1536-channel model) through a non-contiguous view."""
    from motif_ssm.motif_regular import motif_regular_batched
    torch.manual_seed(0)
    big = 0.01 * torch.randn(3000, 16, 20, device=DEV)
    a = big[:, :, 2:18]  # (3000, 16, 16) view, row stride 20
    fre = torch.full((13,), -1.0)
    fre[1] = 0.25
    loss, obs = motif_regular_batched(a, fre, 1e5, 5e-5)
    pick = [0, 1, 1499, 2999]
    for i in pick:
        r, o = MO.motif_regular_ref(a[i].cpu(), fre, 1e5, 5e-5)
        torch.testing.assert_close(loss[i].cpu(), r, rtol=RTOL, atol=ATOL)
        torch.testing.assert_close(obs[i].cpu(), o, rtol=RTOL, atol=ATOL)


class _Layer(nn.Module):
    def __init__(self, mixer):
        super().__init__()
        self.mixer = mixer


def _model(per_dim_layers):
    from motif_ssm.modules import Mambamotif
    torch.manual_seed(5)
    layers = []
    for i, per_dim in enumerate(per_dim_layers):
        m = Mambamotif(d_model=16, d_state=16, layer_idx=i, pq_rank=2, pq_per_dim=per_dim, device=DEV)
        with torch.no_grad():
            m.P.copy_(torch.randn_like(m.P))
            m.Q.copy_(torch.randn_like(m.Q))
            m.pq_k.fill_(0.005)
        layers.append(_Layer(m))
    root = nn.Module()
    root.backbone = nn.Module()
    root.backbone.layers = nn.ModuleList(layers)
    return root


@pytest.mark.parametrize("mode,samples,only_layer", [
    ("sampled_channel", 16, -1), ("sampled_channel", 0, -1), ("mean_matrix", 16, -1), ("sampled_channel", 5, 1)])
def test_compute_model_motif_loss_matches_oracle(mode, samples, only_layer):
    from motif_ssm.motif_regular import compute_model_motif_loss, motifRegular
    model = _model([True, False, True])
    fre = [0.0455015, 0.1438295, 0.0891085, 0.053934, -1, -1, -1, -1, -1, -1, 0.065183, 0.1245175, 0.0]
    reg = motifRegular(fre, device=DEV)
    params = [p for n, p in model.named_parameters() if n.endswith((".P", ".Q", ".pq_k"))]
    rng = torch.cuda.get_rng_state()
    loss, obs = compute_model_motif_loss(model, reg, 1e5, 5e-5, per_dim_mode=mode, channel_samples=samples,
                                         only_layer=only_layer)
    loss.backward()
    got = [None if p.grad is None else p.grad.clone() for p in params]
    for p in params:
        p.grad = None
    torch.cuda.set_rng_state(rng)
    mods = [(n, m) for n, m in model.named_modules()
            if only_layer < 0 or f".layers.{only_layer}.mixer" in n]
    rl, ro = MO.compute_model_motif_loss_ref(mods, fre, 1e5, 5e-5, per_dim_mode=mode, channel_samples=samples)
    rl.backward()
    torch.testing.assert_close(loss.detach().cpu(), rl.detach(), rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(obs.cpu(), ro, rtol=RTOL, atol=ATOL)
    for g, p in zip(got, params):
        if p.grad is None or g is None:
            assert (g is None or g.abs().max().item() == 0.0) and (p.grad is None or p.grad.abs().max().item() == 0.0)
            continue
        _grad_close(g, p.grad)
    assert reg.obs.shape == (14,) and reg.obs.is_cuda


def test_no_coupled_layers_raises():
    from motif_ssm.motif_regular import compute_model_motif_loss, motifRegular
    with pytest.raises(RuntimeError):
        compute_model_motif_loss(nn.Linear(2, 2).to(DEV), motifRegular([0.25] * 13, device=DEV), 1e5, 5e-5)
