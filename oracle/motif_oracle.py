"""CPU oracle for the motif regulariser.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import
this module, as the checker / the timed CPU reference; the product never does.

Plain-torch restatement (fp32 unless the caller passes fp64) of the reference's
``motifRegular`` (``motif/train_kpq_motif_pile_lm.py:405-466``) and
``compute_model_motif_loss`` (``:590-642``), one matrix at a time as the reference does.
Gradients come from torch autograd through the restatement.

Parity pinning: ``tests/test_oracle_golden.py`` checks ``motif_regular_ref`` against
fixtures produced by the reference's own class (``tests/golden/make_golden.py``).
"""
import torch

# (a, b, c, coef) of q_k = coef * sum(X_a o (X_b @ X_c)), k = 1..13, with
# X0 = m o m^T, X1 = w o m^T, X2 = m o w^T, X3 = w o w^T (train_kpq_motif_pile_lm.py:434-450).
TERMS = [
    (1, 1, 0, 0.5), (0, 1, 2, 0.5), (1, 0, 2, 1.0), (1, 1, 2, 1.0), (3, 1, 0, 1.0),
    (3, 2, 0, 1.0), (3, 1, 2, 0.5), (3, 2, 1, 0.5), (3, 3, 0, 0.5), (1, 2, 2, 1.0 / 3.0),
    (3, 2, 2, 1.0), (3, 3, 2, 1.0), (3, 3, 3, 1.0 / 6.0),
]


def motif_densities_ref(a, amplitude, bias):
    """The 13 motif densities q_k / (cc (cc-1) (cc-2) / 6) of one cc x cc matrix (:427-450)."""
    cc = a.shape[-1]
    off = 1.0 - torch.eye(cc, dtype=a.dtype, device=a.device)
    w = torch.sigmoid(amplitude * (a * a - bias)) * off
    m = off - w
    X = [m * m.T, w * m.T, m * w.T, w * w.T]
    ncomb = int(cc * (cc - 1) * (cc - 2) / 6)
    return torch.stack([coef * (X[ia] * (X[ib] @ X[ic])).sum() for ia, ib, ic, coef in TERMS]) / ncomb


def motif_regular_ref(a, fre, amplitude, bias, loss_form="mse", log_eps=1e-12, loss_weights=None):
    """(loss, obs[14]) of one matrix (:427-466): targets <= 0 are skipped; obs[0] = 0."""
    obs = motif_densities_ref(a, amplitude, bias)
    fre = torch.as_tensor(fre, dtype=a.dtype).cpu()
    wts = torch.ones(13, dtype=a.dtype) if loss_weights is None else torch.as_tensor(loss_weights, dtype=a.dtype)
    wts = wts.to(a.device)
    r = torch.zeros((), dtype=a.dtype, device=a.device)
    for i in range(13):
        if fre[i] > 0:
            if loss_form == "log_mse":
                diff = torch.log(torch.clamp(obs[i], min=log_eps)) - torch.log(torch.clamp(fre[i], min=log_eps))
            else:
                diff = obs[i] - fre[i]
            r = r + wts[i] * diff ** 2
    return r, torch.cat([torch.zeros(1, dtype=a.dtype, device=a.device), obs.detach()])


def compute_model_motif_loss_ref(modules, fre, amplitude, bias, per_dim_mode="sampled_channel",
                                 channel_samples=16, loss_form="mse", log_eps=1e-12, loss_weights=None):
    """Module walk of :590-642 over ``modules`` (name, module) pairs with P / Q / pq_k.

    Channel sampling calls ``torch.randperm`` on the matrices' device in the same order as
    the reference.  Densities follow the reference's aliasing of the regulariser's ``obs``
    buffer: a per-channel layer contributes its last channel's, a shared-matrix layer the
    final matrix's.
    """
    losses, obs, last = [], [], [None]
    shared_slots = []

    def cal(x):
        r, o = motif_regular_ref(x.cpu().float(), fre, amplitude, bias, loss_form, log_eps, loss_weights)
        last[0] = o
        return r

    for _, module in modules:
        P, Q = getattr(module, "P", None), getattr(module, "Q", None)
        if P is None or Q is None:
            continue
        pq_k = getattr(module, "pq_k", None)
        P_eff = P if pq_k is None else (pq_k * P)
        pq_square = torch.matmul(P_eff.float(), Q.float())
        if pq_square.dim() == 3 and per_dim_mode != "mean_matrix":
            d_inner = int(pq_square.shape[0])
            n_sample = d_inner if channel_samples <= 0 else min(int(channel_samples), d_inner)
            if n_sample == d_inner:
                idx = torch.arange(d_inner, device=pq_square.device)
            else:
                idx = torch.randperm(d_inner, device=pq_square.device)[:n_sample]
            blk = [cal(pq_square[int(c.item())]) for c in idx]
            losses.append(torch.stack(blk).mean())
            obs.append(last[0].clone())
        else:
            x = pq_square.mean(dim=0) if pq_square.dim() == 3 else pq_square
            losses.append(cal(x))
            shared_slots.append(len(obs))
            obs.append(None)
    if not losses:
        raise RuntimeError("No motif-compatible blocks (with P/Q) found.")
    for s in shared_slots:
        obs[s] = last[0]
    return torch.stack(losses).mean(), torch.stack(obs).mean(dim=0)
