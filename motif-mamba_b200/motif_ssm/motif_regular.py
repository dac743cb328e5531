"""Motif regulariser of the P/Q coupling on ``libmotif_ssm.so``.

Drop-in for the training script's ``motifRegular`` and ``compute_model_motif_loss``
(``motif/train_kpq_motif_pile_lm.py:405-466, 590-642``).  For a cc x cc matrix ``a``
(``P_eff @ Q``; cc = d_state) the regulariser reads ``w = sigmoid(amplitude (a^2 - bias))``
(diagonal zeroed) as a soft directed graph, counts the 13 connected three-node motifs
through products of ``w``, ``1 - w`` and their transposes, divides by cc (cc-1) (cc-2) / 6
and penalises the squared (or log-squared) distance to target densities.

The reference evaluates one matrix per ``cal`` call with ~60 small torch kernels and, in
per-channel mode, a host sync per sampled channel.  Here one ``motif_regular`` launch
evaluates every matrix of every layer (forward), and one more gives all gradients
(analytic backward, recomputing the forward in the same kernel).  There is no CPU path:
the matrices must be CUDA fp32 tensors.
"""
import ctypes

import torch

from . import _lib
from ._lib import lib, check
from .selective_scan_cuda import _ptr, _stream

N_MOTIFS = 13


def _launch(a, target, weight, amplitude, bias, log_mse, log_eps, dloss=None):
    M, cc = a.shape[0], a.shape[-1]
    loss = torch.empty(M, dtype=torch.float32, device=a.device)
    obs = torch.empty(M, N_MOTIFS + 1, dtype=torch.float32, device=a.device)
    args = _lib.MotifRegularArgs()
    args.n_mat, args.cc = M, cc
    args.a, args.a_ms = _ptr(a), a.stride(0)
    args.target = _ptr(target)
    args.weight = _ptr(weight) if weight is not None else None
    args.amplitude, args.bias = float(amplitude), float(bias)
    args.log_mse, args.log_eps = int(bool(log_mse)), float(log_eps)
    args.loss, args.obs = _ptr(loss), _ptr(obs)
    da = None
    if dloss is not None:
        da = torch.empty_like(a)
        args.dloss = _ptr(dloss)
        args.da, args.da_ms = _ptr(da), da.stride(0)
    with torch.cuda.device(a.device):
        check(lib.motif_regular(ctypes.byref(args), _stream(a.device)))
    return loss, obs, da


def _prep(a, target, weight):
    if not a.is_cuda:
        raise RuntimeError("motif_regular: the matrices must be CUDA tensors (no CPU path)")
    if a.dim() != 3 or a.shape[1] != a.shape[2]:
        raise ValueError(f"motif_regular: expected (n, cc, cc) matrices, got {tuple(a.shape)}")
    a = a.float().contiguous()
    target = target.to(device=a.device, dtype=torch.float32).contiguous()
    if target.numel() != N_MOTIFS:
        raise ValueError("motif_regular: target must hold 13 values")
    if weight is not None:
        weight = weight.to(device=a.device, dtype=torch.float32).contiguous()
        if weight.numel() != N_MOTIFS:
            raise ValueError("motif_regular: loss weights must hold 13 values")
    return a, target, weight


class MotifRegularFn(torch.autograd.Function):
    """(n, cc, cc) matrices -> per-matrix loss (n,) and motif densities (n, 14) (no gradient)."""

    @staticmethod
    def forward(ctx, a, target, weight, amplitude, bias, log_mse, log_eps):
        a, target, weight = _prep(a, target, weight)
        loss, obs, _ = _launch(a, target, weight, amplitude, bias, log_mse, log_eps)
        ctx.save_for_backward(a, target, weight)
        ctx.cfg = (amplitude, bias, log_mse, log_eps)
        ctx.mark_non_differentiable(obs)
        return loss, obs

    @staticmethod
    def backward(ctx, dloss, dobs):
        a, target, weight = ctx.saved_tensors
        if dloss is None:
            return (None,) * 7
        _, _, da = _launch(a, target, weight, *ctx.cfg, dloss=dloss.float().contiguous())
        return da, None, None, None, None, None, None


def motif_regular_batched(a, target, amplitude, bias, weight=None, loss_form="mse", log_eps=1e-12):
    """Loss (n,) and densities (n, 14) of a batch of matrices, differentiable in ``a``."""
    if loss_form not in ("mse", "log_mse"):
        # the reference treats every other string as mse (train_kpq_motif_pile_lm.py:452-458)
        loss_form = "mse"
    return MotifRegularFn.apply(a, target, weight, amplitude, bias, loss_form == "log_mse", log_eps)


class motifRegular:
    """Same constructor, attributes and ``cal`` as the reference's class
    (``motif/train_kpq_motif_pile_lm.py:405-466``); ``cal`` runs the kernel.

    ``cal`` returns ``(loss, self.obs)`` where ``self.obs`` is the SAME tensor every call,
    overwritten in place with the newest densities, as in the reference.
    """

    def __init__(self, fre, device="cuda", cc=16, loss_form: str = "mse", log_eps: float = 1e-12, loss_weights=None):
        self.device = device
        self.L = torch.ones([1, cc], device=self.device)
        self.P = 1.0 - torch.eye(cc, device=self.device)
        self.obs = torch.zeros([14], requires_grad=False, device=self.device)
        self.fre = torch.zeros([13], device=self.device)
        self.loss_form = str(loss_form)
        self.log_eps = float(log_eps)
        if loss_weights is None:
            self.loss_weights = torch.ones([13], device=self.device)
        else:
            if len(loss_weights) != 13:
                raise ValueError("loss_weights must have length 13")
            self.loss_weights = torch.tensor(loss_weights, device=self.device, dtype=torch.float32)
        self.cc = int(cc)
        self.sum = int(cc * (cc - 1) * (cc - 2) / 6)
        for i in range(13):
            self.fre[i] = fre[i]

    def cal_batched(self, a, amplitude, bias):
        """Loss (n,) and densities (n, 14) of n matrices in one launch; ``self.obs`` takes
        the last matrix's densities (what n successive ``cal`` calls leave there)."""
        if a.shape[-2:] != (self.cc, self.cc):
            raise ValueError(f"motifRegular: expected {self.cc} x {self.cc} matrices, got {tuple(a.shape)}")
        loss, obs = motif_regular_batched(a, self.fre, amplitude, bias, weight=self.loss_weights,
                                          loss_form=self.loss_form, log_eps=self.log_eps)
        if obs.shape[0] > 0:
            with torch.no_grad():
                self.obs.copy_(obs[-1])
        return loss, obs

    def cal(self, a, amplitude, bias):
        loss, _ = self.cal_batched(a.unsqueeze(0), amplitude, bias)
        return loss[0], self.obs


MotifRegular = motifRegular


def compute_model_motif_loss(model, motif_regularizer, amplitude, bias, per_dim_mode="sampled_channel",
                             channel_samples=16, only_layer=-1):
    """Mean motif loss over the coupled layers and their mean densities, as the reference's
    ``compute_model_motif_loss`` (``motif/train_kpq_motif_pile_lm.py:590-642``), with every
    matrix of every layer in one kernel launch.

    Same module walk, layer filter, ``P_eff = pq_k * P``, channel sampling
    (``torch.randperm`` per per-channel layer, in module order, so the RNG stream matches)
    and averaging.  The densities follow the reference's aliasing of ``motifRegular.obs``:
    a per-channel layer contributes the densities of its last sampled channel, and every
    shared-matrix (or ``mean_matrix``) layer contributes the densities of the very last
    matrix evaluated.
    """
    mats, layers = [], []  # layers: (start, count, per_channel)
    n = 0
    layer_filter = int(only_layer)
    for module_name, module in model.named_modules():
        if layer_filter >= 0 and f".layers.{layer_filter}.mixer" not in module_name:
            continue
        P = getattr(module, "P", None)
        Q = getattr(module, "Q", None)
        if P is None or Q is None:
            continue
        pq_k = getattr(module, "pq_k", None)
        P_eff = P if pq_k is None else (pq_k * P)
        pq_square = torch.matmul(P_eff.float(), Q.float())
        if pq_square.dim() == 3 and per_dim_mode != "mean_matrix":
            d_inner = int(pq_square.shape[0])
            n_sample = d_inner if channel_samples <= 0 else min(int(channel_samples), d_inner)
            if n_sample == d_inner:
                blk = pq_square
            else:
                idx = torch.randperm(d_inner, device=pq_square.device)[:n_sample]
                blk = pq_square.index_select(0, idx)
            mats.append(blk)
            layers.append((n, n_sample, True))
            n += n_sample
        else:
            m = pq_square.mean(dim=0) if pq_square.dim() == 3 else pq_square
            mats.append(m.unsqueeze(0))
            layers.append((n, 1, False))
            n += 1
    if len(mats) == 0:
        raise RuntimeError("No motif-compatible blocks (with P/Q) found.")
    loss_all, obs_all = motif_regularizer.cal_batched(torch.cat(mats, dim=0), amplitude, bias)
    losses, obs = [], []
    for start, count, per_channel in layers:
        losses.append(loss_all[start:start + count].mean() if per_channel else loss_all[start])
        obs.append(obs_all[start + count - 1] if per_channel else obs_all[-1])
    return torch.stack(losses).mean(), torch.stack(obs).mean(dim=0)
