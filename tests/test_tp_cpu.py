"""Channel-sharded tensor parallelism: 2 gloo ranks on the CPU reproduce the unsharded
mixer stack.  The CUDA kernels are replaced by the CPU oracle inside the ranks (the test
covers the sharding and the two all-reduces, not the kernels)."""
import os
import sys
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _patch_ops():
    from oracle import ssm_oracle as O
    from motif_ssm import modules

    def conv(x, w, b=None, activation=None):
        return O.causal_conv1d_ref(x, w, b, activation)

    def scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False, return_last_state=False,
             P=None, Q=None, gamma=None):
        return O.selective_scan_ref(u, delta, A, B, C, D, z=z, delta_bias=delta_bias,
                                    delta_softplus=delta_softplus, return_last_state=return_last_state, P=P, Q=Q)

    def inner(*a, **k):
        return O.mamba_inner_ref(*a, **{kk: v for kk, v in k.items() if kk != "checkpoint_lvl"})

    def scan_chunk(u, delta, A, B, C, D, z, delta_bias, h0, P=None, Q=None):
        """The gated scan of a chunk from state h0: the oracle from zero plus h0's decayed
        contribution (y_t += sum_n C_tn exp(A_n sum_{s<=t} dt_s) h0_n), gated afterwards."""
        if P is not None:
            assert h0 is None
            return O.selective_scan_ref(u, delta, A, B, C, D, z=z, delta_bias=delta_bias, delta_softplus=True,
                                        return_last_state=True, P=P, Q=Q)
        out, last = O.selective_scan_ref(u, delta, A, B, C, D, z=None, delta_bias=delta_bias,
                                         delta_softplus=True, return_last_state=True)
        if h0 is not None:
            dt = torch.nn.functional.softplus(delta.float() + delta_bias[:, None])
            dec = torch.exp(A[None, :, None, :] * torch.cumsum(dt, dim=-1)[..., None])  # (b, d, l, n)
            out = out + torch.einsum("bnl,bdln,bdn->bdl", C.float(), dec, h0)
            last = last + dec[:, :, -1] * h0
        return out * torch.nn.functional.silu(z.float()), last

    modules.causal_conv1d_fn = conv
    modules.selective_scan_fn = scan
    modules.mamba_inner_fn = inner
    modules._scan_chunk = scan_chunk
    return modules


def _worker(rank, world, port, q, pq_rank=0, pq_per_dim=False, n_chunks=0):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "motif-mamba_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        modules = _patch_ops()
        torch.manual_seed(0)
        model = modules.MambaLMHeadModel(modules.MambaConfig(
            d_model=32, n_layer=2, vocab_size=40,
            ssm_cfg={"d_state": 8, "pq_rank": pq_rank, "pq_per_dim": pq_per_dim}))
        if pq_rank:  # a coupling strong enough to change the outputs
            g = torch.Generator().manual_seed(3)
            with torch.no_grad():
                for layer in model.backbone.layers:
                    layer.mixer.pq_k.fill_(20.0)
                    layer.mixer.P.copy_(0.5 * torch.randn(layer.mixer.P.shape, generator=g))
                    layer.mixer.Q.copy_(0.5 * torch.randn(layer.mixer.Q.shape, generator=g))
        ids = torch.randint(0, 40, (2, 150 if n_chunks else 24))
        with torch.no_grad():
            ref = model(ids)
            modules.shard_model_tp(model, rank, world)
            out = modules.tp_prefill(model, ids, n_chunks=n_chunks, num_last_tokens=0) if n_chunks else model(ids)
        q.put((rank, (out - ref).abs().max().item(), ref.abs().max().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("pq_rank,pq_per_dim", [(0, False), (2, False), (2, True)],
                         ids=["plain", "pq_shared", "pq_per_channel"])
def test_tp2_gloo_matches_unsharded(pq_rank, pq_per_dim):
    """Also with the motif P/Q coupling: a per-channel P / Q is sliced with the channels,
    a shared one replicated."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, pq_rank, pq_per_dim)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, scale in res:
        assert err <= 1e-4 * max(1.0, scale), (rank, err, scale)


def test_tp2_gloo_chunked_prefill_matches_unsharded():
    """tp_prefill: the sequence in 3 chunks (64, 64, 22 steps) carried through the conv halo and
    the scan state, out_proj all-reduces issued asynchronously."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, 0, False, 3)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, scale in res:
        assert err <= 1e-4 * max(1.0, scale), (rank, err, scale)


def _grad_worker(rank, world, port, q):
    """Training through the shards: loss = sum(logits * W) for a fixed W; the sharded
    parameters' gradients must equal the matching slices of the unsharded model's."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "motif-mamba_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        modules = _patch_ops()
        torch.manual_seed(0)
        model = modules.MambaLMHeadModel(modules.MambaConfig(d_model=32, n_layer=2, vocab_size=40,
                                                             ssm_cfg={"d_state": 8}))
        g = torch.Generator().manual_seed(1)
        ids = torch.randint(0, 40, (2, 24), generator=g)
        wl = torch.randn(2, 24, 40, generator=g)
        ref_logits = model(ids)
        (ref_logits * wl).sum().backward()
        full = [(layer.mixer.d_inner, {k: v.grad.clone() for k, v in layer.mixer.named_parameters()})
                for layer in model.backbone.layers]
        emb_ref = model.backbone.embedding.weight.grad.clone()
        model.zero_grad()
        modules.shard_model_tp(model, rank, world)
        logits = model(ids)
        (logits * wl).sum().backward()
        errs = {"logits": ((logits - ref_logits).abs().max().item(), ref_logits.abs().max().item()),
                "embedding": ((model.backbone.embedding.weight.grad - emb_ref).abs().max().item(),
                              emb_ref.abs().max().item())}
        for i, (layer, (di, gr)) in enumerate(zip(model.backbone.layers, full)):
            m, dl = layer.mixer, di // world
            lo, hi = rank * dl, (rank + 1) * dl
            want = {"in_proj_w": torch.cat([gr["in_proj.weight"][lo:hi], gr["in_proj.weight"][di + lo:di + hi]]),
                    "conv_w": gr["conv1d.weight"][lo:hi, 0], "conv_b": gr["conv1d.bias"][lo:hi],
                    "x_proj_w": gr["x_proj.weight"][:, lo:hi], "dt_proj_w": gr["dt_proj.weight"][lo:hi],
                    "dt_proj_b": gr["dt_proj.bias"][lo:hi], "A_log": gr["A_log"][lo:hi], "D": gr["D"][lo:hi],
                    "out_proj_w": gr["out_proj.weight"][:, lo:hi]}
            for k, w in want.items():
                got = getattr(m, k).grad
                errs[f"layer{i}.{k}"] = ((got - w.to(got.dtype)).abs().max().item(), w.abs().max().item())
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def test_tp2_gloo_backward_matches_unsharded():
    """Sharded training step (autograd through the shards and both all-reduces) against the
    unsharded model: logits, every sharded parameter's gradient slice and the replicated
    embedding's gradient, on 2 gloo ranks."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_grad_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs in res:
        for k, (err, scale) in errs.items():
            assert err <= 1e-4 * max(1.0, scale), (rank, k, err, scale)
