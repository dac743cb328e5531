"""Tensor-parallel mixer stack on 2 GPUs over NCCL (child processes), against the same
model unsharded on GPU 0.  Skipped when fewer than 2 GPUs are visible."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "motif-mamba_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from motif_ssm.modules import MambaConfig, MambaLMHeadModel, shard_model_tp
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        torch.manual_seed(0)
        model = MambaLMHeadModel(MambaConfig(d_model=256, n_layer=2, vocab_size=128, ssm_cfg={"d_state": 16}),
                                 device=dev)
        ids = torch.randint(0, 128, (2, 700), device=dev, generator=torch.Generator(device=dev).manual_seed(1))
        with torch.no_grad():
            ref = model(ids)
            shard_model_tp(model, rank, world)
            out = model(ids)
        torch.cuda.synchronize()
        q.put((rank, (out - ref).abs().max().item(), ref.abs().max().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_nccl_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, scale in res:
        assert err <= 1e-3 * max(1.0, scale), (rank, err, scale)


def _grad_worker(rank, world, port, q):
    """fp32 training step: loss = sum(logits * W); the shards' gradients against the matching
    slices of the unsharded model's (its mixers run mamba_inner_fn, the shards selective_scan_fn,
    the conv and the two NCCL all-reduces with their autograd rules)."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "motif-mamba_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from motif_ssm.modules import MambaConfig, MambaLMHeadModel, shard_model_tp
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        torch.manual_seed(0)
        model = MambaLMHeadModel(MambaConfig(d_model=256, n_layer=2, vocab_size=128, ssm_cfg={"d_state": 16}),
                                 device=dev)
        g = torch.Generator(device=dev).manual_seed(1)
        ids = torch.randint(0, 128, (2, 700), device=dev, generator=g)
        wl = torch.randn(2, 700, 128, device=dev, generator=g)
        (model(ids) * wl).sum().backward()
        full = [(l.mixer.d_inner, {k: v.grad.clone() for k, v in l.mixer.named_parameters()})
                for l in model.backbone.layers]
        emb_ref = model.backbone.embedding.weight.grad.clone()
        model.zero_grad()
        shard_model_tp(model, rank, world)
        (model(ids) * wl).sum().backward()
        errs = {"embedding": ((model.backbone.embedding.weight.grad - emb_ref).abs().max().item(),
                              emb_ref.abs().max().item())}
        for i, (layer, (di, gr)) in enumerate(zip(model.backbone.layers, full)):
            m, dl = layer.mixer, di // world
            lo, hi = rank * dl, (rank + 1) * dl
            want = {"in_proj_w": torch.cat([gr["in_proj.weight"][lo:hi], gr["in_proj.weight"][di + lo:di + hi]]),
                    "conv_w": gr["conv1d.weight"][lo:hi, 0], "x_proj_w": gr["x_proj.weight"][:, lo:hi],
                    "dt_proj_w": gr["dt_proj.weight"][lo:hi], "A_log": gr["A_log"][lo:hi], "D": gr["D"][lo:hi],
                    "out_proj_w": gr["out_proj.weight"][:, lo:hi]}
            for k, w in want.items():
                errs[f"layer{i}.{k}"] = ((getattr(m, k).grad - w).abs().max().item(), w.abs().max().item())
        torch.cuda.synchronize()
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_nccl_backward_matches_unsharded():
    """Gradients are sums over tokens, so the bound's absolute term scales with the largest
    magnitude of each gradient (as for all sums in these tests)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_grad_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs in res:
        for k, (err, scale) in errs.items():
            assert err <= 1e-3 * max(1.0, scale), (rank, k, err, scale)
