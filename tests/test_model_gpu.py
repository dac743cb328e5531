"""The mixer and LM stack (callers of the hot path) on the GPU kernels, against the
reference's own Mambamotif outputs (golden) and the oracle restatement of the stack."""
import os

import pytest
import torch

from oracle import ssm_oracle as O
from ssm_cases import assert_close

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"


def _golden_module(name="small"):
    from motif_ssm.modules import Mambamotif
    rec = torch.load(os.path.join(GOLD, f"module_{name}.pt"), weights_only=False)
    cfg = rec["config"]
    mod = Mambamotif(d_model=cfg["d_model"], d_state=cfg["d_state"], d_conv=cfg["d_conv"], expand=cfg["expand"],
                     layer_idx=0, pq_rank=cfg.get("pq_rank", 0), pq_per_dim=cfg.get("pq_per_dim", False),
                     device=DEV)
    mod.load_state_dict({k: v.to(DEV) for k, v in rec["state_dict"].items()})
    return rec, mod


def test_mixer_prefill_matches_reference_module():
    rec, mod = _golden_module()
    with torch.no_grad():
        y = mod(rec["hidden"].to(DEV))                    # fused mamba_inner_fn path
    assert_close(y, rec["y_prefill"], 1e-3, 1e-3, "Mambamotif prefill")


@pytest.mark.parametrize("name", ["pq2", "pq3_perdim"])
def test_pq_mixer_prefill_matches_reference_module(name):
    """Mambamotif with the motif P/Q coupling (pq_k * P, Q) on the ss_pq kernels."""
    rec, mod = _golden_module(name)
    with torch.no_grad():
        y = mod(rec["hidden"].to(DEV))
    assert_close(y, rec["y_prefill"], 1e-3, 1e-3, f"{name} prefill")


@pytest.mark.parametrize("name", ["small", "pq2", "pq3_perdim"])
def test_mixer_prefill_with_cache_then_decode_matches_reference_module(name):
    from motif_ssm.modules import InferenceParams
    rec, mod = _golden_module(name)
    hs = rec["hidden"].to(DEV)
    params = InferenceParams(max_seqlen=64, max_batch_size=hs.shape[0])
    with torch.no_grad():
        y = mod(hs, inference_params=params)              # conv + selective_scan_fn, stores states
        assert_close(y, rec["y_prefill"], 1e-3, 1e-3, "prefill with cache")
        conv_state, ssm_state = params.key_value_memory_dict[0]
        assert_close(conv_state, rec["conv_state0"], 1e-6, 1e-6, "conv_state after prefill")
        assert_close(ssm_state, rec["ssm_state0"], 1e-3, 1e-3, "ssm_state after prefill")
        params.seqlen_offset = hs.shape[1]
        for i in range(rec["step_in"].shape[0]):
            o = mod(rec["step_in"][i].to(DEV), inference_params=params)
            params.seqlen_offset += 1
            assert_close(o, rec["step_out"][i], 1e-3, 1e-3, f"decode step {i}")


def _stack_oracle(model, ids):
    """The stack restated with the oracle pieces on the CPU (fp32)."""
    sd = {k: v.detach().float().cpu() for k, v in model.state_dict().items()}
    h = sd["backbone.embedding.weight"][ids.cpu()]
    residual = None
    for i in range(model.config.n_layer):
        p = f"backbone.layers.{i}."
        residual = h if residual is None else h + residual
        x = O.rms_norm_ref(residual, sd[p + "norm.weight"])
        xz = torch.einsum("od,bld->bol", sd[p + "mixer.in_proj.weight"], x)
        A = -torch.exp(sd[p + "mixer.A_log"])
        h = O.mamba_inner_ref(xz, sd[p + "mixer.conv1d.weight"], sd[p + "mixer.conv1d.bias"],
                              sd[p + "mixer.x_proj.weight"], sd[p + "mixer.dt_proj.weight"],
                              sd[p + "mixer.out_proj.weight"], None, A, None, None, sd[p + "mixer.D"],
                              delta_bias=sd[p + "mixer.dt_proj.bias"])
    residual = h + residual
    x = O.rms_norm_ref(residual, sd["backbone.norm_f.weight"])
    return x @ sd["lm_head.weight"].t()


def test_lm_stack_fp32_matches_oracle_stack():
    from motif_ssm.modules import MambaConfig, MambaLMHeadModel
    torch.manual_seed(0)
    cfg = MambaConfig(d_model=64, n_layer=3, vocab_size=100, ssm_cfg={"d_state": 16})
    model = MambaLMHeadModel(cfg, device=DEV)
    ids = torch.randint(0, 100, (2, 96), device=DEV)
    with torch.no_grad():
        logits = model(ids)
    ref = _stack_oracle(model, ids)
    assert_close(logits, ref, 1e-3, 1e-3, "LM logits")


def test_lm_stack_config2_24_layers_bf16_matches_oracle_stack():
    """BASELINE config 2's stack (24 layers, d_model 768, d_inner 1536, n 16, RMSNorm, vocab
    512) in bf16 with its random init, on a short slice (2 x 128 random ids): logits against
    the oracle stack evaluated in fp32 on the same bf16 weights, at the bf16 tolerance."""
    from motif_ssm.modules import MambaConfig, MambaLMHeadModel
    torch.manual_seed(0)
    cfg = MambaConfig(d_model=768, n_layer=24, vocab_size=512, ssm_cfg={"d_state": 16})
    model = MambaLMHeadModel(cfg, device=DEV, dtype=torch.bfloat16)
    model.eval()
    ids = torch.randint(0, 512, (2, 128), device=DEV, generator=torch.Generator(device=DEV).manual_seed(3))
    with torch.no_grad():
        logits = model(ids)
    ref = _stack_oracle(model, ids)
    assert_close(logits, ref, 2e-2, 2e-2, "24-layer bf16 LM logits")


def test_lm_greedy_decode_matches_full_prefill():
    """Decoding token by token through the cache gives the logits a full prefill gives."""
    from motif_ssm.modules import InferenceParams, MambaConfig, MambaLMHeadModel
    torch.manual_seed(1)
    cfg = MambaConfig(d_model=64, n_layer=2, vocab_size=64, ssm_cfg={"d_state": 16})
    model = MambaLMHeadModel(cfg, device=DEV)
    ids = torch.randint(0, 64, (3, 40), device=DEV)
    with torch.no_grad():
        full = model(ids)
        params = InferenceParams(max_seqlen=40, max_batch_size=3)
        pre = model(ids[:, :30], inference_params=params, num_last_tokens=1)
        assert_close(pre[:, 0], full[:, 29], 1e-3, 1e-3, "prefill last logits")
        params.seqlen_offset = 30
        for t in range(30, 40):
            o = model(ids[:, t:t + 1], inference_params=params, num_last_tokens=1)
            params.seqlen_offset += 1
            assert_close(o[:, 0], full[:, t], 1e-3, 1e-3, f"decode logits t={t}")


def test_lm_stack_backward_runs_bf16():
    from motif_ssm.modules import MambaConfig, MambaLMHeadModel
    torch.manual_seed(2)
    cfg = MambaConfig(d_model=128, n_layer=2, vocab_size=256, ssm_cfg={"d_state": 16})
    model = MambaLMHeadModel(cfg, device=DEV, dtype=torch.bfloat16)
    ids = torch.randint(0, 256, (2, 300), device=DEV)
    logits = model(ids)
    loss = torch.nn.functional.cross_entropy(logits.float().flatten(0, 1), ids.flatten())
    loss.backward()
    for n, p in model.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), n


def test_graphed_decode_matches_eager_decode():
    from motif_ssm.modules import GraphedDecoder, InferenceParams, MambaConfig, MambaLMHeadModel
    torch.manual_seed(3)
    cfg = MambaConfig(d_model=128, n_layer=3, vocab_size=96, ssm_cfg={"d_state": 16})
    model = MambaLMHeadModel(cfg, device=DEV, dtype=torch.bfloat16)
    ids = torch.randint(0, 96, (4, 50), device=DEV)
    with torch.no_grad():
        pe = InferenceParams(max_seqlen=60, max_batch_size=4)
        pg = InferenceParams(max_seqlen=60, max_batch_size=4)
        model(ids[:, :40], inference_params=pe, num_last_tokens=1)
        model(ids[:, :40], inference_params=pg, num_last_tokens=1)
        pe.seqlen_offset = pg.seqlen_offset = 40
        dec = GraphedDecoder(model, pg, batch=4)
        for t in range(40, 50):
            eager = model(ids[:, t:t + 1], inference_params=pe, num_last_tokens=1)
            pe.seqlen_offset += 1
            graphed = dec.step(ids[:, t:t + 1])
            assert torch.equal(graphed, eager), t


def test_pq_mixer_trains_pq_only():
    """``create(train_pq_only=True)`` leaves only P, Q, pq_k trainable; their gradients
    through the module match autograd through the CPU oracle's slow-path restatement."""
    from motif_ssm.modules import Mambamotif
    torch.manual_seed(4)
    mod, info = Mambamotif.create(d_model=32, d_state=16, pq_rank=2, train_pq_only=True, layer_idx=0, device=DEV)
    assert info == {"missing_keys": [], "unexpected_keys": []}
    assert sorted(n for n, p in mod.named_parameters() if p.requires_grad) == ["P", "Q", "pq_k"]
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():  # a coupling strong enough to matter (~1.5 % of the output), still stable
        mod.pq_k.fill_(8.0)
        mod.P.copy_(0.5 * torch.randn(mod.P.shape, generator=g))
        mod.Q.copy_(0.5 * torch.randn(mod.Q.shape, generator=g))
    hs = torch.randn(2, 100, 32, generator=g)
    w = torch.randn(2, 100, 32, generator=g)
    (mod(hs.to(DEV)) * w.to(DEV)).sum().backward()
    sd = {k: v.detach().float().cpu().clone() for k, v in mod.state_dict().items()}
    for k in ("P", "Q", "pq_k"):
        sd[k].requires_grad_(True)
    (O.mixer_pq_prefill_ref(sd, hs) * w).sum().backward()
    for k in ("P", "Q", "pq_k"):
        assert_close(getattr(mod, k).grad, sd[k].grad, 1e-3, 1e-3, f"d{k}", scaled=True)


def test_graphed_prefill_matches_eager():
    from motif_ssm.modules import GraphedForward, MambaConfig, MambaLMHeadModel
    torch.manual_seed(11)
    model = MambaLMHeadModel(MambaConfig(d_model=128, n_layer=2, vocab_size=64, ssm_cfg={"d_state": 16}),
                             device=DEV, dtype=torch.bfloat16)
    gf = GraphedForward(model, 2, 600)
    for seed in (0, 1):
        ids = torch.randint(0, 64, (2, 600), device=DEV, generator=torch.Generator(device=DEV).manual_seed(seed))
        with torch.no_grad():
            eager = model(ids, num_last_tokens=1)
        assert torch.equal(gf(ids), eager), seed
