"""MotifMamba mixer and LM stack on this library's kernels (callers of the hot path).

* ``Mambamotif`` -- the reference mixer (``mamba_ssm/modules/mamba_simplemotif.py:31-443``),
  including the motif low-rank coupling (``pq_rank > 0``: fp32 ``P``, ``Q`` and the scalar
  ``pq_k``, scan with ``P_eff = pq_k * P``; ``:138-155, 270-335``).  Parameter names,
  shapes and initialisation follow the reference (dt-bias inverse-softplus init ``:102-110``,
  S4D-real ``A_log`` ``:116-123``, ``D = 1`` ``:135``).  Prefill runs ``mamba_inner_fn``
  (fused conv -> x_proj -> dt_proj -> scan -> out_proj); with an inference cache it runs
  conv + ``selective_scan_fn`` and stores the decode states; ``step`` runs
  ``causal_conv1d_update`` + ``selective_state_update``.
* ``Block``, ``MixerModel``, ``MambaLMHeadModel`` -- the pre-norm residual stack of
  ``mamba_ssm/models/mixer_seq_simple.py:118-309`` (the export lacks ``Block`` and
  ``RMSNorm``; their semantics -- Add -> Norm -> Mixer, residual kept in fp32 when
  ``residual_in_fp32`` -- are restated from ``:142-146, 190-211``).  RMSNorm is
  ``x * rsqrt(mean(x^2) + eps) * w``.
"""
import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from .causal_conv1d import causal_conv1d_fn, causal_conv1d_update
from . import selective_scan_cuda as _ssc
from .selective_scan_interface import mamba_inner_fn, selective_scan_fn
from .norm import add_rms_norm
from .norm import supported as rms_fused_supported
from .selective_state_update import dtproj_supported, selective_state_update, selective_state_update_dtproj


class Mambamotif(nn.Module):
    SIZE_PRESETS = {
        "tiny": {"d_model": 256, "d_state": 16, "d_conv": 4, "expand": 2},
        "small": {"d_model": 512, "d_state": 32, "d_conv": 4, "expand": 2},
        "base": {"d_model": 768, "d_state": 64, "d_conv": 4, "expand": 2},
    }

    def __init__(self, d_model, d_state=16, d_conv=4, expand=2, dt_rank="auto", dt_min=0.001, dt_max=0.1,
                 dt_init="random", dt_scale=1.0, dt_init_floor=1e-4, conv_bias=True, bias=False,
                 use_fast_path=True, layer_idx=None, pq_rank=0, pq_per_dim=False, pq_k_init=1e-4,
                 device=None, dtype=None):
        fk = {"device": device, "dtype": dtype}
        super().__init__()
        self.pq_rank, self.pq_per_dim = int(pq_rank), bool(pq_per_dim)
        self.d_model, self.d_state, self.d_conv, self.expand = d_model, d_state, d_conv, expand
        self.d_inner = int(expand * d_model)
        self.dt_rank = math.ceil(d_model / 16) if dt_rank == "auto" else dt_rank
        self.use_fast_path = use_fast_path
        self.layer_idx = layer_idx
        self.in_proj = nn.Linear(d_model, self.d_inner * 2, bias=bias, **fk)
        self.conv1d = nn.Conv1d(self.d_inner, self.d_inner, kernel_size=d_conv, groups=self.d_inner,
                                padding=d_conv - 1, bias=conv_bias, **fk)
        self.activation = "silu"
        self.x_proj = nn.Linear(self.d_inner, self.dt_rank + d_state * 2, bias=False, **fk)
        self.dt_proj = nn.Linear(self.dt_rank, self.d_inner, bias=True, **fk)
        std = self.dt_rank ** -0.5 * dt_scale
        if dt_init == "constant":
            nn.init.constant_(self.dt_proj.weight, std)
        elif dt_init == "random":
            nn.init.uniform_(self.dt_proj.weight, -std, std)
        else:
            raise NotImplementedError(dt_init)
        dt = torch.exp(torch.rand(self.d_inner, **fk) * (math.log(dt_max) - math.log(dt_min))
                       + math.log(dt_min)).clamp(min=dt_init_floor)
        with torch.no_grad():
            self.dt_proj.bias.copy_(dt + torch.log(-torch.expm1(-dt)))  # inverse softplus
        self.dt_proj.bias._no_reinit = True
        A = torch.arange(1, d_state + 1, dtype=torch.float32, device=device).repeat(self.d_inner, 1)
        self.A_log = nn.Parameter(torch.log(A))
        self.A_log._no_weight_decay = True
        self.D = nn.Parameter(torch.ones(self.d_inner, device=device))
        self.D._no_weight_decay = True
        if self.pq_rank > 0:  # N(0, 1e-2) factors, fp32 whatever the module dtype (:140-151)
            if self.pq_per_dim:
                P = torch.empty(self.d_inner, d_state, self.pq_rank, device=device)
                Q = torch.empty(self.d_inner, self.pq_rank, d_state, device=device)
            else:
                P = torch.empty(d_state, self.pq_rank, device=device)
                Q = torch.empty(self.pq_rank, d_state, device=device)
            nn.init.normal_(P, std=1e-2)
            nn.init.normal_(Q, std=1e-2)
            self.P = nn.Parameter(P)
            self.Q = nn.Parameter(Q)
            self.pq_k = nn.Parameter(torch.tensor(float(pq_k_init), device=device, dtype=torch.float32))
        else:
            self.register_parameter("P", None)
            self.register_parameter("Q", None)
            self.register_parameter("pq_k", None)
        self.out_proj = nn.Linear(self.d_inner, d_model, bias=bias, **fk)

    @staticmethod
    def _extract_state_dict(raw_obj, state_dict_key=None):
        """The state dict inside a checkpoint object (mamba_simplemotif.py:159-170)."""
        if not isinstance(raw_obj, dict):
            raise ValueError("Checkpoint must be a dict or contain a dict-like state_dict")
        if state_dict_key is not None:
            if not isinstance(raw_obj.get(state_dict_key), dict):
                raise ValueError(f"state_dict_key='{state_dict_key}' not found in checkpoint")
            return raw_obj[state_dict_key]
        for k in ("state_dict", "model_state_dict", "model", "net"):
            if isinstance(raw_obj.get(k), dict):
                return raw_obj[k]
        return raw_obj

    def load_checkpoint(self, checkpoint_path, strict=False, state_dict_key=None, strip_module_prefix=True):
        """Load weights; returns the missing / unexpected keys (mamba_simplemotif.py:172-189)."""
        state = self._extract_state_dict(torch.load(checkpoint_path, map_location="cpu"), state_dict_key)
        cleaned = {}
        for k, v in state.items():
            if isinstance(v, torch.Tensor):
                if strip_module_prefix and k.startswith("module."):
                    k = k[len("module."):]
                cleaned[k] = v
        res = self.load_state_dict(cleaned, strict=strict)
        return {"missing_keys": list(res.missing_keys), "unexpected_keys": list(res.unexpected_keys)}

    @classmethod
    def create(cls, *, init_mode="scratch", checkpoint_path=None, model_size=None, load_strict=False,
               train_pq_only=False, state_dict_key=None, **kwargs):
        """Scratch or checkpoint construction (mamba_simplemotif.py:191-228); returns
        ``(model, load_info)``."""
        if model_size is not None:
            if model_size not in cls.SIZE_PRESETS:
                raise ValueError(f"Unknown model_size='{model_size}', choose from {list(cls.SIZE_PRESETS)}")
            cfg = dict(cls.SIZE_PRESETS[model_size])
            cfg.update(kwargs)
        else:
            cfg = dict(kwargs)
        model = cls(**cfg)
        info = {"missing_keys": [], "unexpected_keys": []}
        if init_mode == "load":
            if checkpoint_path is None:
                raise ValueError("checkpoint_path is required when init_mode='load'")
            info = model.load_checkpoint(checkpoint_path, strict=load_strict, state_dict_key=state_dict_key)
        elif init_mode != "scratch":
            raise ValueError("init_mode must be 'scratch' or 'load'")
        if train_pq_only:
            model.set_train_pq_only(True)
        return model, info

    def set_train_pq_only(self, enable=True):
        """Freeze everything but P, Q and pq_k (mamba_simplemotif.py:230-239)."""
        if self.P is None or self.Q is None:
            raise RuntimeError("P/Q are not initialized. Set pq_rank > 0 when constructing Mambamotif.")
        for p in self.parameters():
            p.requires_grad_(not enable)
        for p in (self.P, self.Q, self.pq_k):
            p.requires_grad_(True)

    def _decode_consts(self):
        """A = -exp(A_log), the fp32 dt bias and the fp32 D for inference, recomputed only
        when A_log, the bias or D change (tracked by their version counters and storage), so
        a prefill or decode step does not launch the elementwise kernels and casts per layer
        for them.  A CUDA graph captured over ``forward`` / ``step`` reads these cached
        tensors: in-place edits of A_log / dt_proj.bias / D after capture need a new capture."""
        key = (self.A_log._version, self.A_log.data_ptr(), self.dt_proj.bias._version,
               self.dt_proj.bias.data_ptr(), self.D._version, self.D.data_ptr())
        if getattr(self, "_dc_key", None) != key:
            with torch.no_grad():
                self._dc = (-torch.exp(self.A_log.float()), self.dt_proj.bias.float().contiguous(),
                            self.D.float().contiguous())
            self._dc_key = key
        return self._dc

    def _scan_consts(self):
        """(A, D, dt bias) in fp32 for the scan: cached when no gradient can flow to them,
        otherwise computed in the autograd graph."""
        if torch.is_grad_enabled() and (self.A_log.requires_grad or self.D.requires_grad
                                        or self.dt_proj.bias.requires_grad):
            return -torch.exp(self.A_log.float()), self.D.float(), self.dt_proj.bias.float()
        A, dt_bias, D = self._decode_consts()
        return A, D, dt_bias

    def _P_eff(self):
        return None if self.P is None else self.pq_k * self.P

    def forward(self, hidden_states, inference_params=None):
        """hidden_states (B, L, D) -> (B, L, D)."""
        batch, seqlen, _ = hidden_states.shape
        conv_state = ssm_state = None
        if inference_params is not None:
            conv_state, ssm_state = self._get_states_from_cache(inference_params, batch)
            if inference_params.seqlen_offset > 0:
                out, _, _ = self.step(hidden_states, conv_state, ssm_state)
                return out
        # in_proj and the (b l d) -> (b d l) transpose in one GEMM (mamba_simplemotif.py:257-261)
        xz = (self.in_proj.weight @ hidden_states.reshape(-1, self.d_model).t()).view(-1, batch, seqlen)
        xz = xz.transpose(0, 1)
        if self.in_proj.bias is not None:
            xz = xz + self.in_proj.bias.to(xz.dtype).unsqueeze(-1)
        A, D, dt_bias = self._scan_consts()
        if self.use_fast_path and self.P is None and inference_params is None:
            return mamba_inner_fn(xz, self.conv1d.weight, self.conv1d.bias, self.x_proj.weight,
                                  self.dt_proj.weight, self.out_proj.weight, self.out_proj.bias, A, None, None,
                                  D, delta_bias=dt_bias, delta_softplus=True)
        x, z = xz.chunk(2, dim=1)
        if conv_state is not None:
            conv_state.copy_(F.pad(x, (self.d_conv - x.shape[-1], 0)))
        x = causal_conv1d_fn(x, self.conv1d.weight.reshape(self.d_inner, -1), self.conv1d.bias,
                             activation=self.activation)
        x_dbl = self.x_proj(x.transpose(1, 2).reshape(-1, self.d_inner))
        dt, B, C = torch.split(x_dbl, [self.dt_rank, self.d_state, self.d_state], dim=-1)
        dt = (self.dt_proj.weight @ dt.t()).view(self.d_inner, batch, seqlen).transpose(0, 1)
        B = B.view(batch, seqlen, -1).transpose(1, 2).contiguous()
        C = C.view(batch, seqlen, -1).transpose(1, 2).contiguous()
        y = selective_scan_fn(x, dt, A, B, C, D, z=z, delta_bias=dt_bias,
                              delta_softplus=True, return_last_state=ssm_state is not None,
                              P=self._P_eff(), Q=self.Q)
        if ssm_state is not None:
            y, last_state = y
            ssm_state.copy_(last_state)
        return self.out_proj(y.transpose(1, 2))

    def step(self, hidden_states, conv_state, ssm_state):
        """One decode token (mamba_simplemotif.py:337-402); states are updated in place.

        With P / Q the reference runs a one-step ``selective_scan_fn`` (``:367-395``), which
        starts from a zero state rather than from ``ssm_state`` and then overwrites
        ``ssm_state`` with that step's state; this restatement keeps that behaviour so that
        decode outputs match the reference's."""
        assert hidden_states.shape[1] == 1, "decoding one token at a time"
        xz = self.in_proj(hidden_states.squeeze(1))
        x, z = xz.chunk(2, dim=-1)
        x = causal_conv1d_update(x, conv_state, self.conv1d.weight.reshape(self.d_inner, -1), self.conv1d.bias,
                                 self.activation)
        x_db = self.x_proj(x)
        dt, B, C = torch.split(x_db, [self.dt_rank, self.d_state, self.d_state], dim=-1)
        if self.P is None and dtproj_supported(ssm_state, x, dt, self.dt_proj.weight):
            # dt_proj folded into the state update kernel (same rounding of dt as the GEMM)
            A, dt_bias, _ = self._decode_consts()
            y = selective_state_update_dtproj(ssm_state, x, dt, self.dt_proj.weight, A, B, C, self.D, z=z,
                                              dt_bias=dt_bias, dt_softplus=True)
            return self.out_proj(y).unsqueeze(1), conv_state, ssm_state
        dt = F.linear(dt, self.dt_proj.weight)
        if self.P is not None:
            A = -torch.exp(self.A_log.float())
            dt = F.softplus(dt + self.dt_proj.bias.to(dtype=dt.dtype))
            y, last_state = selective_scan_fn(x.unsqueeze(-1), dt.unsqueeze(-1), A, B.unsqueeze(-1),
                                              C.unsqueeze(-1), D=self.D.float(), z=z.unsqueeze(-1),
                                              delta_bias=None, delta_softplus=False, return_last_state=True,
                                              P=self._P_eff(), Q=self.Q)
            ssm_state.copy_(last_state.to(ssm_state.dtype))
            return self.out_proj(y[..., 0]).unsqueeze(1), conv_state, ssm_state
        A, dt_bias, _ = self._decode_consts()
        y = selective_state_update(ssm_state, x, dt, A, B, C, self.D, z=z, dt_bias=dt_bias, dt_softplus=True)
        return self.out_proj(y).unsqueeze(1), conv_state, ssm_state

    def allocate_inference_cache(self, batch_size, max_seqlen, dtype=None, **kwargs):
        device = self.out_proj.weight.device
        conv_state = torch.zeros(batch_size, self.d_inner, self.d_conv, device=device,
                                 dtype=self.conv1d.weight.dtype if dtype is None else dtype)
        ssm_state = torch.zeros(batch_size, self.d_inner, self.d_state, device=device,
                                dtype=self.dt_proj.weight.dtype if dtype is None else dtype)
        return conv_state, ssm_state

    def _get_states_from_cache(self, inference_params, batch_size):
        assert self.layer_idx is not None
        cache = inference_params.key_value_memory_dict
        if self.layer_idx not in cache:
            cache[self.layer_idx] = self.allocate_inference_cache(batch_size, inference_params.max_seqlen)
        return cache[self.layer_idx]


@dataclass
class InferenceParams:
    """Decode cache: per-layer (conv_state, ssm_state) and the number of tokens seen."""
    max_seqlen: int
    max_batch_size: int
    seqlen_offset: int = 0
    key_value_memory_dict: dict = field(default_factory=dict)


class RMSNorm(nn.Module):
    def __init__(self, hidden_size, eps=1e-5, device=None, dtype=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size, device=device, dtype=dtype))

    def forward(self, x):
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


def add_norm(x, residual, norm, residual_in_fp32=True):
    """residual <- x + residual, normed <- norm(residual); one fused kernel for RMSNorm
    (``norm.add_rms_norm``, what the reference's fused_add_norm path computes), the torch
    expression for LayerNorm or shapes the kernel does not take."""
    if isinstance(norm, RMSNorm) and rms_fused_supported(x, residual, norm.weight):
        return add_rms_norm(x, residual, norm.weight, norm.eps, residual_in_fp32)
    residual = x if residual is None else x + residual
    if residual_in_fp32:
        residual = residual.float()
    return norm(residual.to(norm.weight.dtype)), residual


class Block(nn.Module):
    """Add -> Norm -> Mixer (mixer_seq_simple.py:142-146): returns (mixer_out, residual)."""

    def __init__(self, dim, mixer, norm, residual_in_fp32=True):
        super().__init__()
        self.mixer, self.norm, self.residual_in_fp32 = mixer, norm, residual_in_fp32

    def forward(self, hidden_states, residual=None, inference_params=None):
        hidden_states, residual = add_norm(hidden_states, residual, self.norm, self.residual_in_fp32)
        return self.mixer(hidden_states, inference_params=inference_params), residual

    def allocate_inference_cache(self, batch_size, max_seqlen, dtype=None, **kw):
        return self.mixer.allocate_inference_cache(batch_size, max_seqlen, dtype=dtype, **kw)


@dataclass
class MambaConfig:
    """Same fields and defaults as the reference (mamba_ssm/models/config_mamba.py:4-18)."""
    d_model: int = 2560
    d_intermediate: int = 0
    n_layer: int = 64
    vocab_size: int = 50277
    ssm_cfg: dict = field(default_factory=dict)
    attn_layer_idx: list = field(default_factory=list)
    attn_cfg: dict = field(default_factory=dict)
    rms_norm: bool = True
    residual_in_fp32: bool = True
    fused_add_norm: bool = True
    pad_vocab_size_multiple: int = 8
    tie_embeddings: bool = True


def _init_weights(module, n_layer, initializer_range=0.02, rescale_prenorm_residual=True, n_residuals_per_layer=1):
    """GPT-2 style init of the reference stack (mixer_seq_simple.py:86-115)."""
    if isinstance(module, nn.Linear):
        if module.bias is not None and not getattr(module.bias, "_no_reinit", False):
            nn.init.zeros_(module.bias)
    elif isinstance(module, nn.Embedding):
        nn.init.normal_(module.weight, std=initializer_range)
    if rescale_prenorm_residual:
        for name, p in module.named_parameters():
            if name in ("out_proj.weight", "fc2.weight"):
                nn.init.kaiming_uniform_(p, a=math.sqrt(5))
                with torch.no_grad():
                    p /= math.sqrt(n_residuals_per_layer * n_layer)


class MixerModel(nn.Module):
    def __init__(self, d_model, n_layer, vocab_size, ssm_cfg=None, norm_epsilon=1e-5, rms_norm=True,
                 residual_in_fp32=True, device=None, dtype=None, **unused):
        fk = {"device": device, "dtype": dtype}
        super().__init__()
        ssm_cfg = dict(ssm_cfg or {})
        ssm_cfg.pop("layer", None)
        self.embedding = nn.Embedding(vocab_size, d_model, **fk)
        norm_cls = (lambda: RMSNorm(d_model, eps=norm_epsilon, **fk)) if rms_norm else \
            (lambda: nn.LayerNorm(d_model, eps=norm_epsilon, **fk))
        self.layers = nn.ModuleList([
            Block(d_model, Mambamotif(d_model, layer_idx=i, **ssm_cfg, **fk), norm_cls(), residual_in_fp32)
            for i in range(n_layer)])
        self.norm_f = norm_cls()
        self.apply(lambda m: _init_weights(m, n_layer))

    def allocate_inference_cache(self, batch_size, max_seqlen, dtype=None, **kw):
        return {i: l.allocate_inference_cache(batch_size, max_seqlen, dtype=dtype, **kw)
                for i, l in enumerate(self.layers)}

    def forward(self, input_ids, inference_params=None):
        hidden, residual = self.embedding(input_ids), None
        for layer in self.layers:
            hidden, residual = layer(hidden, residual, inference_params=inference_params)
        return add_norm(hidden, residual, self.norm_f)[0]


class MambaLMHeadModel(nn.Module):
    """Embedding -> MixerModel -> tied lm_head (mixer_seq_simple.py:215-309)."""

    def __init__(self, config: MambaConfig, device=None, dtype=None):
        super().__init__()
        self.config = config
        vocab = config.vocab_size
        if vocab % config.pad_vocab_size_multiple:
            vocab += config.pad_vocab_size_multiple - vocab % config.pad_vocab_size_multiple
        self.backbone = MixerModel(config.d_model, config.n_layer, vocab, ssm_cfg=config.ssm_cfg,
                                   rms_norm=config.rms_norm, residual_in_fp32=config.residual_in_fp32,
                                   device=device, dtype=dtype)
        self.lm_head = nn.Linear(config.d_model, vocab, bias=False, device=device, dtype=dtype)
        if config.tie_embeddings:
            self.lm_head.weight = self.backbone.embedding.weight

    def allocate_inference_cache(self, batch_size, max_seqlen, dtype=None, **kw):
        return self.backbone.allocate_inference_cache(batch_size, max_seqlen, dtype=dtype, **kw)

    def forward(self, input_ids, inference_params=None, num_last_tokens=0):
        hidden = self.backbone(input_ids, inference_params=inference_params)
        if num_last_tokens > 0:
            hidden = hidden[:, -num_last_tokens:]
        return self.lm_head(hidden)

    @torch.no_grad()
    def generate_greedy(self, input_ids, max_new_tokens):
        """Prefill with the inference cache, then greedy decode one token per step."""
        batch = input_ids.shape[0]
        params = InferenceParams(max_seqlen=input_ids.shape[1] + max_new_tokens, max_batch_size=batch)
        logits = self.forward(input_ids, inference_params=params, num_last_tokens=1)
        params.seqlen_offset = input_ids.shape[1]
        out = [logits.argmax(-1)]
        for _ in range(max_new_tokens - 1):
            logits = self.forward(out[-1], inference_params=params, num_last_tokens=1)
            params.seqlen_offset += 1
            out.append(logits.argmax(-1))
        return torch.cat(out, dim=1)


# ---------------------------------------------------------------------------------------
# Channel-sharded tensor parallelism (inference prefill).  d_inner is split over the ranks
# of `group`: in_proj rows (x and z halves of this rank's channels), conv1d, dt_proj rows,
# A, D and the scan are local.  x_proj contracts over d_inner, so each rank's x_dbl is a
# partial sum: all-reduce #1 (b*l x (dt_rank + 2n)) before dt_proj / B / C; out_proj is
# row-split: all-reduce #2 (b*l x d_model) after it.  Both are NCCL sums on the current
# stream.  The reference has no TP; this follows the plan of its channel-independent scan.
# ---------------------------------------------------------------------------------------
class TPMambamotif(nn.Module):
    """One mixer's shard.  Build with ``TPMambamotif.from_full(full_mixer, rank, world, group)``."""

    def __init__(self, d_model, d_inner_local, d_state, d_conv, dt_rank, rank, world, group, device=None,
                 dtype=None):
        super().__init__()
        fk = {"device": device, "dtype": dtype}
        self.d_model, self.d_local, self.d_state, self.d_conv, self.dt_rank = d_model, d_inner_local, d_state, d_conv, dt_rank
        self.rank, self.world, self.group = rank, world, group
        self.in_proj_w = nn.Parameter(torch.empty(2 * d_inner_local, d_model, **fk))
        self.conv_w = nn.Parameter(torch.empty(d_inner_local, d_conv, **fk))
        self.conv_b = nn.Parameter(torch.empty(d_inner_local, **fk))
        self.x_proj_w = nn.Parameter(torch.empty(dt_rank + 2 * d_state, d_inner_local, **fk))
        self.dt_proj_w = nn.Parameter(torch.empty(d_inner_local, dt_rank, **fk))
        self.dt_proj_b = nn.Parameter(torch.empty(d_inner_local, device=device, dtype=torch.float32))
        self.A_log = nn.Parameter(torch.empty(d_inner_local, d_state, device=device, dtype=torch.float32))
        self.D = nn.Parameter(torch.empty(d_inner_local, device=device, dtype=torch.float32))
        self.out_proj_w = nn.Parameter(torch.empty(d_model, d_inner_local, **fk))
        self.P_eff = self.Q = None  # motif coupling: pq_k * P and Q (this rank's channels if per channel)

    @classmethod
    def from_full(cls, full, rank, world, group):
        """Channel shard `rank` of a full mixer.  A per-channel P / Q is sliced with the
        channels; a shared one (same for every channel) is replicated."""
        di = full.d_inner
        assert di % world == 0, "d_inner must divide by the tensor-parallel size"
        dl = di // world
        lo, hi = rank * dl, (rank + 1) * dl
        w = full.in_proj.weight
        m = cls(full.d_model, dl, full.d_state, full.d_conv, full.dt_rank, rank, world, group,
                device=w.device, dtype=w.dtype)
        with torch.no_grad():
            m.in_proj_w.copy_(torch.cat([w[lo:hi], w[di + lo:di + hi]], dim=0))
            m.conv_w.copy_(full.conv1d.weight[lo:hi, 0])
            m.conv_b.copy_(full.conv1d.bias[lo:hi])
            m.x_proj_w.copy_(full.x_proj.weight[:, lo:hi])
            m.dt_proj_w.copy_(full.dt_proj.weight[lo:hi])
            m.dt_proj_b.copy_(full.dt_proj.bias[lo:hi].float())
            m.A_log.copy_(full.A_log[lo:hi])
            m.D.copy_(full.D[lo:hi])
            m.out_proj_w.copy_(full.out_proj.weight[:, lo:hi])
            if full.P is not None:
                P_eff, Q = (full.pq_k * full.P).float(), full.Q.float()
                if full.pq_per_dim:
                    P_eff, Q = P_eff[lo:hi], Q[lo:hi]
                m.P_eff, m.Q = P_eff.contiguous(), Q.contiguous()
        return m

    def _all_reduce(self, t):
        if self.world > 1:
            torch.distributed.all_reduce(t, group=self.group)
        return t

    # halo of the causal conv carried from one sequence chunk to the next: 8 steps (not
    # d_conv - 1 = 3) so that the conv output of a chunk starts 16-byte aligned
    HALO = 8

    @torch.no_grad()
    def forward_chunk(self, hidden_states, carry):
        """One sequence chunk of this shard's mixer.  ``carry`` holds what the next chunk needs
        from this one (the pre-conv x tail and the fp32 scan state; empty dict for the first
        chunk) and is updated.  Returns this rank's out_proj partial sum (not all-reduced);
        the x_proj partial sums are all-reduced here (fp32)."""
        batch, seqlen, _ = hidden_states.shape
        xz = (self.in_proj_w @ hidden_states.reshape(-1, self.d_model).t()).view(-1, batch, seqlen).transpose(0, 1)
        x, z = xz.chunk(2, dim=1)
        tail = carry.get("x_tail")
        xin = x if tail is None else torch.cat([tail, x], dim=-1)
        carry["x_tail"] = x[..., -self.HALO:] if seqlen >= self.HALO else xin[..., -self.HALO:]
        xc = causal_conv1d_fn(xin, self.conv_w, self.conv_b, activation="silu")
        if tail is not None:
            xc = xc[..., tail.shape[-1]:]
        # x_proj partial sums stay fp32 through the all-reduce and are rounded once, as the
        # unsharded GEMM rounds its fp32 accumulator once
        xt = xc.transpose(1, 2).reshape(-1, self.d_local)
        if xt.dtype in (torch.bfloat16, torch.float16):
            x_dbl = torch.mm(xt, self.x_proj_w.t(), out_dtype=torch.float32)
        else:
            x_dbl = xt @ self.x_proj_w.t()
        x_dbl = self._all_reduce(x_dbl.contiguous()).to(xc.dtype)   # all-reduce #1
        dt, B, C = torch.split(x_dbl, [self.dt_rank, self.d_state, self.d_state], dim=-1)
        dt = (self.dt_proj_w @ dt.t()).view(self.d_local, batch, seqlen).transpose(0, 1)
        B = B.reshape(batch, seqlen, -1).transpose(1, 2).contiguous()
        C = C.reshape(batch, seqlen, -1).transpose(1, 2).contiguous()
        key = (self.A_log._version, self.A_log.data_ptr())
        if getattr(self, "_A_key", None) != key:  # A = -exp(A_log), once per change of A_log
            self._A, self._A_key = -torch.exp(self.A_log), key
        y, carry["h"] = _scan_chunk(xc, dt, self._A, B, C, self.D, z, self.dt_proj_b, carry.get("h"),
                                    self.P_eff, self.Q)
        return y.transpose(1, 2).reshape(-1, self.d_local) @ self.out_proj_w.t()

    def forward(self, hidden_states, inference_params=None):
        """Prefill (no autograd): ``forward_chunk`` over the whole sequence and the out_proj
        all-reduce.  With autograd on (training), ``forward_train``."""
        if torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters()):
            return self.forward_train(hidden_states)
        with torch.no_grad():
            batch, seqlen, _ = hidden_states.shape
            out = self.forward_chunk(hidden_states, {})
            return self._all_reduce(out.contiguous()).view(batch, seqlen, self.d_model)  # all-reduce #2

    def forward_train(self, hidden_states):
        """The shard's mixer with autograd (the sharded counterpart of the unsharded mixer's
        training forward).  The replicated input enters through an operator whose backward
        all-reduces its gradient (each rank's in_proj rows see only this rank's channels); the
        x_proj and out_proj partial sums leave through an all-reduce whose backward is the
        identity for out_proj (every rank continues with the same replicated values, so each
        already holds the full gradient) and an all-reduce for x_proj (each rank uses the full
        x_dbl for its own channels only).  x_proj partial sums are reduced in fp32 and rounded once, as in the
        prefill path.  The motif P / Q coupling is not trained here (its sharded copies are
        not parameters)."""
        if self.P_eff is not None:
            raise NotImplementedError("TPMambamotif: training with the motif P/Q coupling is not supported")
        h = _TPCopy.apply(hidden_states, self.group, self.world)
        xz = torch.matmul(self.in_proj_w, h.transpose(1, 2))                  # (b, 2 d_local, l)
        x, z = xz.chunk(2, dim=1)
        xc = causal_conv1d_fn(x, self.conv_w, self.conv_b, activation="silu")
        x_dbl = F.linear(xc.transpose(1, 2).float(), self.x_proj_w.float())   # (b, l, r + 2n) partial sums
        x_dbl = _TPReduce.apply(x_dbl, self.group, self.world, True).to(xc.dtype)  # all-reduce #1
        dt, B, C = torch.split(x_dbl, [self.dt_rank, self.d_state, self.d_state], dim=-1)
        delta = torch.matmul(self.dt_proj_w, dt.transpose(1, 2))               # (b, d_local, l)
        B = B.transpose(1, 2).contiguous()
        C = C.transpose(1, 2).contiguous()
        y = selective_scan_fn(xc, delta, -torch.exp(self.A_log), B, C, self.D, z=z, delta_bias=self.dt_proj_b,
                              delta_softplus=True)
        out = F.linear(y.transpose(1, 2), self.out_proj_w)                     # (b, l, d_model) partial sums
        return _TPReduce.apply(out.contiguous(), self.group, self.world, False)  # all-reduce #2


class _TPCopy(torch.autograd.Function):
    """Replicated activations into a channel shard: identity forward, gradient all-reduced."""

    @staticmethod
    def forward(ctx, x, group, world):
        ctx.group, ctx.world = group, world
        return x

    @staticmethod
    def backward(ctx, g):
        if ctx.world > 1:
            g = g.contiguous()
            torch.distributed.all_reduce(g, group=ctx.group)
        return g, None, None


class _TPReduce(torch.autograd.Function):
    """Partial sums of the shards summed into full values (all-reduce forward).  Backward: when
    every rank then uses the full value for its own channels only (x_dbl feeds this rank's
    dt_proj rows and scan), each rank's gradient is a partial one and is all-reduced
    (``sharded_after``); when every rank continues with the same replicated computation (the
    out_proj sum feeds the residual stream), each rank already holds the full gradient."""

    @staticmethod
    def forward(ctx, x, group, world, sharded_after):
        ctx.group, ctx.world, ctx.sharded_after = group, world, sharded_after
        x = x.contiguous().clone()
        if world > 1:
            torch.distributed.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        if ctx.sharded_after and ctx.world > 1:
            g = g.contiguous().clone()
            torch.distributed.all_reduce(g, group=ctx.group)
        return g, None, None, None


def _scan_chunk(u, delta, A, B, C, D, z, delta_bias, h0, P=None, Q=None):
    """The gated scan of one sequence chunk started from state ``h0`` (fp32 (b, d, n), None:
    zero); returns (out_z, fp32 state after the chunk).  With P / Q (no initial-state support in
    that kernel) the sequence must come as one chunk."""
    if P is not None:
        assert h0 is None, "the motif P/Q scan runs a sequence as one chunk"
        y, last = selective_scan_fn(u, delta, A, B, C, D, z=z, delta_bias=delta_bias, delta_softplus=True,
                                    return_last_state=True, P=P, Q=Q)
        return y, last
    out, x, out_z = _ssc.fwd(u, delta, A, B.unsqueeze(1), C.unsqueeze(1), D=D, z=z, delta_bias=delta_bias,
                             delta_softplus=True, initial_state=h0)
    return out_z, x[:, :, -1, 1::2].contiguous()


@torch.no_grad()
def tp_prefill(model, input_ids, n_chunks=1, num_last_tokens=1):
    """Prefill of a channel-sharded model (``shard_model_tp``), optionally with the sequence
    split into ``n_chunks`` chunks processed layer by layer: each chunk's out_proj all-reduce is
    issued asynchronously and waited for only when layer l + 1 reaches that chunk, so it can run
    while the next chunk's in_proj, conv and x_proj GEMMs run (the scan carries its state across
    chunks, the conv an 8-step halo).  All collectives go to the one communicator of the shards'
    group, in the same order on every rank.  Returns the logits of the last ``num_last_tokens``
    tokens (all of them for 0)."""
    import torch.distributed as dist
    backbone = model.backbone
    mixer0 = backbone.layers[0].mixer
    world, group = mixer0.world, mixer0.group
    batch, seqlen = input_ids.shape
    per = -(-seqlen // n_chunks)                 # ceil(seqlen / n_chunks)
    step = max(64, -(-per // 64) * 64)           # chunk length: rounded up to a multiple of 64 steps
    bounds = [(t, min(seqlen, t + step)) for t in range(0, seqlen, step)]
    emb = backbone.embedding(input_ids)
    hid = [emb[:, t0:t1].contiguous() for t0, t1 in bounds]
    res = [None] * len(bounds)
    pend = [None] * len(bounds)
    for layer in backbone.layers:
        carry = {}
        for i in range(len(bounds)):
            if pend[i] is not None:
                pend[i].wait()
                pend[i] = None
            normed, res[i] = add_norm(hid[i], res[i], layer.norm, layer.residual_in_fp32)
            o = layer.mixer.forward_chunk(normed, carry)
            if world > 1:
                pend[i] = dist.all_reduce(o, group=group, async_op=True)  # all-reduce #2
            hid[i] = o.view(batch, bounds[i][1] - bounds[i][0], -1)
    for w in pend:
        if w is not None:
            w.wait()
    hidden = torch.cat(hid, dim=1)
    residual = torch.cat(res, dim=1)
    if num_last_tokens > 0:
        hidden, residual = hidden[:, -num_last_tokens:], residual[:, -num_last_tokens:]
    return model.lm_head(add_norm(hidden, residual, backbone.norm_f)[0])


def shard_model_tp(model, rank, world, group=None):
    """Replace every mixer of a MambaLMHeadModel by its channel shard for `rank` (in place).
    Embedding, norms and lm_head stay replicated."""
    for layer in model.backbone.layers:
        layer.mixer = TPMambamotif.from_full(layer.mixer, rank, world, group)
    return model


class GraphedForward:
    """A no-cache forward of a MambaLMHeadModel (prefill) for one fixed input shape, captured as
    a CUDA graph, so that short or small-batch prefills are not bound by the host launching
    ~15 kernels per layer.  ``out = gf(ids)`` copies ids into the static input buffer, replays
    and returns the static output buffer (valid until the next call)."""

    def __init__(self, model, batch, seqlen, num_last_tokens=1, warmup=2):
        self.model = model
        dev = model.lm_head.weight.device
        self.ids = torch.zeros(batch, seqlen, dtype=torch.long, device=dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s), torch.no_grad():
            for _ in range(warmup):
                model(self.ids, num_last_tokens=num_last_tokens)
        torch.cuda.current_stream(dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.out = model(self.ids, num_last_tokens=num_last_tokens)

    def __call__(self, ids):
        self.ids.copy_(ids)
        self.graph.replay()
        return self.out


class GraphedDecoder:
    """One decode step of a MambaLMHeadModel captured as a CUDA graph.

    Decode runs ~a dozen small kernels per layer (in_proj, conv update, x_proj, dt_proj,
    state update, out_proj, norms), so it is launch-bound; replaying a captured graph
    issues the whole step at once.  The cache tensors of `params` and the token buffer are
    captured by address: feed tokens with ``step(tokens)``, which copies them into the
    static buffer, replays, and returns the static logits buffer (valid until the next step).
    """

    def __init__(self, model, params, batch, warmup=2):
        self.model, self.params = model, params
        dev = model.lm_head.weight.device
        self.tokens = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        snapshot = {k: (a.clone(), b.clone()) for k, (a, b) in params.key_value_memory_dict.items()}
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s), torch.no_grad():
            for _ in range(warmup):
                model(self.tokens, inference_params=params, num_last_tokens=1)
        torch.cuda.current_stream(dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.logits = model(self.tokens, inference_params=params, num_last_tokens=1)
        for k, (a, b) in snapshot.items():  # undo the state changes of warm-up and capture
            params.key_value_memory_dict[k][0].copy_(a)
            params.key_value_memory_dict[k][1].copy_(b)

    def step(self, tokens):
        self.tokens.copy_(tokens)
        self.graph.replay()
        self.params.seqlen_offset += 1
        return self.logits
