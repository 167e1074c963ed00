"""Llama-architecture causal LM with explicit per-layer forward/backward.
The reference runs HF's modules under autograd, one checkpointed layer at a
time (slide_fsdp.py:546-640, model loaded in train.py:94-123); here each
decoder layer is a fixed program of sm_100a kernels with a hand-written
backward.

Parameter names and ``named_parameters()`` order match HuggingFace's
``LlamaForCausalLM`` (model.embed_tokens, model.layers.{i}.self_attn.{q,k,v,o}_proj,
model.layers.{i}.mlp.{gate,up,down}_proj, model.layers.{i}.{input,post_attention}_layernorm,
model.norm, lm_head), so HF checkpoints load and ``save_pretrained`` writes
the HF layout.

The layers do not rely on autograd.  Each exposes ``forward`` (activations
only) plus ``forward_train``/``backward`` that keep exactly the tensors the
backward needs and write parameter gradients into ``param.grad`` (which the
SlideFSDP engine points at a slot of its GPU buffer pool).  Because q/k/v and
gate/up are adjacent in the flat parameter layout, the kernels see them as one
fused ``[6144, 4096]`` QKV weight and one ``[28672, 4096]`` gate/up weight.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .. import ops


@dataclass
class LlamaConfig:
    vocab_size: int = 128256
    hidden_size: int = 4096
    intermediate_size: int = 14336
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: Optional[int] = None
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: Optional[dict] = None
    max_position_embeddings: int = 131072
    tie_word_embeddings: bool = False
    initializer_range: float = 0.02
    model_type: str = "llama"
    bos_token_id: int = 128000
    eos_token_id: int = 128001

    def __post_init__(self):
        if self.head_dim is None:
            self.head_dim = self.hidden_size // self.num_attention_heads
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("num_attention_heads must be a multiple of num_key_value_heads")

    # ---- presets (comparison configs) ------------------------------------
    @classmethod
    def llama31_8b(cls) -> "LlamaConfig":
        return cls(
            rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                          "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
        )

    @classmethod
    def llama_70b(cls) -> "LlamaConfig":
        return cls(hidden_size=8192, intermediate_size=28672, num_hidden_layers=80,
                   num_attention_heads=64, num_key_value_heads=8,
                   rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                 "high_freq_factor": 4.0,
                                 "original_max_position_embeddings": 8192})

    @classmethod
    def tiny(cls) -> "LlamaConfig":
        """4 layers, hidden 256, 4 heads (dim 64), 2 KV heads, SwiGLU 688,
        vocab 1024, theta 10000 (the CPU plumbing configuration)."""
        return cls(vocab_size=1024, hidden_size=256, intermediate_size=688, num_hidden_layers=4,
                   num_attention_heads=4, num_key_value_heads=2, rope_theta=10000.0,
                   max_position_embeddings=2048, bos_token_id=1, eos_token_id=2)

    # ---- HF interop -----------------------------------------------------
    @classmethod
    def from_hf(cls, hf_config) -> "LlamaConfig":
        d = hf_config.to_dict() if hasattr(hf_config, "to_dict") else dict(hf_config)
        keys = {f for f in cls.__dataclass_fields__}
        kw = {k: v for k, v in d.items() if k in keys}
        rp = d.get("rope_parameters")
        if rp is not None:  # transformers >= 5 keeps theta/scaling here
            kw.setdefault("rope_theta", rp.get("rope_theta", kw.get("rope_theta", 10000.0)))
            if rp.get("rope_type", "default") != "default":
                kw["rope_scaling"] = {k: v for k, v in rp.items() if k != "rope_theta"}
        return cls(**kw)

    def to_hf_dict(self) -> dict:
        d = asdict(self)
        d["architectures"] = ["LlamaForCausalLM"]
        d["hidden_act"] = "silu"
        d["attention_bias"] = False
        d["mlp_bias"] = False
        d["torch_dtype"] = "bfloat16"
        return d

    def to_hf(self):
        from transformers import LlamaConfig as HFLlamaConfig

        d = self.to_hf_dict()
        d.pop("model_type", None)
        d.pop("architectures", None)
        return HFLlamaConfig(**d)

    # ---- sizes -----------------------------------------------------------
    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def decoder_layer_params(self) -> int:
        H, I = self.hidden_size, self.intermediate_size
        return H * (self.q_size + 2 * self.kv_size) + self.q_size * H + 3 * H * I + 2 * H

    def num_params(self) -> int:
        emb = self.vocab_size * self.hidden_size
        head = 0 if self.tie_word_embeddings else emb
        return emb + head + self.hidden_size + self.num_hidden_layers * self.decoder_layer_params()


# --------------------------------------------------------------------------
# Batch context shared by every layer of one step.


@dataclass
class StepContext:
    batch: int
    seq_len: int
    cos: torch.Tensor
    sin: torch.Tensor
    input_ids: Optional[torch.Tensor] = None  # [T] int64 on the device
    targets: Optional[torch.Tensor] = None    # [T] int64 (shifted labels)

    @property
    def tokens(self) -> int:
        return self.batch * self.seq_len


_ROPE_CACHE: Dict[Any, Tuple[torch.Tensor, torch.Tensor]] = {}


def make_context(cfg: LlamaConfig, input_ids: torch.Tensor, labels: Optional[torch.Tensor],
                 device: torch.device) -> StepContext:
    B, S = input_ids.shape
    key = (cfg.head_dim, S, cfg.rope_theta, json.dumps(cfg.rope_scaling, sort_keys=True), str(device))
    if key not in _ROPE_CACHE:
        _ROPE_CACHE[key] = ops.rope_tables(cfg.head_dim, S, cfg.rope_theta, cfg.rope_scaling, device)
    cos, sin = _ROPE_CACHE[key]
    ctx = StepContext(batch=B, seq_len=S, cos=cos, sin=sin,
                      input_ids=input_ids.reshape(-1).to(device, non_blocking=True))
    if labels is not None:
        # shifted targets; the number of valid targets is counted on the
        # device by the loss kernel (no host synchronisation per step)
        ctx.targets = ops.shift_labels(labels.to(device, non_blocking=True))
    return ctx


# --------------------------------------------------------------------------
# Parameter holders (HF names)


class _Weight(nn.Module):
    """A bias-free linear's weight holder, ``weight`` is ``[out, in]``."""

    def __init__(self, out_f: int, in_f: int, device=None, dtype=None):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(out_f, in_f, device=device, dtype=dtype))


class RMSNorm(nn.Module):
    def __init__(self, hidden: int, eps: float, device=None, dtype=None):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden, device=device, dtype=dtype))
        self.variance_epsilon = eps


class LlamaAttention(nn.Module):
    def __init__(self, cfg: LlamaConfig, device=None, dtype=None):
        super().__init__()
        H = cfg.hidden_size
        self.q_proj = _Weight(cfg.q_size, H, device, dtype)
        self.k_proj = _Weight(cfg.kv_size, H, device, dtype)
        self.v_proj = _Weight(cfg.kv_size, H, device, dtype)
        self.o_proj = _Weight(H, cfg.q_size, device, dtype)


class LlamaMLP(nn.Module):
    def __init__(self, cfg: LlamaConfig, device=None, dtype=None):
        super().__init__()
        H, I = cfg.hidden_size, cfg.intermediate_size
        self.gate_proj = _Weight(I, H, device, dtype)
        self.up_proj = _Weight(I, H, device, dtype)
        self.down_proj = _Weight(H, I, device, dtype)


def _fused_rows(tensors: List[torch.Tensor]) -> torch.Tensor:
    """View several row-major [r_i, c] tensors that are adjacent in memory as
    one [sum r_i, c] tensor (no copy).  Falls back to a concatenated copy when
    they are not adjacent (a model not managed by the engine)."""
    base = tensors[0]
    cols = base.shape[1]
    ptr = base.data_ptr()
    es = base.element_size()
    adjacent = all(t.is_contiguous() for t in tensors)
    for t in tensors:
        if t.data_ptr() != ptr or t.shape[1] != cols:
            adjacent = False
            break
        ptr += t.numel() * es
    if adjacent:
        rows = sum(t.shape[0] for t in tensors)
        return base.as_strided((rows, cols), (cols, 1))
    return torch.cat(tensors, 0)


def _wgrad_in_chunks(dy: torch.Tensor, x: torch.Tensor, out: torch.Tensor, ready, chunks: int) -> None:
    """out = dy^T x, computed in ``chunks`` row blocks of ``out`` (256-row
    aligned); ``ready`` gets each block as soon as it is final, so its
    reduce-scatter and host store (on the gradient stream) overlap the
    GEMM of the next block."""
    rows = out.shape[0]
    step = -(-rows // max(1, chunks))
    step = -(-step // 256) * 256
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        ops.linear_wgrad(dy[:, r0:r1], x, out=out[r0:r1])
        ready(out[r0:r1])


class LlamaDecoderLayer(nn.Module):
    # row blocks of the two largest weight gradients when the engine syncs
    # gradients per range (each block's reduce-scatter overlaps the next)
    WGRAD_CHUNKS_GATE_UP = 4
    WGRAD_CHUNKS_DOWN = 2

    def __init__(self, cfg: LlamaConfig, device=None, dtype=None):
        super().__init__()
        self.cfg = cfg
        self.self_attn = LlamaAttention(cfg, device, dtype)
        self.mlp = LlamaMLP(cfg, device, dtype)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device, dtype)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device, dtype)

    # fused weight views ----------------------------------------------------
    def _w(self):
        a, m = self.self_attn, self.mlp
        w_qkv = _fused_rows([a.q_proj.weight.data, a.k_proj.weight.data, a.v_proj.weight.data])
        w_gu = _fused_rows([m.gate_proj.weight.data, m.up_proj.weight.data])
        return w_qkv, a.o_proj.weight.data, w_gu, m.down_proj.weight.data

    def _g(self):
        a, m = self.self_attn, self.mlp
        gs = [a.q_proj.weight.grad, a.k_proj.weight.grad, a.v_proj.weight.grad,
              a.o_proj.weight.grad, m.gate_proj.weight.grad, m.up_proj.weight.grad,
              m.down_proj.weight.grad, self.input_layernorm.weight.grad,
              self.post_attention_layernorm.weight.grad]
        if any(g is None for g in gs):
            for p in self.parameters():
                if p.grad is None:
                    p.grad = torch.zeros_like(p)
            return self._g()
        g_qkv = _fused_rows(gs[0:3])
        g_gu = _fused_rows(gs[4:6])
        return g_qkv, gs[3], g_gu, gs[6], gs[7], gs[8]

    # forward ---------------------------------------------------------------
    def forward_train(self, h: torch.Tensor, ctx: StepContext, save: bool = True, qkv_fn=None,
                      ln1_weight=None):
        """``qkv_fn(x1, rope)``, when given, produces the rotated QKV projection
        (the engine passes the fused all-gather + QKV GEMM of shard mode;
        ``rope`` = (cos, sin, seq_len, n_q, n_kv, head_dim)); the other
        weights are read after it returns.  The input norm runs before that
        gather, so it then takes its weight from ``ln1_weight`` (fetched on
        its own by the engine) instead of the not-yet-filled unit."""
        cfg = self.cfg
        Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        w_ln1 = ln1_weight if ln1_weight is not None else self.input_layernorm.weight.data
        x1, rstd1 = ops.rmsnorm_fwd(h, w_ln1, cfg.rms_norm_eps)
        rope = (ctx.cos, ctx.sin, ctx.seq_len, Hq, Hkv, D)
        if qkv_fn is not None:
            qkv = qkv_fn(x1, rope)
        else:
            qkv = ops.linear_fwd_rope(x1, self._w()[0], *rope)
        w_qkv, w_o, w_gu, w_down = self._w()
        o, lse = ops.attention_fwd(qkv, Hq, Hkv, D, ctx.seq_len)
        h2 = ops.linear_fwd(o, w_o, residual=h)
        x2, rstd2 = ops.rmsnorm_fwd(h2, self.post_attention_layernorm.weight.data, cfg.rms_norm_eps)
        gu = ops.linear_fwd(x2, w_gu)
        a = ops.swiglu_fwd(gu)
        h3 = ops.linear_fwd(a, w_down, residual=h2)
        saved = (h, x1, rstd1, qkv, o, lse, h2, x2, rstd2, gu, a) if save else None
        return h3, saved

    def forward(self, h: torch.Tensor, ctx: StepContext) -> torch.Tensor:
        return self.forward_train(h, ctx, save=False)[0]

    def backward(self, saved, dh3: torch.Tensor, ctx: StepContext, grad_ready=None) -> torch.Tensor:
        """``grad_ready(t)``, when given, is called (on the compute stream's
        timeline) with each weight gradient -- or, for the down and gate/up
        projections, each row block of it -- as soon as it is final: down,
        gate/up, o, qkv; the norm gradients come last."""
        cfg = self.cfg
        ready = grad_ready if grad_ready is not None else (lambda t: None)
        h, x1, rstd1, qkv, o, lse, h2, x2, rstd2, gu, a = saved
        Hq, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        w_qkv, w_o, w_gu, w_down = self._w()
        g_qkv, g_o, g_gu, g_down, g_ln1, g_ln2 = self._g()
        da = ops.linear_dgrad(dh3, w_down)
        if grad_ready is not None:
            _wgrad_in_chunks(dh3, a, g_down, ready, self.WGRAD_CHUNKS_DOWN)
        else:
            ops.linear_wgrad(dh3, a, out=g_down)
        dgu = ops.swiglu_bwd(da, gu)
        del da
        dx2 = ops.linear_dgrad(dgu, w_gu)
        if grad_ready is not None:
            _wgrad_in_chunks(dgu, x2, g_gu, ready, self.WGRAD_CHUNKS_GATE_UP)
        else:
            ops.linear_wgrad(dgu, x2, out=g_gu)
        del dgu
        dh2, dw2 = ops.rmsnorm_bwd(dx2, h2, self.post_attention_layernorm.weight.data, rstd2, dh3)
        g_ln2.copy_(dw2)
        do = ops.linear_dgrad(dh2, w_o)
        ops.linear_wgrad(dh2, o, out=g_o)
        ready(g_o)
        dqkv = ops.attention_bwd(do, qkv, o, lse, Hq, Hkv, D, ctx.seq_len)
        del do
        ops.rope_qkv_(dqkv, Hq, Hkv, D, ctx.cos, ctx.sin, ctx.seq_len, inverse=True)
        dx1 = ops.linear_dgrad(dqkv, w_qkv)
        ops.linear_wgrad(dqkv, x1, out=g_qkv)
        ready(g_qkv)
        del dqkv
        dh, dw1 = ops.rmsnorm_bwd(dx1, h, self.input_layernorm.weight.data, rstd1, dh2)
        g_ln1.copy_(dw1)
        return dh


class Embedding(nn.Module):
    def __init__(self, vocab: int, hidden: int, device=None, dtype=None):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(vocab, hidden, device=device, dtype=dtype))
        self.num_embeddings = vocab
        self.embedding_dim = hidden

    def forward_ids(self, ids: torch.Tensor) -> torch.Tensor:
        return ops.embedding_fwd(ids.reshape(-1), self.weight.data)

    def backward_ids(self, dh: torch.Tensor, ids: torch.Tensor) -> None:
        if self.weight.grad is None:
            self.weight.grad = torch.zeros_like(self.weight)
        ops.embedding_bwd(dh, ids.reshape(-1), self.num_embeddings, out=self.weight.grad)


class LlamaModel(nn.Module):
    def __init__(self, cfg: LlamaConfig, device=None, dtype=None):
        super().__init__()
        self.embed_tokens = Embedding(cfg.vocab_size, cfg.hidden_size, device, dtype)
        self.layers = nn.ModuleList(LlamaDecoderLayer(cfg, device, dtype)
                                    for _ in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device, dtype)


class LlamaForCausalLM(nn.Module):
    """Container with HF-compatible structure and names.  Build with
    ``device="meta"`` to defer allocation: SlideFSDP then initialises the
    host master directly (N(0, initializer_range), norms = 1)."""

    def __init__(self, cfg: LlamaConfig, device=None, dtype=torch.float32):
        super().__init__()
        self.config = cfg
        self.model = LlamaModel(cfg, device, dtype)
        self.lm_head = _Weight(cfg.vocab_size, cfg.hidden_size, device, dtype)
        if device is None or torch.device(device).type != "meta":
            self.init_weights()

    # HF-like accessors used by SlideFSDP to split the model
    def get_decoder(self):
        return self.model

    def get_input_embeddings(self):
        return self.model.embed_tokens

    def get_output_embeddings(self):
        return self.lm_head

    @torch.no_grad()
    def init_weights(self, seed: Optional[int] = None) -> None:
        gen = torch.Generator(device="cpu")
        if seed is not None:
            gen.manual_seed(seed)
        std = self.config.initializer_range
        for name, p in self.named_parameters():
            if name.endswith("layernorm.weight") or name == "model.norm.weight":
                p.fill_(1.0)
            else:
                p.copy_(torch.randn(p.shape, generator=gen, dtype=torch.float32) * std)

    # Plain eager forward (reference for tests / inference)
    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, labels: Optional[torch.Tensor] = None):
        cfg = self.config
        dev = self.model.embed_tokens.weight.device
        ctx = make_context(cfg, input_ids, labels, dev)
        h = self.model.embed_tokens.forward_ids(ctx.input_ids)
        for layer in self.model.layers:
            h = layer(h, ctx)
        x, _ = ops.rmsnorm_fwd(h, self.model.norm.weight.data, cfg.rms_norm_eps)
        logits = ops.linear_fwd(x, self.lm_head.weight.data)
        loss = None
        if labels is not None:
            loss, _, _ = ops.cross_entropy_fwd_bwd(logits, ctx.targets)
        return loss, logits.view(input_ids.shape[0], input_ids.shape[1], -1)

    def save_pretrained(self, output_dir: str, dtype: torch.dtype = torch.bfloat16) -> str:
        from ..utils.checkpoint_io import save_hf_checkpoint

        state = {n: p.detach() for n, p in self.named_parameters()}
        return save_hf_checkpoint(output_dir, self.config.to_hf_dict(), state, dtype)
