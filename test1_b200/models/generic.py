"""Layer programs for any HuggingFace causal LM (the reference accepts any
``PreTrainedModel`` whose decoder has ``.layers`` or ``.block``,
slide_fsdp.py:213-244).

Architectures with the plain Llama structure run on ``models.llama`` and the
sm_100a kernels.  Everything else (biases, other norms, other attention
variants, e.g. Qwen2) runs its own HF modules here under autograd, one layer
at a time, with the same engine (host master, sliding pool, host optimizer):

  forward_train  no-grad forward of the HF layer; the input is the checkpoint
  backward       recompute the layer with grad enabled from the checkpoint and
                 back-propagate ``dh`` through it; parameter gradients land in
                 ``param.grad`` (views into the engine's pool unit, zeroed
                 first, since autograd accumulates into an existing grad)
"""
from __future__ import annotations

import torch
import torch.nn as nn


def _zero_grads(module: nn.Module) -> None:
    for p in module.parameters():
        if p.grad is None:
            p.grad = torch.zeros_like(p)
        else:
            p.grad.zero_()


class GenericContext:
    """Batch context of the generic path: hidden states are [B, S, H]."""

    def __init__(self, batch: int, seq_len: int, position_embeddings, position_ids, input_ids,
                 targets, masks=None):
        self.masks = masks or {}  # attention type -> mask object of the HF attention backend
        self.batch = batch
        self.seq_len = seq_len
        self.position_embeddings = position_embeddings
        self.position_ids = position_ids
        self.input_ids = input_ids
        self.targets = targets


class GenericDecoderLayer(nn.Module):
    """Adapter around one HF decoder layer."""

    def __init__(self, layer: nn.Module):
        super().__init__()
        self.layer = layer

    @property
    def params_root(self) -> nn.Module:
        """The module whose parameter names the engine lays out (HF names)."""
        return self.layer

    def _call(self, h: torch.Tensor, ctx: GenericContext) -> torch.Tensor:
        B, S = ctx.batch, ctx.seq_len
        x = h.view(B, S, -1)
        mask = ctx.masks.get(getattr(self.layer, "attention_type", "full_attention"))
        kwargs = dict(attention_mask=mask, position_ids=ctx.position_ids, use_cache=False)
        if ctx.position_embeddings is not None:
            kwargs["position_embeddings"] = ctx.position_embeddings
        out = self.layer(x, **kwargs)
        if isinstance(out, (tuple, list)):
            out = out[0]
        return out.reshape(B * S, -1)

    def forward_train(self, h: torch.Tensor, ctx, save: bool = True, qkv_fn=None, ln1_weight=None):
        with torch.no_grad():
            out = self._call(h, ctx)
        return out, (h if save else None)

    def forward(self, h, ctx):
        return self.forward_train(h, ctx, save=False)[0]

    def backward(self, saved, dh: torch.Tensor, ctx, grad_ready=None) -> torch.Tensor:
        h = saved.detach().requires_grad_(True)
        _zero_grads(self.layer)
        with torch.enable_grad():
            out = self._call(h, ctx)
            torch.autograd.backward(out, dh)
        return h.grad


class GenericEmbedding(nn.Module):
    def __init__(self, emb: nn.Module):
        super().__init__()
        self.emb = emb

    @property
    def params_root(self) -> nn.Module:
        return self.emb

    def forward_ids(self, ids: torch.Tensor) -> torch.Tensor:
        with torch.no_grad():
            return self.emb(ids.reshape(-1))

    def backward_ids(self, dh: torch.Tensor, ids: torch.Tensor) -> None:
        _zero_grads(self.emb)
        with torch.enable_grad():
            out = self.emb(ids.reshape(-1))
            torch.autograd.backward(out, dh)


class GenericOutputLayer(nn.Module):
    """Final norm + lm_head of any architecture; loss = mean token
    cross-entropy on shifted labels (ignore_index -100)."""

    def __init__(self, norm: nn.Module, lm_head: nn.Module):
        super().__init__()
        self.norm = norm
        self.lm_head = lm_head

    def loss_and_grad(self, h: torch.Tensor, ctx):
        x = h.detach().requires_grad_(True)
        _zero_grads(self)
        with torch.enable_grad():
            logits = self.lm_head(self.norm(x)).float()
            loss = torch.nn.functional.cross_entropy(logits, ctx.targets, ignore_index=-100)
            loss.backward()
        return loss.detach(), x.grad

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        with torch.no_grad():
            return self.lm_head(self.norm(h))


def causal_masks(config, batch: int, seq_len: int, hidden: int, position_ids, device, dtype) -> dict:
    """Causal (and sliding-window) masks in the form the model's attention
    backend wants (None where it applies causality itself, e.g. SDPA)."""
    try:
        from transformers.masking_utils import create_causal_mask, create_sliding_window_causal_mask
    except Exception:  # pragma: no cover - older transformers
        return {}
    emb = torch.empty(1, device=device, dtype=dtype).expand(batch, seq_len, hidden)
    kw = dict(config=config, inputs_embeds=emb, attention_mask=None, past_key_values=None,
              position_ids=position_ids)
    out = {"full_attention": create_causal_mask(**kw)}
    if "sliding_attention" in (getattr(config, "layer_types", None) or ()):
        out["sliding_attention"] = create_sliding_window_causal_mask(**kw)
    return out


def is_native_llama(model: nn.Module) -> bool:
    """True when the HF model has exactly the structure models.llama runs:
    bias-free q/k/v/o and gate/up/down projections, RMSNorm, untied heads."""
    cfg = getattr(model, "config", None)
    if getattr(cfg, "model_type", None) not in ("llama", "mistral"):
        return False
    if getattr(cfg, "attention_bias", False) or getattr(cfg, "mlp_bias", False):
        return False
    if getattr(cfg, "hidden_act", "silu") != "silu":
        return False
    return not getattr(cfg, "tie_word_embeddings", False)
