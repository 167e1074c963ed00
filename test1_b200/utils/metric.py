"""Training FLOPs per batch (Megatron-LM style accounting with grouped-query
attention and SwiGLU), as the reference reports TFLOPS (utils/metric.py:4-53):

  F = 12 B S L h^2 [ (1 + G/H + S/h) q/h + (I/h) * 3/2 + V / (2 L h) ]

with h hidden, L layers, H query heads, G KV heads, q = H * head_dim, I the
SwiGLU width, V the vocabulary.  The factor 12 = 3 (forward + 2x backward) x
2 (multiply-add) x 2 (the two GEMMs of each pair); no activation-recompute
term (as in the reference).  ``with_recompute`` adds the recomputed forward.
"""
from __future__ import annotations


def calculate_flops_per_batch(model_or_config, batch_size: int, seq_length: int,
                              with_recompute: bool = False) -> float:
    cfg = getattr(model_or_config, "config", model_or_config)
    h = cfg.hidden_size
    L = cfg.num_hidden_layers
    H = cfg.num_attention_heads
    G = getattr(cfg, "num_key_value_heads", H)
    V = cfg.vocab_size
    I = cfg.intermediate_size
    head_dim = getattr(cfg, "head_dim", None) or h // H
    q = head_dim * H
    S, B = seq_length, batch_size
    layers = 12 * B * S * L * h * h * ((1 + G / H + S / h) * (q / h) + (I / h) * 1.5)
    vocab = 12 * B * S * L * h * h * (V / (2 * L * h))
    flops = layers + vocab
    if with_recompute:
        flops += layers / 3  # one more forward of every decoder layer
    return flops
