"""Plain-PyTorch statements of every op of the Llama training step (the
reference computes them with HF / Liger modules; its loss is Liger's fused
linear cross-entropy or nn.CrossEntropyLoss, slide_fsdp.py:87-109).

These are the numerics oracle for the sm_100a kernels (tests compare each
kernel against the function of the same name here, computed in fp32) and the
implementation used when tensors live on the CPU (the gloo/CPU test path).

Layout conventions shared with the kernels:
  * activations are token-major 2-D ``[T, features]`` with T = batch * seq;
  * linear weights are ``[out, in]`` row-major (PyTorch / HF layout);
  * q/k/v are views ``[T, heads, head_dim]``; attention works per sequence of
    ``seq_len`` tokens, causal, with grouped-query heads (``Hq % Hkv == 0``);
  * RoPE follows HF's rotate-half convention (pairs (i, i + D/2)).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

# ----------------------------------------------------------------- RMSNorm


def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1) + eps)
    y = (xf * rstd[:, None] * w.float()).to(x.dtype)
    return y, rstd


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor, rstd: torch.Tensor,
                residual_grad: Optional[torch.Tensor] = None):
    """Returns (dx [+ residual_grad], dw)."""
    xf, dyf, wf = x.float(), dy.float(), w.float()
    xhat = xf * rstd[:, None]
    dxhat = dyf * wf
    c = (dxhat * xhat).mean(-1, keepdim=True)
    dx = rstd[:, None] * (dxhat - xhat * c)
    if residual_grad is not None:
        dx = dx + residual_grad.float()
    dw = (dyf * xhat).sum(0)
    return dx.to(x.dtype), dw.to(w.dtype)


# ------------------------------------------------------------------ Linear


def _mm_dtype(x: torch.Tensor) -> torch.dtype:
    # fp32 inputs give an fp32 product; bf16/fp16 inputs use the library GEMM
    # in that dtype (fp32 accumulation, one rounding at the end).
    return x.dtype if x.dtype in (torch.bfloat16, torch.float16) else torch.float32


def linear_fwd(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    dt = _mm_dtype(x)
    y = x.to(dt) @ w.to(dt).t()
    if residual is not None:
        y = (y.float() + residual.float())
    return y.to(x.dtype)


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    dt = _mm_dtype(dy)
    return (dy.to(dt) @ w.to(dt)).to(dy.dtype)


def linear_fwd_rope(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, seq_len: int,
                    n_q: int, n_kv: int, head_dim: int) -> torch.Tensor:
    qkv = linear_fwd(x, w)
    return rope_qkv_(qkv, n_q, n_kv, head_dim, cos, sin, seq_len)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    dt = _mm_dtype(dy)
    g = dy.to(dt).t() @ x.to(dt)
    if out is None:
        return g.to(dy.dtype)
    out.copy_(g.to(out.dtype))
    return out


# -------------------------------------------------------------------- RoPE


def rope_tables(head_dim: int, seq_len: int, theta: float, scaling: Optional[dict] = None,
                device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables [seq_len, head_dim/2] (fp32) for positions 0..seq_len-1.
    ``scaling`` supports HF's "llama3" frequency remapping (rope_type llama3)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling is not None:
        rtype = scaling.get("rope_type", scaling.get("type"))
        if rtype == "llama3":
            factor = scaling["factor"]
            lo = scaling["low_freq_factor"]
            hi = scaling["high_freq_factor"]
            old = scaling["original_max_position_embeddings"]
            low_wavelen = old / lo
            high_wavelen = old / hi
            wavelen = 2 * math.pi / inv_freq
            scaled = torch.where(wavelen > low_wavelen, inv_freq / factor, inv_freq)
            smooth = (old / wavelen - lo) / (hi - lo)
            smoothed = (1 - smooth) * scaled / factor + smooth * scaled
            medium = (wavelen >= high_wavelen) & (wavelen <= low_wavelen)
            inv_freq = torch.where(medium, smoothed, scaled)
        elif rtype not in (None, "default"):
            raise NotImplementedError(f"rope scaling {rtype!r}")
    pos = torch.arange(seq_len, dtype=torch.float64)
    freqs = torch.outer(pos, inv_freq)
    return freqs.cos().float().to(device), freqs.sin().float().to(device)


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, seq_len: int,
               inverse: bool = False) -> torch.Tensor:
    """x: [T, heads, D] with T = batch * seq_len; returns the rotated tensor.
    ``inverse`` rotates by -theta (the backward of the forward rotation)."""
    T, Hh, D = x.shape
    half = D // 2
    pos = torch.arange(T, device=x.device) % seq_len
    c = cos[pos][:, None, :]
    s = sin[pos][:, None, :]
    if inverse:
        s = -s
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    out = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
    return out.to(x.dtype)


# --------------------------------------------------------------- attention


def attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_len: int,
                  scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Causal GQA attention.  q [T,Hq,D], k/v [T,Hkv,D] -> (o [T,Hq,D], lse [Hq,T] fp32)."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    B = T // seq_len
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    qf = q.float().view(B, seq_len, Hq, D).transpose(1, 2)
    kf = k.float().view(B, seq_len, Hkv, D).transpose(1, 2).repeat_interleave(Hq // Hkv, dim=1)
    vf = v.float().view(B, seq_len, Hkv, D).transpose(1, 2).repeat_interleave(Hq // Hkv, dim=1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    mask = torch.ones(seq_len, seq_len, dtype=torch.bool, device=q.device).tril()
    s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)  # [B,Hq,S]
    p = torch.exp(s - lse[..., None])
    o = p @ vf
    o = o.transpose(1, 2).reshape(T, Hq, D).to(q.dtype)
    lse = lse.permute(1, 0, 2).reshape(Hq, T)
    return o, lse


def attention_bwd(do: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  o: torch.Tensor, lse: torch.Tensor, seq_len: int, scale: Optional[float] = None):
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    B = T // seq_len
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    qf = q.float().view(B, seq_len, Hq, D).transpose(1, 2)
    kf = k.float().view(B, seq_len, Hkv, D).transpose(1, 2).repeat_interleave(G, dim=1)
    vf = v.float().view(B, seq_len, Hkv, D).transpose(1, 2).repeat_interleave(G, dim=1)
    dof = do.float().view(B, seq_len, Hq, D).transpose(1, 2)
    of = o.float().view(B, seq_len, Hq, D).transpose(1, 2)
    lse_b = lse.view(Hq, B, seq_len).permute(1, 0, 2)
    s = (qf @ kf.transpose(-1, -2)) * scale
    mask = torch.ones(seq_len, seq_len, dtype=torch.bool, device=q.device).tril()
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.exp(s - lse_b[..., None])
    dv = p.transpose(-1, -2) @ dof
    dp = dof @ vf.transpose(-1, -2)
    delta = (dof * of).sum(-1, keepdim=True)
    ds = p * (dp - delta) * scale
    dq = ds @ kf
    dk = ds.transpose(-1, -2) @ qf
    dk = dk.view(B, Hkv, G, seq_len, D).sum(2)
    dv = dv.view(B, Hkv, G, seq_len, D).sum(2)
    dq = dq.transpose(1, 2).reshape(T, Hq, D).to(q.dtype)
    dk = dk.transpose(1, 2).reshape(T, Hkv, D).to(k.dtype)
    dv = dv.transpose(1, 2).reshape(T, Hkv, D).to(v.dtype)
    return dq, dk, dv


# ------------------------------------------------------------------ SwiGLU


def swiglu_fwd(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    g = gate.float()
    return (g * torch.sigmoid(g) * up.float()).to(gate.dtype)


def swiglu_bwd(da: torch.Tensor, gate: torch.Tensor, up: torch.Tensor):
    g, u, d = gate.float(), up.float(), da.float()
    sg = torch.sigmoid(g)
    silu = g * sg
    dg = d * u * sg * (1 + g * (1 - sg))
    du = d * silu
    return dg.to(gate.dtype), du.to(up.dtype)


# --------------------------------------------------------------- embedding


def embedding_fwd(ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return w[ids.reshape(-1)]


def embedding_bwd(dh: torch.Tensor, ids: torch.Tensor, num_rows: int,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    g = torch.zeros(num_rows, dh.shape[1], dtype=torch.float32, device=dh.device)
    g.index_add_(0, ids.reshape(-1), dh.float())
    if out is None:
        return g.to(dh.dtype)
    out.copy_(g.to(out.dtype))
    return out


# ----------------------------------------------------------- cross-entropy


def shift_labels(labels: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    """labels [B,S] -> per-position targets [B*S]: position s predicts
    labels[s+1]; the last position of each sequence is ignored."""
    out = torch.full_like(labels, ignore_index)
    out[:, :-1] = labels[:, 1:]
    return out.reshape(-1)


def cross_entropy_fwd_bwd(logits: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100,
                          grad_scale: Optional[float] = None):
    """Mean cross-entropy over targets != ignore_index and its gradient.
    Returns (loss fp32 scalar, dlogits in logits' dtype, n_valid).  The
    gradient is multiplied by ``grad_scale`` (default 1/n_valid)."""
    lf = logits.float()
    valid = targets != ignore_index
    n_valid = int(valid.sum())
    lse = torch.logsumexp(lf, dim=-1)
    tgt = targets.clamp_min(0)
    picked = lf.gather(1, tgt[:, None])[:, 0]
    per_tok = torch.where(valid, lse - picked, torch.zeros_like(lse))
    loss = per_tok.sum() / max(n_valid, 1)
    scale = grad_scale if grad_scale is not None else 1.0 / max(n_valid, 1)
    p = torch.exp(lf - lse[:, None])
    p[torch.arange(p.shape[0], device=p.device), tgt] -= 1.0
    p = p * valid[:, None].float() * scale
    return loss, p.to(logits.dtype), n_valid


def linear_cross_entropy(x: torch.Tensor, w: torch.Tensor, targets: torch.Tensor, dx: torch.Tensor,
                         dw: torch.Tensor, chunk_rows: int, ignore_index: int = -100):
    """Output layer without the [T, V] logits: mean cross-entropy of
    logits = x w^T over targets != ignore_index, processed in chunks of
    ``chunk_rows`` tokens.  Writes dx = dlogits w and dw = dlogits^T x (in
    fp32 arithmetic, rounded once into their dtype); returns (loss fp32
    scalar, n_valid)."""
    T = x.shape[0]
    valid = targets != ignore_index
    n_valid = int(valid.sum())
    scale = 1.0 / max(n_valid, 1)
    wf = w.float()
    dw32 = torch.zeros_like(wf)
    total = torch.zeros((), dtype=torch.float32, device=x.device)
    for t0 in range(0, T, max(1, chunk_rows)):
        t1 = min(T, t0 + chunk_rows)
        xc = x[t0:t1].float()
        logits = xc @ wf.t()
        loss_c, dl, n_c = cross_entropy_fwd_bwd(logits, targets[t0:t1], ignore_index, grad_scale=scale)
        total = total + loss_c * n_c  # loss_c is the chunk's mean over its n_c valid targets
        dx[t0:t1].copy_(dl @ wf)
        dw32 += dl.t() @ xc
    dw.copy_(dw32)
    return total / max(n_valid, 1), n_valid


# ------------------------------------------------ fused-layout entry points
# The model keeps q/k/v as column blocks of one [T, (Hq + 2 Hkv) * D] buffer
# and gate/up as the two halves of one [T, 2 I] buffer; these wrappers state
# the ops on those layouts (the kernels work on them in place).


def rope_qkv_(qkv: torch.Tensor, n_q: int, n_kv: int, head_dim: int, cos: torch.Tensor,
              sin: torch.Tensor, seq_len: int, inverse: bool = False) -> torch.Tensor:
    T = qkv.shape[0]
    D = head_dim
    q = qkv[:, : n_q * D].reshape(T, n_q, D)
    k = qkv[:, n_q * D:(n_q + n_kv) * D].reshape(T, n_kv, D)
    qkv[:, : n_q * D] = rope_apply(q, cos, sin, seq_len, inverse).reshape(T, -1)
    qkv[:, n_q * D:(n_q + n_kv) * D] = rope_apply(k, cos, sin, seq_len, inverse).reshape(T, -1)
    return qkv


def _split_qkv(qkv, n_q, n_kv, D):
    T = qkv.shape[0]
    q = qkv[:, : n_q * D].reshape(T, n_q, D)
    k = qkv[:, n_q * D:(n_q + n_kv) * D].reshape(T, n_kv, D)
    v = qkv[:, (n_q + n_kv) * D:].reshape(T, n_kv, D)
    return q, k, v


def attention_qkv_fwd(qkv: torch.Tensor, n_q: int, n_kv: int, head_dim: int, seq_len: int):
    q, k, v = _split_qkv(qkv, n_q, n_kv, head_dim)
    o, lse = attention_fwd(q, k, v, seq_len)
    return o.reshape(qkv.shape[0], n_q * head_dim), lse


def attention_qkv_bwd(do: torch.Tensor, qkv: torch.Tensor, o: torch.Tensor, lse: torch.Tensor,
                      n_q: int, n_kv: int, head_dim: int, seq_len: int) -> torch.Tensor:
    T = qkv.shape[0]
    q, k, v = _split_qkv(qkv, n_q, n_kv, head_dim)
    dq, dk, dv = attention_bwd(do.reshape(T, n_q, head_dim), q, k, v,
                               o.reshape(T, n_q, head_dim), lse, seq_len)
    return torch.cat([dq.reshape(T, -1), dk.reshape(T, -1), dv.reshape(T, -1)], dim=1)


def swiglu_gu_fwd(gu: torch.Tensor) -> torch.Tensor:
    I = gu.shape[1] // 2
    return swiglu_fwd(gu[:, :I], gu[:, I:])


def swiglu_gu_bwd(da: torch.Tensor, gu: torch.Tensor) -> torch.Tensor:
    I = gu.shape[1] // 2
    dg, du = swiglu_bwd(da, gu[:, :I], gu[:, I:])
    return torch.cat([dg, du], dim=1)
