"""Python wrappers of the sm_100a kernels in ``test1_b200._cuda``.

Each function has the signature of its namesake in ``ops.reference`` and
returns tensors of the same layout.  Shapes/dtypes are checked in C++.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _native
from . import reference as _ref

_C = None


def _c():
    global _C
    if _C is None:
        _C = _native.cuda()
    return _C


def launch_count() -> int:
    return int(_c().launch_count()) if _C is not None else 0


# ------------------------------------------------------------------ RMSNorm
def rmsnorm_fwd(x, w, eps):
    y, rstd = _c().rmsnorm_fwd(x, w, float(eps))
    return y, rstd


def rmsnorm_bwd(dy, x, w, rstd, residual_grad=None):
    dx, dw = _c().rmsnorm_bwd(dy, x, w, rstd, residual_grad)
    return dx, dw


# ------------------------------------------------------------------- Linear
def linear_fwd(x, w, residual=None):
    out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    _c().gemm_bf16(x, w, out, False, False, residual)
    return out


def rope_fusable(head_dim) -> bool:
    """The GEMM epilogue applies RoPE for head_dim 128 in GEMM mode 2."""
    return head_dim == 128 and gemm_get_mode() == 2


def linear_fwd_rope(x, w, cos, sin, seq_len, n_q, n_kv, head_dim):
    out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    if rope_fusable(head_dim) and x.is_contiguous() and w.is_contiguous():
        _c().gemm_bf16_rope(x, w, out, cos, sin, int(seq_len), int((n_q + n_kv) * head_dim))
        return out
    _c().gemm_bf16(x, w, out, False, False, None)
    return rope_qkv_(out, n_q, n_kv, head_dim, cos, sin, seq_len)


def linear_dgrad(dy, w):
    out = torch.empty(dy.shape[0], w.shape[1], dtype=dy.dtype, device=dy.device)
    _c().gemm_bf16(dy, w, out, False, True, None)
    return out


def linear_wgrad(dy, x, out=None):
    if out is None:
        out = torch.empty(dy.shape[1], x.shape[1], dtype=dy.dtype, device=dy.device)
    _c().gemm_bf16(dy, x, out, True, True, None)
    return out


def gemm(a, b, c, a_mn=False, b_mn=False, residual=None):
    _c().gemm_bf16(a, b, c, a_mn, b_mn, residual)
    return c


def gemm_set_streamk(on: bool) -> None:
    """Stream-K tail of the default (TMA-store) pair GEMM: the last partial
    wave of tiles is split along K over otherwise idle clusters."""
    _c().gemm_set_streamk(bool(on))


def gemm_set_mode(mode: int) -> None:
    """0: single-CTA 128x256 tiles; 1: CTA-pair (cta_group::2) 256x256 tiles."""
    _c().gemm_set_mode(int(mode))


def gemm_get_mode() -> int:
    return int(_c().gemm_get_mode())


def attn_set_mode(mode: int) -> None:
    """Attention: 0 = mma.sync tiles, 1 = tcgen05 (TMEM accumulators, one
    128-row query tile per CTA), 2 = tcgen05 forward with two query tiles per
    CTA in ping-pong (the default; sequences not a multiple of 256 use 1)."""
    _c().attn_set_mode(int(mode))


def attn_set_bwd_pipelined(on: bool) -> None:
    """tcgen05 attention backward: the pipelined kernel (default; Q
    double-buffered, dQ drained while dK runs, the next scores computed
    during the drain) or the serial one."""
    _c().attn_set_bwd_pipelined(bool(on))


def attn_fwd2_set_poly(n: int) -> None:
    """Two-tile forward: how many of every 8 exponentials run as a polynomial
    on the FMA pipe instead of the MUFU unit (0, 1 or 2)."""
    _c().attn_fwd2_set_poly(int(n))


def attention_fwd_tc2(qkv, n_q, n_kv, seq_len):
    """The two-tile tcgen05 forward directly (seq_len % 256 == 0)."""
    return _c().attention_fwd_tc2(qkv, n_q, n_kv, seq_len)


def attn_get_mode() -> int:
    return int(_c().attn_get_mode())


def gemm_error(reset: bool = False) -> int:
    return int(_c().gemm_check_error(reset))


# --------------------------------------------------------------------- RoPE
def rope_qkv_(qkv, n_q, n_kv, head_dim, cos, sin, seq_len, inverse=False):
    _c().rope_qkv(qkv, n_q, n_kv, head_dim, cos, sin, seq_len, inverse)
    return qkv


# ---------------------------------------------------------------- attention
def attention_qkv_fwd(qkv, n_q, n_kv, head_dim, seq_len):
    C = _c()
    if hasattr(C, "attention_fwd"):
        return C.attention_fwd(qkv, n_q, n_kv, head_dim, seq_len)
    raise NotImplementedError("native attention kernel not built")


def attention_qkv_bwd(do, qkv, o, lse, n_q, n_kv, head_dim, seq_len):
    C = _c()
    if hasattr(C, "attention_bwd"):
        return C.attention_bwd(do, qkv, o, lse, n_q, n_kv, head_dim, seq_len)
    raise NotImplementedError("native attention kernel not built")


# ------------------------------------------------------------------- SwiGLU
def swiglu_gu_fwd(gu):
    return _c().swiglu_fwd(gu)


def swiglu_gu_bwd(da, gu):
    return _c().swiglu_bwd(da, gu)


# ---------------------------------------------------------------- embedding
def embedding_fwd(ids, w):
    return _c().embedding_fwd(ids, w)


def embedding_bwd(dh, ids, num_rows, out=None):
    if out is None:
        out = torch.empty(num_rows, dh.shape[1], dtype=dh.dtype, device=dh.device)
    _c().embedding_bwd(dh, ids, out)
    return out


# ----------------------------------------------- chunked linear cross-entropy
def linear_cross_entropy(x, w, targets, dx, dw, chunk_rows, ignore_index=-100):
    loss, count = _c().linear_cross_entropy(x, w, targets, dx, dw, int(chunk_rows), int(ignore_index))
    return loss.reshape(()), count


# ------------------------------------------------------------ cross-entropy
def cross_entropy_fwd_bwd(logits, targets, ignore_index=-100, grad_scale=None):
    """Overwrites ``logits`` with the gradient; returns (loss [] fp32 on the
    device, dlogits (= logits), n_valid [1] int32 on the device)."""
    loss, count = _c().cross_entropy_fwd_bwd(logits, targets, int(ignore_index),
                                             -1.0 if grad_scale is None else float(grad_scale))
    return loss.reshape(()), logits, count
