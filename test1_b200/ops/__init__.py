"""Ops of the Llama training step.

Every function takes and returns plain tensors.  CUDA tensors run the
hand-written sm_100a kernels of ``test1_b200._cuda`` (``ops.native``); CPU
tensors run the PyTorch statements in ``ops.reference`` (the oracle, and the
path of the CPU/gloo tests).  There is no silent fallback on the GPU: if the
CUDA extension is missing, the first op raises.

Setting ``T1_OPS=torch`` runs the PyTorch statements on CUDA tensors too; it
exists only to measure the framework against library kernels and is never
the default.
"""
from __future__ import annotations

import os

from . import reference

_FORCE_TORCH = os.environ.get("T1_OPS", "native").lower() == "torch"


def use_native(t) -> bool:
    return t.is_cuda and not _FORCE_TORCH


def _impl(t):
    if use_native(t):
        from . import native

        return native
    return reference


def rmsnorm_fwd(x, w, eps):
    return _impl(x).rmsnorm_fwd(x, w, eps)


def rmsnorm_bwd(dy, x, w, rstd, residual_grad=None):
    return _impl(x).rmsnorm_bwd(dy, x, w, rstd, residual_grad)


def linear_fwd(x, w, residual=None):
    return _impl(x).linear_fwd(x, w, residual)


def linear_fwd_rope(x, w, cos, sin, seq_len, n_q, n_kv, head_dim):
    """QKV projection with the rotary embedding of the q and k heads applied:
    x @ w^T, then rotate column blocks [0, (n_q + n_kv) head_dim) by position
    t % seq_len (on the GPU fused into the GEMM epilogue when possible)."""
    return _impl(x).linear_fwd_rope(x, w, cos, sin, seq_len, n_q, n_kv, head_dim)


def linear_dgrad(dy, w):
    return _impl(dy).linear_dgrad(dy, w)


def linear_wgrad(dy, x, out=None):
    return _impl(dy).linear_wgrad(dy, x, out)


def rope_qkv_(qkv, n_q, n_kv, head_dim, cos, sin, seq_len, inverse=False):
    """Rotate the q and k column blocks of ``qkv`` [T, (n_q+2 n_kv) D] in place."""
    return _impl(qkv).rope_qkv_(qkv, n_q, n_kv, head_dim, cos, sin, seq_len, inverse)


def attention_fwd(qkv, n_q, n_kv, head_dim, seq_len):
    """Causal GQA attention on the fused qkv buffer -> (o [T, n_q D], lse [n_q, T])."""
    return _impl(qkv).attention_qkv_fwd(qkv, n_q, n_kv, head_dim, seq_len)


def attention_bwd(do, qkv, o, lse, n_q, n_kv, head_dim, seq_len):
    """-> dqkv [T, (n_q + 2 n_kv) D] (gradients of the rotated q, k and of v)."""
    return _impl(qkv).attention_qkv_bwd(do, qkv, o, lse, n_q, n_kv, head_dim, seq_len)


def swiglu_fwd(gu):
    """gu [T, 2I] = [gate | up] -> silu(gate) * up [T, I]."""
    return _impl(gu).swiglu_gu_fwd(gu)


def swiglu_bwd(da, gu):
    """-> dgu [T, 2I] = [dgate | dup]."""
    return _impl(gu).swiglu_gu_bwd(da, gu)


def embedding_fwd(ids, w):
    return _impl(w).embedding_fwd(ids, w)


def embedding_bwd(dh, ids, num_rows, out=None):
    return _impl(dh).embedding_bwd(dh, ids, num_rows, out)


def cross_entropy_fwd_bwd(logits, targets, ignore_index=-100, grad_scale=None):
    return _impl(logits).cross_entropy_fwd_bwd(logits, targets, ignore_index, grad_scale)


def linear_cross_entropy(x, w, targets, dx, dw, chunk_rows, ignore_index=-100):
    """Output layer's lm_head GEMM + cross-entropy forward and backward in
    token chunks (no [T, V] logits kept): writes dx [T, H] and dw [V, H],
    returns (loss fp32 scalar, n_valid)."""
    return _impl(x).linear_cross_entropy(x, w, targets, dx, dw, chunk_rows, ignore_index)


shift_labels = reference.shift_labels
rope_tables = reference.rope_tables


def native_launch_count() -> int:
    """Number of sm_100a kernel launches issued through ``ops.native`` so far."""
    import sys

    mod = sys.modules.get(__name__ + ".native")
    return 0 if mod is None else mod.launch_count()
