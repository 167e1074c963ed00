"""One GEMM shape, a few launches: the small case for an ncu capture of the
tcgen05 GEMM (Llama-3.1-8B QKV projection: 4096 x 6144 x 4096, ~130 MB of
operands).  Usage: python benchmark/gemm_profile_case.py [fwd|dgrad|wgrad] [--pair | --pair-tma]
[--shape qkv|o|down] (--pair: CTA pairs with the register-store epilogue;
--pair-tma: CTA pairs with the shared-memory + TMA-store epilogue, the
default; --shape: the QKV (default), O (4096^3, a stream-K tail) or down
(4096 x 4096 x 14336) projection)."""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from test1_b200.ops import native  # noqa: E402


def main() -> None:
    kind = sys.argv[1] if len(sys.argv) > 1 and not sys.argv[1].startswith("--") else "fwd"
    if "--pair-tma" in sys.argv:
        native.gemm_set_mode(2)
    elif "--pair" in sys.argv:
        native.gemm_set_mode(1)
    shape = sys.argv[sys.argv.index("--shape") + 1] if "--shape" in sys.argv else "qkv"
    M, N, K = {"qkv": (4096, 6144, 4096), "o": (4096, 4096, 4096), "down": (4096, 4096, 14336)}[shape]
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    dy = torch.randn(M, N, device="cuda").bfloat16()
    for _ in range(3):
        if kind == "fwd":
            native.gemm(x, w, torch.empty(M, N, device="cuda", dtype=torch.bfloat16))
        elif kind == "dgrad":
            native.gemm(dy, w, torch.empty(M, K, device="cuda", dtype=torch.bfloat16), False, True)
        else:
            native.gemm(dy, x, torch.empty(N, K, device="cuda", dtype=torch.bfloat16), True, True)
    torch.cuda.synchronize()
    assert native.gemm_error() == 0
    print("ok", kind)


if __name__ == "__main__":
    main()
