"""test1_b200: a Blackwell-native layer-sliding offload trainer.

Public API (same names as the SlideFSDP reference):
    SlideFSDPConfig, SlideFSDP, LayerAdam, SlidingCheckpoint
"""
from .config import SlideFSDPConfig
from .optim.layer_adam import LayerAdam

__all__ = ["SlideFSDPConfig", "SlideFSDP", "LayerAdam", "SlidingCheckpoint", "LlamaConfig",
           "LlamaForCausalLM"]
__version__ = "0.1.0"


def __getattr__(name):
    if name == "SlideFSDP":
        from .slide_fsdp import SlideFSDP

        return SlideFSDP
    if name == "SlidingCheckpoint":
        from .sliding_checkpoint import SlidingCheckpoint

        return SlidingCheckpoint
    if name in ("LlamaConfig", "LlamaForCausalLM"):
        from .models import llama

        return getattr(llama, name)
    raise AttributeError(name)
