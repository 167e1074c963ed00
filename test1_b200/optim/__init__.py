from .layer_adam import LayerAdam, reference_adamw_

__all__ = ["LayerAdam", "reference_adamw_"]
