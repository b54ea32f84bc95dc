from .layers import Attention, Norm
from .model import QuantaWeaveBlock, QuantaWeaveMoEForCausalLM
from .moe import SparseSwiGLU, TopKMoE

__all__ = ["Attention", "Norm", "QuantaWeaveBlock", "QuantaWeaveMoEForCausalLM", "SparseSwiGLU", "TopKMoE"]
