"""Multi-GPU building blocks: process groups, symmetric (peer-mapped) device
buffers and the expert-parallel MoE exchange."""
from .dist import ParallelState, init_distributed
from .ep_moe import EPMoE
from .symm import SymmetricBuffer
from .tp import TPGroup, head_split

__all__ = ["ParallelState", "init_distributed", "SymmetricBuffer", "EPMoE", "TPGroup", "head_split"]
