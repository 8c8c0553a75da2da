"""dsm: a B200 (sm_100a) DSpark draft-layer MoE behind the reference ``MoE`` interface.

``dsm.MoE(args, layer_id)(x, input_ids)`` is a drop-in for ``dspark_mlx.model.moe.MoE``;
every call runs hand-written CUDA kernels from ``libdsm.so`` (C ABI in ``include/dsm.h``).
"""

from .config import DSparkArgs
from .moe import Expert, Gate, MoE
from .weights import PackedMatrix, affine_quantize, pack

__all__ = ["DSparkArgs", "Gate", "Expert", "MoE", "PackedMatrix", "pack", "affine_quantize"]
