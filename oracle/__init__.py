"""CPU oracle for the DSpark draft-layer MoE block.

Test infrastructure only: the checker the CUDA path is compared against. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import this package;
the product package (``dsm``) never does and has no CPU fallback.
"""

from .moe_oracle import *  # noqa: F401,F403
from .formats import *  # noqa: F401,F403
from .block_oracle import *  # noqa: F401,F403
from .head_oracle import *  # noqa: F401,F403
from .attention_oracle import *  # noqa: F401,F403
from .qwen3_attn_oracle import *  # noqa: F401,F403
from .draft_block_oracle import *  # noqa: F401,F403
from .drafter_oracle import *  # noqa: F401,F403
