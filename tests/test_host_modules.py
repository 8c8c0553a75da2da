"""Host-side behaviour of the GPU-only modules (CPU, no device): inputs on the CPU are
refused, since the package has no CPU path."""

from __future__ import annotations

import pytest
import torch

ARGS = dict(vocab_size=64, dim=256, moe_inter_dim=128, n_routed_experts=8, n_activated_experts=2,
            n_shared_experts=1, n_hash_layers=0, score_func="sigmoid", route_scale=2.5, swiglu_limit=10.0)


def test_gpu_modules_reject_cpu_tensors():
    from dsm.attention import DSparkAttention
    from dsm.head import DSparkHead

    args = dict(ARGS, hc_mult=2, dspark_markov_rank=16, n_heads=4, head_dim=32, rope_head_dim=16, q_lora_rank=48,
                o_groups=2, o_lora_rank=24, window_size=8)
    with pytest.raises(ValueError, match="GPU"):
        DSparkHead(args)(torch.zeros(1, 2, 2, 256), torch.zeros(1, dtype=torch.int32))
    with pytest.raises(ValueError, match="GPU"):
        DSparkAttention(args, max_seq_len=16)(torch.zeros(1, 3, 256), 0, torch.zeros(1, 4, 256))
    with pytest.raises(ValueError, match="GPU"):
        from dsm.qwen3 import Qwen3MLP

        Qwen3MLP(dict(hidden_size=256, intermediate_size=512))(torch.zeros(2, 256))
    with pytest.raises(ValueError):
        from dsm import MoE
        from dsm.config import DSparkArgs

        MoE(DSparkArgs.from_dict(ARGS), 0)(torch.zeros(2, 256))
