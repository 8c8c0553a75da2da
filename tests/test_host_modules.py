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


QWEN3_ARGS = dict(hidden_size=96, num_attention_heads=4, num_key_value_heads=2, head_dim=32, rms_norm_eps=1e-6)


def test_qwen3_attention_rejects_cpu_tensors_and_bad_arguments():
    from dsm.qwen3_attention import Qwen3DSparkAttention

    a = Qwen3DSparkAttention(QWEN3_ARGS)
    cos, sin = torch.zeros(9, 32), torch.zeros(9, 32)
    with pytest.raises(ValueError, match="GPU"):
        a(torch.zeros(1, 4, 96), torch.zeros(1, 5, 96), cos, sin)
    with pytest.raises(ValueError, match="GPU"):
        a.context_kv(torch.zeros(1, 5, 96), cos[:5], sin[:5])
    with pytest.raises(ValueError, match="GPU"):
        a.attend_cached(torch.zeros(1, 4, 96), None, None, cos[:4], sin[:4])
    with pytest.raises(ValueError, match="multiple"):
        Qwen3DSparkAttention(dict(QWEN3_ARGS, num_key_value_heads=3))


def test_qwen3_rope_tables_match_the_oracle():
    import oracle
    from dsm.qwen3_attention import rope_tables

    for pos in (torch.arange(13), torch.arange(2048, 2055)):
        mine = rope_tables(pos, 128, 1000000.0)
        ref = oracle.qwen3_rope_tables(pos, 128, 1000000.0)
        assert torch.equal(mine[0], ref[0]) and torch.equal(mine[1], ref[1])


def test_qwen3_layer_rejects_cpu_tensors():
    from dsm.qwen3_layer import Qwen3DSparkLayer

    layer = Qwen3DSparkLayer(dict(QWEN3_ARGS, intermediate_size=128))
    with pytest.raises(ValueError, match="GPU"):
        layer(torch.zeros(1, 4, 96), torch.zeros(1, 5, 96), torch.zeros(9, 32), torch.zeros(9, 32))
    with pytest.raises(ValueError, match="GPU"):
        layer.forward_cached(torch.zeros(1, 4, 96), None, None, torch.zeros(4, 32), torch.zeros(4, 32))


def test_draft_block_rejects_cpu_tensors_and_wrong_stages():
    from dsm.draft_block import DSparkBlock
    from test_oracle_draft_block import ARGS

    blk = DSparkBlock(ARGS, 0, max_seq_len=16)
    with pytest.raises(ValueError, match="GPU"):
        blk(torch.zeros(1, 5, 4, 256), 3, torch.zeros(1, dtype=torch.int32), torch.zeros(1, 1, 256))
    with pytest.raises(ValueError, match="GPU"):
        blk.forward_embed(torch.zeros(1, 3, 768), torch.zeros(1, dtype=torch.int32), blk.main_proj)
    later = DSparkBlock(dict(ARGS, n_mtp_layers=3), 1, max_seq_len=16)
    assert not hasattr(later, "main_proj") and not hasattr(later, "markov_head")
    with pytest.raises(ValueError, match="stage 0"):
        later.forward_embed(torch.zeros(1, 3, 768), torch.zeros(1, dtype=torch.int32), None)
    with pytest.raises(ValueError, match="last stage"):
        later.forward_head(torch.zeros(1, 5, 4, 256), torch.zeros(1, dtype=torch.int32), None)
