"""Checkpoint ingestion on the GPU: a synthetic DeepSeek-V4-style draft checkpoint (packed
e2m1 experts with e8m0 group-32 scales, an fp8 shared expert with 128x128 e8m0 scales) is
read from safetensors shards straight onto the device and held packed. The MoE and the FFN
sub-layer built from it must match the oracle running on the weights as the reference's
loader leaves them, dequantised to fp32 (``dspark_mlx/loading.py:103-114``)."""

from __future__ import annotations

import pytest
import torch

import oracle
from checkpoint_fixture import make_checkpoint, reference_moe_weights, write_sharded
from dsm import MoE, _lib, loading
from dsm.block import DSparkFFN
from dsm.config import DSparkArgs
from helpers import MOE_TOL, max_rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCORE = dict(vocab_size=512, dim=512, moe_inter_dim=256, n_routed_experts=16, n_activated_experts=4,
             n_shared_experts=1, n_hash_layers=0, score_func="sigmoid", route_scale=2.5, swiglu_limit=10.0)
HASH = dict(SCORE, n_hash_layers=1, score_func="sqrtsoftplus", route_scale=1.5)


def _oracle_moe(t, args, prefix, x, ids):
    routed, shared = reference_moe_weights(t, prefix, args["n_routed_experts"])
    ws = {wk: oracle.OracleWeights("dense", routed[wk]) for wk in routed}
    g = lambda k: t.get(f"{prefix}.gate.{k}")  # noqa: E731
    return oracle.moe_forward(x, ids, gate_weight=g("weight").float(), topk=args["n_activated_experts"],
                              score_func=args["score_func"], route_scale=args["route_scale"],
                              swiglu_limit=args["swiglu_limit"], w1=ws["w1"], w3=ws["w3"], w2=ws["w2"],
                              shared=shared, gate_bias=g("bias"), tid2eid=g("tid2eid"))


@pytest.mark.parametrize("experts,n_tokens", [("fp4", 24), ("fp4", 700), ("fp8", 24), ("fp8", 700)])
def test_moe_from_checkpoint_matches_reference_dequant(tmp_path, experts, n_tokens):
    t = make_checkpoint(SCORE, layer_id=0, experts=experts, shared="fp8", seed=11)
    write_sharded(t, str(tmp_path), n_shards=2)
    dt = loading.read_draft_tensors(str(tmp_path), device=DEV)
    assert all(v.is_cuda for v in dt.values())
    moe = MoE(DSparkArgs.from_dict(SCORE), 0).to(DEV)
    loading.load_moe(moe, dt, "mtp.0.ffn")
    assert moe.expert_format == experts and moe.shared_experts.format == "fp8"
    x = torch.randn(n_tokens, SCORE["dim"], generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    y = moe(x.to(DEV))
    torch.cuda.synchronize()
    assert y.dtype == x.dtype and _lib.device_error() == 0
    ref = _oracle_moe(t, SCORE, "mtp.0.ffn", x, None)
    assert max_rel_err(y, ref) < MOE_TOL, max_rel_err(y, ref)


def test_ffn_sublayer_from_checkpoint_hash_routing(tmp_path):
    t = make_checkpoint(HASH, layer_id=0, experts="fp4", shared="fp8", seed=13)
    write_sharded(t, str(tmp_path), n_shards=3)
    dt = loading.read_draft_tensors(str(tmp_path), device=DEV)
    ffn = DSparkFFN(HASH, 0).to(DEV)
    loading.load_ffn_sublayer(ffn, dt, "mtp.0")
    g = torch.Generator().manual_seed(4)
    hc, dim = ffn.hc_mult, HASH["dim"]
    x = torch.randn(3, 7, hc, dim, generator=g).to(torch.bfloat16)
    ids = torch.randint(0, HASH["vocab_size"], (3, 7), generator=g, dtype=torch.int32)
    out = ffn(x.to(DEV), ids.to(DEV))
    torch.cuda.synchronize()
    assert out.shape == x.shape and _lib.device_error() == 0
    ref = oracle.ffn_sublayer(x, ids, moe=lambda xn, i: _oracle_moe(t, HASH, "mtp.0.ffn", xn, i),
                              hc_fn=t["mtp.0.hc_ffn_fn"], hc_scale=t["mtp.0.hc_ffn_scale"],
                              hc_base=t["mtp.0.hc_ffn_base"], norm_weight=t["mtp.0.ffn_norm.weight"].float(), hc=hc,
                              iters=ffn.hc_sinkhorn_iters, norm_eps=ffn.norm_eps, hc_eps=ffn.hc_eps)
    assert max_rel_err(out, ref) < MOE_TOL, max_rel_err(out, ref)
