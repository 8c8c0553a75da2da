"""Checkpoint ingestion (host logic, CPU): key mapping and shard selection
(``dspark_mlx/loading.py:49-54``, ``dspark_mlx/loader.py:87-107``), expert stacking
(``loading.py:88-100``), and the exact e8m0 -> packed-format scale conversion against the
oracle's restatement of the reference's dequant helpers (``loading.py:103-114``)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from checkpoint_fixture import make_checkpoint, reference_moe_weights, write_sharded
from dsm import MoE, loading
from dsm.block import DSparkFFN
from dsm.config import DSparkArgs

ARGS = dict(vocab_size=64, dim=256, moe_inter_dim=128, n_routed_experts=8, n_activated_experts=2,
            n_shared_experts=1, n_hash_layers=0, score_func="sigmoid", route_scale=2.5, swiglu_limit=10.0)


def test_e8m0_decode_matches_torch_cast():
    codes = np.arange(256, dtype=np.uint8)
    mine = oracle.e8m0_decode(codes)
    lib = torch.from_numpy(codes).view(torch.float8_e8m0fnu).to(torch.float32)
    assert torch.isnan(mine[255]) and torch.isnan(lib[255])
    assert torch.equal(mine[:255], lib[:255])


def test_map_checkpoint_key():
    # the reference's own cases (tests/test_loading.py:33-39)
    assert loading.map_checkpoint_key("mtp.0.attn.wq_a.weight") == "blocks.0.attn.wq_a.weight"
    assert loading.map_checkpoint_key("mtp.2.markov_head.markov_w1.weight") == "blocks.2.markov_head.markov_w1.weight"
    assert loading.map_checkpoint_key("embed.weight") == "embed.weight"
    assert loading.map_checkpoint_key("head.weight") == "head.weight"
    assert loading.map_checkpoint_key("layers.0.attn.wkv.weight") is None


def test_draft_shards_selects_only_the_draft():
    # the reference's own case (tests/test_loader_deepseek.py:31-46)
    wm = {"embed.weight": "s1", "head.weight": "s1", "layers.0.attn.wq_a.weight": "s2",
          "layers.30.ffn.experts.3.w1.weight": "s3", "mtp.0.attn.wq_a.weight": "s9",
          "mtp.0.ffn.experts.5.w1.weight": "s9", "mtp.2.markov_head.markov_w1.weight": "s10"}
    keep, shards = loading.draft_shards(wm)
    assert keep == {"embed.weight", "head.weight", "mtp.0.attn.wq_a.weight", "mtp.0.ffn.experts.5.w1.weight",
                    "mtp.2.markov_head.markov_w1.weight"}
    assert shards == ["s1", "s10", "s9"]  # sorted, unique; the base-only shards are never opened


def test_e8m0_to_fp32_every_code_exact():
    codes = torch.arange(255, dtype=torch.uint8)
    exp = oracle.e8m0_decode(codes.numpy())
    assert torch.equal(loading.e8m0_to_fp32(codes), exp)
    assert torch.equal(loading.e8m0_to_fp32(codes.view(torch.float8_e8m0fnu)), exp)
    assert torch.equal(loading.e8m0_to_fp32(exp), exp)  # already-decoded powers of two
    with pytest.raises(ValueError, match="NaN"):
        loading.e8m0_to_fp32(torch.tensor([255], dtype=torch.uint8))
    with pytest.raises(ValueError, match="powers of two"):
        loading.e8m0_to_fp32(torch.tensor([0.75]))


def _fp4_case(E, R, K, lo, hi, seed):
    g = torch.Generator().manual_seed(seed)
    nib = torch.randint(0, 16, (E, R, K), generator=g, dtype=torch.int32)
    codes = (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8)
    x = torch.randint(lo, hi + 1, (E, R, K // 32), generator=g)
    return codes, (x + 127).to(torch.uint8)


def _reference_fp4(codes, scale):
    nib = torch.stack([codes & 0xF, codes >> 4], dim=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2)
    return oracle.dequant_fp4_groupwise(oracle.e2m1_decode(nib.numpy()), oracle.e8m0_decode(scale.numpy()), 32)


@pytest.mark.parametrize("lo,hi", [(-12, -6), (-127, -110), (100, 117), (-30, -13), (0, 0)])
def test_fp4_scale_split_is_exact(lo, hi):
    codes, scale = _fp4_case(4, 16, 256, lo, hi, seed=lo & 0xFF)
    gs, ts = loading.fp4_scales_from_e8m0(codes, scale)
    assert gs.dtype == torch.uint8 and ts.dtype == torch.float32 and ts.shape == (4,)
    mine = oracle.fp4_weight_dequant(codes, gs, ts)  # the packed format's own dequantisation
    assert torch.equal(mine, _reference_fp4(codes, scale))


def test_fp4_scale_split_zero_groups_and_out_of_range():
    codes, scale = _fp4_case(2, 8, 128, -8, -5, seed=1)
    far = scale.clone()
    codes_z = codes.clone()
    codes_z[1, 3, 0:16] = 0x88  # one group of -0 codes in expert 1
    far[1, 3, 0] = 127 - 60     # far below the rest: harmless, the group is all zeros
    gs, ts = loading.fp4_scales_from_e8m0(codes_z, far)
    assert torch.equal(oracle.fp4_weight_dequant(codes_z, gs, ts), _reference_fp4(codes_z, far))
    far[1, 3, 1] = 127 - 60     # a nonzero group out of range
    with pytest.raises(ValueError, match="expert 1"):
        loading.fp4_scales_from_e8m0(codes_z, far)
    allzero = torch.zeros_like(codes)
    gs, ts = loading.fp4_scales_from_e8m0(allzero, scale)
    assert torch.equal(oracle.fp4_weight_dequant(allzero, gs, ts), torch.zeros(2, 8, 128))


def test_stack_experts_orders_by_id_and_checks_scales():
    t = {f"mtp.0.ffn.experts.{e}.w1.weight": torch.full((2, 2), float(e)) for e in (2, 0, 1)}
    t["mtp.1.ffn.experts.0.w1.weight"] = torch.zeros(2, 2)  # another block: ignored
    st = loading.stack_experts(t, "mtp.0.ffn")
    assert set(st) == {"w1"} and st["w1"][1] is None
    assert torch.equal(st["w1"][0][:, 0, 0], torch.tensor([0.0, 1.0, 2.0]))
    t["mtp.0.ffn.experts.1.w1.scale"] = torch.ones(1)
    with pytest.raises(ValueError, match="some experts have a .scale"):
        loading.stack_experts(t, "mtp.0.ffn")
    del t["mtp.0.ffn.experts.1.w1.scale"], t["mtp.0.ffn.experts.1.w1.weight"]
    with pytest.raises(ValueError, match="expert ids"):
        loading.stack_experts(t, "mtp.0.ffn")


def test_read_draft_tensors_opens_only_draft_shards(tmp_path):
    t = make_checkpoint(ARGS, layer_id=0, experts="fp4", shared="fp8", seed=3)
    t["embed.weight"] = torch.randn(64, 256).to(torch.bfloat16)
    write_sharded(t, str(tmp_path), n_shards=3, base_shard=True)
    got = loading.read_draft_tensors(str(tmp_path))  # the base shard is not safetensors: never opened
    assert set(got) == set(t)
    for k, v in t.items():
        assert got[k].dtype == v.dtype and torch.equal(got[k].view(torch.uint8), v.view(torch.uint8))
    sub = loading.read_draft_tensors(str(tmp_path), keys=["mtp.0.ffn.gate.weight", "layers.0.ffn.gate.weight"])
    assert set(sub) == {"mtp.0.ffn.gate.weight"}


@pytest.mark.parametrize("experts,shared,layer_id", [("fp4", "fp8", 0), ("fp8", "fp8", 0), ("bf16", "bf16", 0),
                                                     ("fp4", "fp8", 1)])
def test_load_moe_holds_packed_weights_equal_to_reference_dequant(experts, shared, layer_id):
    args = dict(ARGS, n_hash_layers=1) if layer_id == 0 and experts == "fp4" and shared == "fp8" else dict(ARGS)
    t = make_checkpoint(args, layer_id=layer_id, experts=experts, shared=shared, seed=5)
    moe = MoE(DSparkArgs.from_dict(args), layer_id)
    used = loading.load_moe(moe, t, "mtp.0.ffn")
    assert set(used) == {k for k in t if k.startswith("mtp.0.ffn.")}
    routed, sh = reference_moe_weights(t, "mtp.0.ffn", args["n_routed_experts"])
    if experts == "fp4":
        assert moe.expert_format == "fp4"
        for wk in ("w1", "w2", "w3"):
            mine = oracle.fp4_weight_dequant(getattr(moe, f"{wk}_codes"), getattr(moe, f"{wk}_scale"),
                                             getattr(moe, f"{wk}_tensor_scale"))
            assert torch.equal(mine, routed[wk])
    elif experts == "fp8":
        assert moe.expert_format == "fp8"
        for wk in ("w1", "w2", "w3"):
            mine = oracle.fp8_weight_dequant(getattr(moe, f"{wk}_codes"), getattr(moe, f"{wk}_scale"))
            assert torch.equal(mine, routed[wk])
    else:
        assert moe.expert_format == "dense"
        for wk in ("w1", "w2", "w3"):
            assert torch.equal(getattr(moe, wk).float(), routed[wk])
    ex = moe.shared_experts
    for i, wk in enumerate(("w1", "w2", "w3")):
        if shared == "fp8":
            assert ex.format == "fp8" and ex.weight_dtype(wk) == torch.float32
            assert torch.equal(oracle.fp8_weight_dequant(getattr(ex, f"{wk}_codes"), getattr(ex, f"{wk}_scale")), sh[i])
        else:
            assert ex.format == "dense" and torch.equal(getattr(ex, wk).weight.float(), sh[i])
    assert torch.equal(moe.gate.weight, t["mtp.0.ffn.gate.weight"].float())
    if moe.gate.hash:
        assert torch.equal(moe.gate.tid2eid, t["mtp.0.ffn.gate.tid2eid"])
    else:
        assert torch.equal(moe.gate.bias, t["mtp.0.ffn.gate.bias"])


def test_load_ffn_sublayer_and_errors():
    t = make_checkpoint(ARGS, layer_id=0, experts="fp4", shared="fp8", seed=7)
    ffn = DSparkFFN(ARGS, 0)
    used = loading.load_ffn_sublayer(ffn, t, "mtp.0")
    assert set(used) == set(t)
    assert torch.equal(ffn.hc_ffn_fn, t["mtp.0.hc_ffn_fn"]) and torch.equal(ffn.ffn_norm.weight,
                                                                            t["mtp.0.ffn_norm.weight"].float())
    bad = dict(t)
    bad["mtp.0.ffn.experts.3.w2.weight"] = torch.zeros(256, 128, dtype=torch.bfloat16)
    del bad["mtp.0.ffn.experts.3.w2.scale"]
    with pytest.raises(ValueError):
        loading.load_moe(MoE(DSparkArgs.from_dict(ARGS), 0), bad, "mtp.0.ffn")
    small = dict(ARGS, moe_inter_dim=64)
    with pytest.raises(ValueError, match="expected"):
        loading.load_moe(MoE(DSparkArgs.from_dict(small), 0), t, "mtp.0.ffn")


def test_shared_fp8_expert_survives_to():
    t = make_checkpoint(ARGS, layer_id=0, experts="fp4", shared="fp8", seed=9)
    moe = MoE(DSparkArgs.from_dict(ARGS), 0)
    loading.load_moe(moe, t, "mtp.0.ffn")
    moe = moe.to(torch.device("cpu"))  # meta placeholders stay placeholders
    assert moe.shared_experts.format == "fp8" and moe.shared_experts.w1.weight.is_meta

