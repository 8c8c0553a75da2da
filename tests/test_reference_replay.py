"""Replay the reference's own MoE unit tests through the PyTorch stand-in for ``mlx``.

This pins the stand-in that generated the golden vectors: the reference's assertions
(``tests/test_moe_gather_mm.py`` and the dequant cases of ``tests/test_loading.py``) must
hold when its code runs over it. Runs only where the reference source tree is present.
"""

from __future__ import annotations

import importlib.util
import os

import pytest

REF = os.environ.get("DSPARK_REFERENCE", "/root/reference")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "dspark_mlx")),
                                reason="reference source tree not present")


def _load_test_module(path):
    import make_golden  # noqa: F401  (tests/golden on sys.path via conftest)

    spec = importlib.util.spec_from_file_location(os.path.basename(path)[:-3], path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def reference():
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import make_golden

    return make_golden.load_reference(REF)


def test_reference_moe_unit_tests(reference):
    mod = _load_test_module(os.path.join(REF, "tests", "test_moe_gather_mm.py"))
    mod.test_sparse_matches_dense()
    mod.test_quantized_paths_close()
    mod.test_loader_stacks_experts()


def test_reference_dequant_unit_tests(reference):
    mod = _load_test_module(os.path.join(REF, "tests", "test_loading.py"))
    mod.test_dequant_fp8_blockwise()
    mod.test_dequant_fp4_groupwise()


def test_qwen3_attention_oracle_matches_reference_torch_model(reference):
    """The reference pins its Qwen3 backbone to a torch transcription of DeepSpec's model
    (``tests/qwen3_ref.py``, ``tests/test_qwen3_arch.py:30-60``): the rope tables against a
    numpy formula within 1e-5, the layer within 2e-3. The oracle's attention is held to the
    same torch model's ``RefAttn`` in fp32, on the reference test's shapes and weight scale."""
    import numpy as np
    import torch

    import oracle

    import sys

    # transformers probes for an installed mlx; the stand-in must not be visible to it
    shim_mods = {k: sys.modules.pop(k) for k in list(sys.modules) if k == "mlx" or k.startswith("mlx.")}
    try:
        ref = _load_test_module(os.path.join(REF, "tests", "qwen3_ref.py"))
    finally:
        sys.modules.update(shim_mods)
    h, nh, nkv, hd, eps, theta = 32, 4, 2, 16, 1e-6, 1_000_000.0
    rng = np.random.default_rng(0)
    attn = ref.RefAttn(h, nh, nkv, hd, eps)
    weights = {k: torch.tensor((rng.standard_normal(tuple(v.shape)) * 0.05).astype(np.float32))
               for k, v in attn.state_dict().items()}
    weights["q_norm.weight"] = weights["q_norm.weight"] + 1
    weights["k_norm.weight"] = weights["k_norm.weight"] + 1
    attn.load_state_dict(weights)
    b, ctx, block = 2, 5, 3
    noise = torch.tensor((rng.standard_normal((b, block, h)) * 0.3).astype(np.float32))
    target = torch.tensor((rng.standard_normal((b, ctx, h)) * 0.3).astype(np.float32))
    positions = np.arange(ctx + block)
    inv = 1.0 / (theta ** (np.arange(0, hd, 2) / hd))
    emb = np.concatenate([positions[:, None] * inv[None, :]] * 2, axis=-1)
    cos_np, sin_np = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    cos, sin = oracle.qwen3_rope_tables(torch.from_numpy(positions), hd, theta)
    assert np.max(np.abs(cos.numpy() - cos_np)) < 1e-5 and np.max(np.abs(sin.numpy() - sin_np)) < 1e-5
    p = {"q_proj": weights["q_proj.weight"], "k_proj": weights["k_proj.weight"], "v_proj": weights["v_proj.weight"],
         "o_proj": weights["o_proj.weight"], "q_norm": weights["q_norm.weight"], "k_norm": weights["k_norm.weight"]}
    with torch.no_grad():
        want = attn(noise, target, torch.from_numpy(cos_np), torch.from_numpy(sin_np))
    got = oracle.qwen3_attention(p, nh, nkv, hd, eps, noise, target, torch.from_numpy(cos_np),
                                 torch.from_numpy(sin_np))
    assert float((got - want).abs().max()) <= 1e-5 * float(want.abs().max())


def test_qwen3_backbone_oracle_matches_reference_torch_model(reference):
    """The reference's own backbone parity test (``tests/test_qwen3_arch.py:30-60``) holds the MLX
    backbone to ``RefQwen3Backbone`` within 2e-3 on its shapes and weight scale; the oracle's
    backbone is held to the same torch model in fp32, within 1e-5 relative."""
    import sys
    import types

    import numpy as np
    import torch

    import oracle

    shim_mods = {k: sys.modules.pop(k) for k in list(sys.modules) if k == "mlx" or k.startswith("mlx.")}
    try:
        ref = _load_test_module(os.path.join(REF, "tests", "qwen3_ref.py"))
    finally:
        sys.modules.update(shim_mods)
    args = types.SimpleNamespace(hidden_size=32, num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                                 intermediate_size=24, num_hidden_layers=2, rms_norm_eps=1e-6, fc_in=64)
    rng = np.random.default_rng(0)
    bb = ref.RefQwen3Backbone(args)
    weights = {k: torch.tensor((rng.standard_normal(tuple(v.shape)) * 0.05).astype(np.float32))
               for k, v in bb.state_dict().items()}
    for k in weights:
        if k.endswith("norm.weight"):
            weights[k] = weights[k] + 1
    bb.load_state_dict(weights)
    b, ctx, block = 1, 5, 3
    noise = torch.tensor((rng.standard_normal((b, block, 32)) * 0.3).astype(np.float32))
    target_hidden = torch.tensor((rng.standard_normal((b, ctx, 64)) * 0.3).astype(np.float32))
    cos, sin = oracle.qwen3_rope_tables(torch.arange(ctx + block), 16, 1_000_000.0)
    with torch.no_grad():
        tctx_ref = bb.project_context(target_hidden)
        want = bb(noise, tctx_ref, cos, sin)
    tctx = oracle.qwen3_project_context(weights, 1e-6, target_hidden)
    assert float((tctx - tctx_ref).abs().max()) <= 1e-5 * float(tctx_ref.abs().max())
    got = oracle.qwen3_backbone(weights, 2, 4, 2, 16, 1e-6, noise, tctx, cos, sin)
    assert float((got - want).abs().max()) <= 1e-5 * float(want.abs().max())


def _load_with_ref_tests(name):
    """A reference test module whose helpers (``cpu_kernels``, ``torch_ref_heads``,
    ``reference_model``) sit beside it in the reference's tests folder."""
    import sys

    ref_tests = os.path.join(REF, "tests")
    if ref_tests not in sys.path:
        sys.path.insert(0, ref_tests)
    return _load_test_module(os.path.join(ref_tests, name))


def test_reference_kernel_parity_tests(reference):
    """The reference's own kernel parity tests (``tests/test_kernels_parity.py``): its
    ``sparse_attn`` and ``hc_split_sinkhorn`` against its torch CPU kernels, run on the stand-in
    that generated the attention and hyper-connection golden vectors."""
    mod = _load_with_ref_tests("test_kernels_parity.py")
    mod.test_sparse_attn_matches_reference()
    mod.test_sparse_attn_equals_dense_when_full_and_no_sink()
    mod.test_hc_sinkhorn_matches_reference()
    mod.test_hc_sinkhorn_columns_normalized()


def test_reference_head_parity_tests(reference):
    """``tests/test_heads_parity.py``: the Markov and confidence heads against the reference's
    torch heads, on the stand-in that generated the draft-head golden vectors."""
    mod = _load_with_ref_tests("test_heads_parity.py")
    mod.test_markov_head_parity()
    mod.test_confidence_head_parity()
    mod.test_config_from_dict_parses_dspark_fields()


def test_reference_rope_roundtrip_test(reference):
    """``tests/test_layers_parity.py``'s RoPE inverse round trip (its other cases need the
    DeepSeek torch model, which is not in the reference tree)."""
    mod = _load_with_ref_tests("test_layers_parity.py")
    mod.test_rope_inverse_roundtrips()


def test_reference_qwen3_backbone_parity_test(reference):
    """The reference's own Qwen3 backbone parity test (``tests/test_qwen3_arch.py:30-60``): its
    MLX backbone against the torch transcription of DeepSpec's model within 2e-3, run on the
    stand-in that generated the Qwen3 attention, layer and backbone golden vectors."""
    import sys
    import types

    if "dspark_mlx.arch" not in sys.modules:
        arch = types.ModuleType("dspark_mlx.arch")
        arch.__path__ = [os.path.join(REF, "dspark_mlx", "arch")]
        sys.modules["dspark_mlx.arch"] = arch
    # transformers probes for an installed mlx when its Qwen3 module loads: hide the stand-in
    shim_mods = {k: sys.modules.pop(k) for k in list(sys.modules) if k == "mlx" or k.startswith("mlx.")}
    try:
        import transformers.models.qwen3.modeling_qwen3  # noqa: F401
    finally:
        sys.modules.update(shim_mods)
    mod = _load_with_ref_tests("test_qwen3_arch.py")
    mod.test_qwen3_backbone_parity()
