"""The C-ABI library loads, exports every entry point ``include/dsm.h`` declares, and
answers size queries / rejects bad arguments on the host (no GPU work)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from dsm import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dsm.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dsm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    assert "dsm_moe_forward" in names and "dsm_router" in names
    assert set(names) == set(_lib.EXPORTED), set(names) ^ set(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for name in _declared():
        assert hasattr(raw, name), f"{name} not exported"


def test_abi_version_and_status_strings():
    L = _lib.lib()
    assert L.dsm_abi_version() == 1
    assert L.dsm_status_string(0) == b"ok"
    assert L.dsm_status_string(1) == b"invalid argument"


def test_size_queries():
    L = _lib.lib()
    # fp8 tile: 16 KB codes + 16 B scale; 256 B header for <= 64 experts
    assert L.dsm_packed_bytes(_lib.WFMT_FP8_B128, 2, 128, 256, 128) == 256 + 2 * 2 * (16384 + 16)
    assert L.dsm_packed_bytes(_lib.WFMT_FP4_G32, 1, 128, 128, 32) == 256 + 8192 + 512
    assert L.dsm_packed_bytes(_lib.WFMT_F16, 1, 100, 100, 0) == 256 + 32768  # padded to one tile
    assert L.dsm_packed_bytes(_lib.WFMT_AFFINE8, 1, 128, 128, 64) == 256 + 16384 + 1024
    assert L.dsm_packed_bytes(99, 1, 128, 128, 64) == 0
    cap = L.dsm_stage_rows_cap(336)
    assert cap >= 336 + 32 and cap % 8 == 0
    assert L.dsm_stage_bytes(cap, 4096) == 32 * cap * 160 * 2
    assert L.dsm_permute_workspace_bytes(131072, 256) == 128 * 256 * 4
    # dense MLP: staged x and h plus up to 8 fp32 partial slabs of the down product
    assert L.dsm_dense_mlp_workspace_bytes(112, 2560, 9728) >= 8 * 112 * 2560 * 4
    assert L.dsm_dense_mlp_workspace_bytes(0, 2560, 9728) == 0
    d = _lib.MoEDesc(n_tokens=56, dim=4096, inter=2048, n_experts=256, topk=6)
    d.s1 = 1
    assert L.dsm_moe_workspace_bytes(ctypes.byref(d)) > 56 * 6 * 4096 * 4


@pytest.mark.parametrize("call", ["router", "permute", "combine", "quantize", "dense_mlp"])
def test_bad_arguments_are_rejected_on_the_host(call):
    L = _lib.lib()
    if call == "router":
        rc = L.dsm_router(None, _lib.DT_BF16, 4, 0, None, 8, None, None, 0, None, _lib.DT_I32, 0, 2, 1, 1.0,
                          None, None, None, None)
    elif call == "permute":
        rc = L.dsm_permute(None, 10, 0, None, None, None, None, None, 0, None)
    elif call == "combine":
        rc = L.dsm_combine(None, None, None, 4, 0, 16, None, None, _lib.DT_BF16, None)
    elif call == "quantize":
        rc = L.dsm_affine_quantize(None, _lib.DT_BF16, 4, 100, 64, 8, None, None, None, None)
    else:  # dim not a multiple of 4
        rc = L.dsm_dense_mlp(None, _lib.DT_BF16, 4, 6, 128, _lib.WFMT_AFFINE8, 64, None, None, None, 1, 0.0, 3, 1,
                             None, _lib.DT_BF16, None, 0, None)
    assert rc == 1
    assert L.dsm_last_error_message().decode()


def test_attention_entry_points_reject_bad_arguments_on_the_host():
    L = _lib.lib()
    bf = _lib.DT_BF16
    cases = [
        # n_heads not a multiple of n_groups
        lambda: L.dsm_sparse_attn(1, 1, 1, bf, 1, 2, 5, 6, 64, 8, 4, 0.1, 16, 1, 1, 0, 4, 1, 1, None),
        # n_win beyond the window
        lambda: L.dsm_sparse_attn(1, 1, 1, bf, 1, 2, 5, 8, 64, 8, 9, 0.1, 16, 1, 1, 0, 4, 1, 1, None),
        # more rows than window slots in one write
        lambda: L.dsm_kv_window_write(1, bf, 2, 9, 64, 0, 8, 1, None),
        # odd rope width
        lambda: L.dsm_rows_norm_rope(1, None, 4, 64, None, 1e-6, 15, 1, 1, 0, 4, 1, bf, None),
        # odd head_dim
        lambda: L.dsm_q_head_norm_rope(1, None, 4, 2, 63, 1e-6, 0, None, None, 0, 1, 1, bf, None),
        # NULL staging buffers
        lambda: L.dsm_stage_rows_hilo(None, 4, 64, None, 1 << 10, None, None),
        lambda: L.dsm_round_rows(1, None, 8, 1, _lib.DT_I32, None),
    ]
    for i, call in enumerate(cases):
        assert call() != 0, i
        assert L.dsm_last_error_message().decode()
    assert L.dsm_sparse_attn_scratch_bytes(8, 7, 64, 128) == 8 * 7 * 64 * 135 * 4


def test_gqa_attention_entry_points_reject_bad_arguments_on_the_host():
    L = _lib.lib()
    bf = _lib.DT_BF16
    cases = [
        # odd head_dim
        lambda: L.dsm_qkv_norm_rope(1, None, 14, 4, 2, 63, 1, 1, 1e-6, 1, 1, 100, 0, 7, 1, 1, 1, 7, 0, bf, None),
        # rows that are not whole sequences of period rows
        lambda: L.dsm_qkv_norm_rope(1, None, 13, 4, 2, 64, 1, 1, 1e-6, 1, 1, 100, 0, 7, 1, 1, 1, 7, 0, bf, None),
        # RoPE table rows out of range
        lambda: L.dsm_qkv_norm_rope(1, None, 14, 4, 2, 64, 1, 1, 1e-6, 1, 1, 10, 5, 7, 1, 1, 1, 7, 0, bf, None),
        # cache rows out of range
        lambda: L.dsm_qkv_norm_rope(1, None, 14, 4, 2, 64, 1, 1, 1e-6, 1, 1, 100, 0, 7, 1, 1, 1, 7, 1, bf, None),
        # query heads without a q output
        lambda: L.dsm_qkv_norm_rope(1, None, 14, 4, 2, 64, 1, 1, 1e-6, 1, 1, 100, 0, 7, None, 1, 1, 7, 0, bf, None),
        # n_heads not a multiple of n_kv
        lambda: L.dsm_gqa_attn(1, 1, 1, 0, 0, 16, 1, 1, bf, 1, 7, 6, 4, 64, 0.1, 1, 1, 1 << 30, None),
        # unsupported head_dim
        lambda: L.dsm_gqa_attn(1, 1, 1, 0, 0, 16, 1, 1, bf, 1, 7, 8, 4, 96, 0.1, 1, 1, 1 << 30, None),
        # context rows without context pointers
        lambda: L.dsm_gqa_attn(1, None, None, 0, 0, 16, 1, 1, bf, 1, 7, 8, 4, 64, 0.1, 1, 1, 1 << 30, None),
        # workspace too small
        lambda: L.dsm_gqa_attn(1, 1, 1, 0, 0, 16, 1, 1, bf, 1, 7, 8, 4, 64, 0.1, 1, 1, 16, None),
    ]
    for i, call in enumerate(cases):
        assert call() != 0, i
        assert L.dsm_last_error_message().decode()
    # 32 query heads over 8 KV heads, a block of 7 after 2048 context rows: 33 key ranges of
    # one 64-key tile each (two CTAs per SM on 148 SMs), room for two fp32 partials of
    # 128 + 2 per row and range
    assert L.dsm_gqa_attn_workspace_bytes(1, 7, 32, 8, 128, 2048) == 32 * 7 * 66 * 130 * 4
    assert L.dsm_gqa_attn_workspace_bytes(1, 7, 32, 8, 128, 0) == 32 * 7 * 2 * 130 * 4
    assert L.dsm_set_attn_kernel(2) != 0 and L.dsm_set_attn_kernel(1) == 0
    assert L.dsm_set_attn_kernel(_lib.ATTN_KERNEL_DEFAULT) == 0
    # split-K linear: up to 8 fp32 partial slabs; bad format, group size and shapes rejected
    assert L.dsm_linear_splitk_workspace_bytes(112, 1024) == 8 * 112 * 1024 * 4
    assert L.dsm_linear_splitk(1, 1, 1 << 10, 2560, 9, 64, 1, 1024, 1, 1024, 112, 1, 1 << 30, None) != 0
    assert L.dsm_linear_splitk(1, 1, 1 << 10, 2560, _lib.WFMT_AFFINE8, 48, 1, 1024, 1, 1024, 112, 1, 1 << 30,
                               None) != 0
    assert L.dsm_linear_splitk(1, 1, 1 << 10, 2560, _lib.WFMT_AFFINE8, 64, 1, 1024, 1, 512, 112, 1, 1 << 30,
                               None) != 0  # ldo < out_dim
    # residual add + RMSNorm: nothing to write, a norm without weights, an unsupported dtype
    assert L.dsm_add_rms_norm(1, 1, bf, 4, 64, None, 1e-6, None, None, None) != 0
    assert L.dsm_add_rms_norm(1, 1, bf, 4, 64, None, 1e-6, None, 1, None) != 0
    assert L.dsm_add_rms_norm(1, 1, _lib.DT_I32, 4, 64, 1, 1e-6, 1, 1, None) != 0
    assert L.dsm_gqa_attn_workspace_bytes(1, 7, 6, 4, 128, 0) == 0


def test_draft_head_host_checks():
    L = _lib.lib()
    d = _lib.HeadDesc(batch=8, block=7, hc_mult=4, dim=4096, vocab=129280, rank=256)
    need = L.dsm_draft_head_workspace_bytes(ctypes.byref(d), _lib.DT_BF16)
    assert need >= 56 * 129280 * 4  # the fp32 base logits
    assert L.dsm_draft_head_workspace_bytes(ctypes.byref(d), _lib.DT_F32) >= 2 * 56 * 129280 * 4  # hi + lo rows
    bad = _lib.HeadDesc(batch=8, block=7, hc_mult=4, dim=64, vocab=100, rank=12)  # rank not a multiple of 8
    rc = L.dsm_draft_head(ctypes.byref(bad), 1, _lib.DT_BF16, 1, _lib.DT_I32, 0.0, None, 1, 1, None, None, 1, 1 << 30,
                          None)
    assert rc != 0 and L.dsm_last_error_message().decode()
    assert ctypes.sizeof(_lib.HeadDesc) % 8 == 0 and _lib.HeadDesc.hc_fn.offset % 8 == 0


def test_desc_struct_layout_matches_header():
    # field offsets of the ctypes mirror must follow the C struct (8-byte pointers, int64 first)
    assert _lib.MoEDesc.n_tokens.offset == 0
    assert _lib.MoEDesc.gate_weight.offset % 8 == 0
    assert ctypes.sizeof(_lib.MoEDesc) % 8 == 0
    names = [f for f, _ in _lib.MoEDesc._fields_]
    text = open(HEADER).read()
    body = text[text.index("typedef struct dsm_moe_desc"):text.index("} dsm_moe_desc;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    c_fields = re.findall(r"\*?\s*([a-z_0-9]+)\s*[,;]", body)
    assert c_fields == names


def test_grouped_linear_rejects_bad_arguments_on_the_host():
    L = _lib.lib()
    # no offsets for several groups, ldo below out_dim, unknown format
    assert L.dsm_grouped_linear(1, 1, 1 << 10, 512, _lib.WFMT_F16, 0, 1, 4, None, 256, 1, 256, None, 224, None) != 0
    assert L.dsm_grouped_linear(1, 1, 1 << 10, 512, _lib.WFMT_F16, 0, 1, 4, 1, 256, 1, 128, None, 224, None) != 0
    assert L.dsm_grouped_linear(1, 1, 1 << 10, 512, 9, 0, 1, 4, 1, 256, 1, 256, None, 224, None) != 0
    assert L.dsm_last_error_message().decode()


def test_split_linear_entry_points_reject_bad_arguments_on_the_host():
    """The K-split products check their shapes and pointers before touching the GPU."""
    L = _lib.lib()
    f16 = _lib.WFMT_F16
    cases = [
        # ldo below out_dim
        lambda: L.dsm_grouped_linear_splitk(1, 1, 128, 512, f16, 0, 1, 4, 1, 256, 1, 128, None, 56, None, 0, None),
        # no offsets for the groups
        lambda: L.dsm_grouped_linear_splitk(1, 1, 128, 512, f16, 0, 1, 4, None, 256, 1, 256, None, 56, None, 0,
                                            None),
        # NULL weights
        lambda: L.dsm_grouped_linear_splitk(1, 1, 128, 512, f16, 0, None, 4, 1, 256, 1, 256, None, 56, None, 0,
                                            None),
        # too many groups
        lambda: L.dsm_grouped_linear_splitk(1, 1, 128, 512, f16, 0, 1, 5000, 1, 256, 1, 256, None, 56, None, 0,
                                            None),
        # ldo below out_dim
        lambda: L.dsm_linear_splitk(1, 1, 128, 512, f16, 0, 1, 256, 1, 128, 56, None, 0, None),
    ]
    for i, call in enumerate(cases):
        assert call() != 0, i
        assert L.dsm_last_error_message().decode()
    assert L.dsm_linear_splitk_workspace_bytes(56, 4096) == 8 * 56 * 4096 * 4
