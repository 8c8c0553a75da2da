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
