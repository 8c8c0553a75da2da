import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "dspark-mlx_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(params=[1, 0], ids=["cuda_core_attn", "tensor_core_attn"])
def attn_kernel(request):
    """Runs a test once per attention kernel family: 1 the CUDA-core kernels, 0 the tensor-core
    (mma.m16n8k16) kernels wherever they apply (bf16). The switch is per host thread; it is put
    back to the library default afterwards."""
    from dsm import _lib

    L = _lib.lib()
    _lib.check(L.dsm_set_attn_kernel(request.param))
    try:
        yield request.param
    finally:
        _lib.check(L.dsm_set_attn_kernel(_lib.ATTN_KERNEL_DEFAULT))
