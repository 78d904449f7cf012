"""CPU: the C-ABI library loads, exports every symbol include/detkernels_b200.h
declares, and rejects bad arguments on the host without touching a GPU."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "detkernels_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dk_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from detkernels_b200 import _lib
    from detkernels_b200 import build as b
    if not os.path.exists(_lib.library_path()):
        b.build()
    return _lib.load()


def test_header_declares_the_expected_entry_points():
    syms = declared_symbols()
    for name in ("dk_rmsnorm_batch_invariant", "dk_rmsnorm_batch_variant", "dk_matmul_batch_invariant",
                 "dk_matmul_batch_variant", "dk_matmul_slice_partials", "dk_matmul_fold_slices",
                 "dk_attention_batch_invariant", "dk_attention_batch_variant", "dk_device_status"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(os.path.join(ROOT, "detkernels_b200", "libdetkernels_b200.so"))
    for name in declared_symbols():
        assert hasattr(raw, name), name


def test_python_binding_covers_the_header():
    from detkernels_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_host_side_validation_without_a_gpu(lib):
    from detkernels_b200 import _lib
    assert lib.dk_abi_version() == _lib.ABI_VERSION == 3
    # unsupported dtype code
    rc = lib.dk_rmsnorm_batch_invariant(None, 0, None, None, 0, 4, 8, 7, 0, 1e-6, None)
    assert rc == _lib.DK_ERR_UNSUPPORTED
    # matmul: f32 is not a tensor-core input here
    rc = lib.dk_matmul_batch_invariant(None, 8, None, 8, None, 8, 2, 8, 8, _lib.DK_F32, None, 0, None)
    assert rc == _lib.DK_ERR_UNSUPPORTED
    assert "bf16 or f16" in _lib.last_error()
    # attention: head_dim outside the built set
    rc = lib.dk_attention_batch_invariant(None, 0, 0, None, None, 0, 0, 0, 1, 1, None, 0, 0, None, 1, None, 0, 1,
                                          4, 4, 96, 1, 0.1, _lib.DK_BF16, None, 0, None)
    assert rc == _lib.DK_ERR_UNSUPPORTED
    # empty calls are no-ops
    assert lib.dk_rmsnorm_batch_invariant(None, 0, None, None, 0, 0, 8, 0, 0, 1e-6, None) == 0


def test_workspace_sizes_follow_the_layout(lib):
    counter = 1 << 20
    # single-split decode needs no scratch; multi-split needs the counter area + partials
    assert lib.dk_attention_workspace_size(4, 1, 8, 8, 64, 256) == 0
    n = lib.dk_attention_workspace_size(4, 1, 32, 8, 128, 1000)
    assert n >= counter + 4 * 8 * 4 * 4 * 128 * 4
    assert lib.dk_rmsnorm_variant_workspace_size(10) >= counter + 40
    assert lib.dk_matmul_variant_workspace_size(3, 5) >= counter + 60


def test_product_package_never_imports_the_oracle():
    pkg = os.path.join(ROOT, "detkernels_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                assert not re.search(r"^\s*(from|import)\s+oracle\b", src, flags=re.M), f


def test_ops_refuse_cpu_tensors():
    import torch

    from detkernels_b200.kernels.attention import attention_batch_invariant
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant
    with pytest.raises(AssertionError):
        rmsnorm_batch_invariant(torch.randn(2, 8), torch.randn(8))
    with pytest.raises(AssertionError):
        matmul_batch_invariant(torch.randn(2, 8), torch.randn(8, 4))
    with pytest.raises(AssertionError):
        attention_batch_invariant(torch.randn(1, 2, 8), torch.randn(1, 2, 4, 8), torch.randn(1, 2, 4, 8))
