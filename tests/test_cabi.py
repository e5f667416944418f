"""The C-ABI library loads (no GPU needed) and exports every entry point that
include/grinqh_b200.h declares; host-only calls behave. No compute calls here."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "grinqh_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(grinqh_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from grinqh import _ext
    lib = ctypes.CDLL(_ext.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding table covers the header exactly
    assert set(names) == set(_ext.SIGNATURES)


def test_status_strings_and_version():
    from grinqh import _ext
    lib = _ext.cabi()
    assert lib.grinqh_abi_version() == 1
    assert lib.grinqh_status_string(0) == b"ok"
    assert lib.grinqh_status_string(4) == b"workspace too small"
    assert lib.grinqh_status_string(99) == b"unknown status"


def test_workspace_size_is_host_only():
    from grinqh import _ext
    lib = _ext.cabi()
    # K split over several CTAs -> fp32 partials + tickets
    ws = lib.grinqh_workspace_size(1, 4096, 4096, 8, 128, _ext.MODE_AUTO)
    assert ws >= 4096 * 4 * 2
    assert lib.grinqh_workspace_size(0, 4096, 4096, 8, 128, _ext.MODE_AUTO) == 0
    assert lib.grinqh_workspace_size(1, 4096, 4096, 8, 128, 17) == 0  # unknown mode


def test_calls_without_gpu_fail_loudly():
    """On a host without a usable sm_100 device every compute entry point returns
    an error status (never silently succeeds)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    from grinqh import _ext
    lib = _ext.cabi()
    st = lib.grinqh_pack_words(None, None, 4, 16, 8, None)
    assert st != 0
    assert lib.grinqh_last_error()


def test_torch_ops_registered():
    import torch
    import grinqh.kernel  # noqa: F401
    for name in ("gemm_or_gemv", "linear", "pack", "pack_codes", "unpack", "grade", "rmsnorm_grade",
                 "silu_mul_grade", "union_linear_masked", "linear_allreduce", "gemv_allreduce"):
        assert hasattr(torch.ops.grinqh, name)
    schema = str(torch.ops.grinqh.gemm_or_gemv.default._schema)
    assert "float[] thresholds" in schema and "bool use_marlin=False" in schema


def test_ops_refuse_cpu_tensors():
    import torch
    import grinqh.kernel as K
    x = torch.randn(1, 256, dtype=torch.bfloat16)
    w = torch.zeros(256, 64, dtype=torch.int32)
    s = torch.ones(2, 256, dtype=torch.bfloat16)
    # no CPU kernel is registered: the dispatcher refuses CPU tensors
    with pytest.raises((RuntimeError, NotImplementedError), match="CPU"):
        K.grinqh_gemm_or_gemv(x, w, s, None, 8, 128, 64, [0.0] * 4)


def test_fake_impl_shapes():
    import torch
    import grinqh.kernel  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(3, 5, 256, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(256, 4 * 320 // 16, dtype=torch.int32, device="cuda")
        s = torch.empty(2, 320, dtype=torch.bfloat16, device="cuda")
        y = torch.ops.grinqh.gemm_or_gemv(x, w, s, None, 8, 128, 80, [0.1, 0.2, 0.3, 0.4])
        assert tuple(y.shape) == (3, 5, 320) and y.dtype == torch.bfloat16
        o, m, u = torch.ops.grinqh.rmsnorm_grade(x, None, None, 1e-5, [0.1] * 4, 8)
        assert tuple(o.shape) == (3, 5, 256) and tuple(m.shape) == (3, 5, 256) and tuple(u.shape) == (256,)
        o, m, u = torch.ops.grinqh.silu_mul_grade(x, [0.1] * 4, 8)
        assert tuple(o.shape) == (3, 5, 128) and m.dtype == torch.uint8 and tuple(u.shape) == (128,)
        y = torch.ops.grinqh.union_linear_masked(x, w, s, None, 8, 128, 80, [0.1] * 4, u)
        assert tuple(y.shape) == (3, 5, 320)
