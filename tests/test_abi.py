"""CPU tests of the C ABI: the library loads, exports every symbol that
include/*.h declares, and rejects bad arguments with the documented codes
before touching a device (the mlx-c int-return + error-text convention)."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names |= set(re.findall(r"^VMLX_API\s+[\w\s\*]+?\b(vmlx_\w+)\s*\(", text, flags=re.M))
    return sorted(names)


def test_header_declares_symbols():
    syms = declared_symbols()
    assert "vmlx_cuda_quantized_matmul" in syms and "vmlx_cuda_gather_qmm" in syms


def test_library_exports_every_declared_symbol(vm):
    lib = ctypes.CDLL(vm._lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_python_signatures_cover_header(vm):
    assert set(declared_symbols()) <= set(vm._lib.SIGNATURES)


def test_version(vm):
    assert vm.lib().vmlx_version() >= 100


def _qmm(vm, **kw):
    args = dict(y=1 << 12, x=1 << 12, w=1 << 12, s=1 << 12, b=1 << 12, transpose=True, gs=64, bits=4,
                mode=b"affine", M=1, N=16, K=64)
    args.update(kw)
    return vm.lib().vmlx_cuda_quantized_matmul(args["y"], args["x"], args["w"], args["s"], args["b"],
                                               args["transpose"], args["gs"], args["bits"], args["mode"],
                                               args["M"], args["N"], args["K"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(mode=b"mxfp4"), 2),
    (dict(transpose=False), 2),
    (dict(bits=3), 2),
    (dict(gs=16), 2),
    (dict(K=100), 1),
    (dict(b=None), 1),
    (dict(x=None), 1),
    (dict(x=(1 << 12) + 2), 1),   # misaligned x
])
def test_matmul_rejects_bad_arguments(vm, kw, code):
    rc = _qmm(vm, **kw)
    assert rc == code
    assert vm.lib().vmlx_last_error()


def test_quantize_rejects_bad_arguments(vm):
    lib = vm.lib()
    assert lib.vmlx_cuda_quantize(1, 1, 1, 1, 0, 4, 100, 64, 4, b"affine", None) == 1
    assert lib.vmlx_cuda_quantize(1, 1, 1, 1, 0, 4, 128, 64, 5, b"affine", None) == 2
    assert lib.vmlx_cuda_quantize(1, 1, 1, 1, 0, 4, 128, 64, 4, b"nvfp4", None) == 2
    assert b"nvfp4" in lib.vmlx_last_error()


def test_gather_rejects_bad_arguments(vm):
    lib = vm.lib()
    base = [1 << 12] * 5
    # no rhs indices
    rc = lib.vmlx_cuda_gather_qmm(*base, None, None, True, 64, 4, b"affine", False, 4, 1, 1, 16, 64, 8, None)
    assert rc == 1
    # batch not a multiple of x_batches without lhs indices
    rc = lib.vmlx_cuda_gather_qmm(*base, None, 1 << 12, True, 64, 4, b"affine", False, 5, 2, 1, 16, 64, 8, None)
    assert rc == 1


def test_python_layer_api_shapes(vm):
    """QuantizedLinear.shape / describe_extra (Quantized.swift:272-275,
    QuantizationTests.swift:9-21) from tensor shapes alone (no device work)."""
    import torch
    ql = vm.QuantizedLinear(torch.zeros(1024, 512 * 4 // 32, dtype=torch.int32), torch.zeros(1024),
                            torch.zeros(1024, 8), torch.zeros(1024, 8), 64, 4)
    assert ql.shape == (1024, 512)
    assert ql.describe_extra() == "(inputDimensions=512, outputDimensions=1024, bias=true)"
    ql2 = vm.QuantizedLinear(torch.zeros(512, 1024 * 8 // 32, dtype=torch.int32), None,
                             torch.zeros(512, 8), torch.zeros(512, 8), 128, 8)
    assert ql2.describe_extra() == "(inputDimensions=1024, outputDimensions=512, bias=false)"


def test_consecutive_broadcast_rule(vm):
    f = vm.ops._consecutive_broadcast
    assert f((4, 1), (4, 8))
    assert f((32,), (32,))
    assert f((), (4, 8))
    assert f((1,), (6,))
    assert not f((8,), (4, 8))
    assert not f((1, 8), (4, 8))


def test_launch_overlap_setter_returns_previous(vm):
    lib = vm.lib()
    prev = lib.vmlx_set_launch_overlap(1)
    assert lib.vmlx_set_launch_overlap(0) == 1
    assert lib.vmlx_set_launch_overlap(prev) == 0
