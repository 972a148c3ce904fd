"""The C ABI without a GPU: libmxq_b200.so loads and exports every entry point include/*.h declares, and the
status convention maps to the reference's exceptions."""
import ctypes
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names |= set(re.findall(r"^\s*(?:const\s+char\s*\*|int64_t|int|void)\s+(mxq_\w+)\s*\(", src, re.M))
    return names


def test_library_exports_every_declared_symbol():
    from mxq import _lib
    L = _lib.lib()
    names = declared()
    assert len(names) >= 40
    missing = [n for n in sorted(names) if not hasattr(L, n)]
    assert not missing, missing
    assert set(_lib._SIGS) <= names


def test_version_and_errors():
    from mxq import _lib
    L = _lib.lib()
    assert L.mxq_version().decode().startswith("mxq_b200")
    # an argument error is reported before anything touches a device
    rc = L.mxq_round_bits(None, None, 30, None, 1, 1, None)
    assert rc == _lib.ERR_VALUE and b"keep must be in [0, 22]" in L.mxq_last_error()
    spec = _lib.MxqQuantSpec(2, 4, 4, 0, 0.0, 0, 0.0, 0, 0)          # (4, 4) is no OCP element format
    rc = L.mxq_block_quantize(None, None, None, 1, 32, 1, 32, ctypes.byref(spec), None)
    assert rc == _lib.ERR_VALUE
    arith = _lib.MxqArith(1, 4, 3, 1, 2.0 ** -16, 448.0, 448.0)
    e = (ctypes.c_int32 * 16)(*([4] * 16))
    m = (ctypes.c_int32 * 16)(*([4] * 16))
    rc = L.mxq_systolic(None, None, None, None, None, 32, 1, 1, 32, 12, ctypes.byref(arith), e, m, None)
    assert rc == _lib.ERR_VALUE and b"must divide block size" in L.mxq_last_error()


def test_empty_block_shapes_refused_like_torch_reshape():
    """The reference blocks V with reshape(*rest, -1, block); torch refuses an empty V whose other dimensions hold a
    zero, before any device work -- and so does this package."""
    import pytest
    import torch
    from mxq import block
    for shape, axis in (((0, 64), 1), ((64, 0), 0), ((0, 0), 0)):
        for q in (block.mxquant.quantize, block.mxgemmini.quantize, block.ocp.quantize):
            with pytest.raises(RuntimeError, match="cannot reshape tensor of 0 elements"):
                q(torch.zeros(shape), "MXFP8_E4M3", axis=axis)
