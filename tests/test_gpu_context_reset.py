"""The library's per-device state across a cudaDeviceReset, in a child process that drives the C ABI through ctypes
and the CUDA runtime alone (no torch CUDA context): block.lut through the workspace entry point and through the
static-scratch one, before and after the reset. The reset makes a new context, which loads the module again with
fresh device globals (the LUT format tables, the static scratch), so both must be set up again: the results after the
reset are bit for bit those before it and the oracle's."""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from _util import assert_bits

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent(r"""
    import ctypes, sys
    import numpy as np
    sys.path.insert(0, sys.argv[1])
    from mxq import _lib
    L = ctypes.CDLL(_lib.LIB_PATH)
    for name in ("mxq_block_lut_quantize", "mxq_block_lut_quantize_static"):
        getattr(L, name).argtypes = _lib._SIGS[name]
    L.mxq_block_lut_workspace.restype = ctypes.c_int64
    L.mxq_block_lut_workspace.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32]
    rt = ctypes.CDLL("libcudart.so.12")
    V = np.load(sys.argv[2])
    rows, cols = V.shape
    spec = _lib.MxqQuantSpec(2, 3, 2, 1, float(np.float32(2.0 ** -23)), 0, 0.0, 0, 0)

    def dev(nbytes):
        p = ctypes.c_void_p()
        assert rt.cudaMalloc(ctypes.byref(p), ctypes.c_size_t(nbytes)) == 0
        return p

    def once(static):
        nb = (rows + 31) // 32
        dV, dP, dX, dS = dev(V.nbytes), dev(V.nbytes), dev(nb * cols * 4), dev(4)
        assert rt.cudaMemcpy(dV, V.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(V.nbytes), 1) == 0
        if static:
            rc = L.mxq_block_lut_quantize_static(dV, dP, dX, rows, cols, 0, 32, ctypes.byref(spec), 1, 50, dS, None)
        else:
            need = L.mxq_block_lut_workspace(rows, cols, 0, 1)
            ws = dev(need)
            rc = L.mxq_block_lut_quantize(dV, dP, dX, rows, cols, 0, 32, ctypes.byref(spec), 1, 50, ws, need, dS,
                                          None)
        assert rc == 0, rc
        assert rt.cudaDeviceSynchronize() == 0
        P = np.empty_like(V)
        X = np.empty((nb, cols), np.float32)
        st = np.zeros(1, np.int32)
        for h, d in ((P, dP), (X, dX), (st, dS)):
            assert rt.cudaMemcpy(h.ctypes.data_as(ctypes.c_void_p), d, ctypes.c_size_t(h.nbytes), 2) == 0
        assert st[0] == 0, st[0]
        return P, X

    out = {}
    for phase in ("before", "after"):
        for static in (False, True):
            out[f"{phase}_{int(static)}_P"], out[f"{phase}_{int(static)}_X"] = once(static)
        if phase == "before":
            assert rt.cudaDeviceReset() == 0
    np.savez(sys.argv[3], **out)
""")


@pytest.mark.parametrize("rows", [256, 250])
def test_block_lut_across_device_reset(oracle, tmp_path, rows):
    """256 rows: the one-launch kernel; 250: the TMA quantizer writing code bytes (its wait-status word is made
    again after the reset) and the tables kernel reading them."""
    rng = np.random.default_rng(21)
    V = (rng.standard_normal((rows, 192)) * 2.0 ** rng.uniform(-8, 8, (1, 192))).astype(np.float32)
    np.save(tmp_path / "V.npy", V)
    res = subprocess.run([sys.executable, "-c", CHILD, os.path.join(ROOT, "microscaling-quant_b200"),
                          str(tmp_path / "V.npy"), str(tmp_path / "out.npz")], capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    got = np.load(tmp_path / "out.npz")
    Po, Xo = oracle.lut_block_quantize(V, "MXFP6_E3M2", 0, 32, "rne", 2.0 ** -23, 1, 50)
    for phase in ("before", "after"):
        for static in (0, 1):
            assert_bits(got[f"{phase}_{static}_P"], Po, f"P {phase} the reset, static {static}")
            assert_bits(got[f"{phase}_{static}_X"], Xo, f"X {phase} the reset, static {static}")
