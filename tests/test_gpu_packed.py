"""The compact operand form on the GPU: block.mxgemmini / block.ocp quantize_packed against the float32 path --
unpack gives back exactly quantize's (P, X), every byte is the OCP bit pattern of its code (checked with an encoder
built here from each format's value table), dequantize_packed equals dequantize -- and values the form cannot hold
(Inf in E4M3, NaN in FP6, the non-power-of-two scale floor of an all-zero block) raise."""
import numpy as np
import pytest
import torch

from _util import assert_bits

pytestmark = pytest.mark.gpu

FMTS = {"MXFP8_E4M3": (4, 3), "MXFP8_E5M2": (5, 2), "MXFP6_E3M2": (3, 2), "MXFP6_E2M3": (2, 3), "MXFP4": (2, 1)}


def ocp_encoder(e, m):
    """float32 bit pattern -> lowest OCP code having that value (E4M3: S.1111.111 NaN; E5M2: exponent 31 Inf/NaN)."""
    bias = (1 << (e - 1)) - 1
    table = {}
    for c in range(1 << (1 + e + m)):
        s, ex, man = c >> (e + m), (c >> m) & ((1 << e) - 1), c & ((1 << m) - 1)
        if (e, m) == (4, 3) and ex == 15 and man == 7:
            continue
        if (e, m) == (5, 2) and ex == 31:
            v = np.inf if man == 0 else None
            if v is None:
                continue
        elif ex == 0:
            v = man * 2.0 ** (1 - bias - m)
        else:
            v = (1 + man / 2 ** m) * 2.0 ** (ex - bias)
        bits = int(np.array([-v if s else v], np.float32).view(np.uint32)[0])
        table.setdefault(bits, c)
    return table


def config2_like(rows, cols, seed):
    rng = np.random.default_rng(seed)
    V = rng.standard_normal((rows, cols)) * 2.0 ** rng.uniform(-20, 20, (rows, 1))
    V[rng.random((rows, cols)) < 0.01] = 0.0
    return V.astype(np.float32)


@pytest.mark.parametrize("family", ["mxgemmini", "ocp"])
@pytest.mark.parametrize("axis", [0, 1])
def test_packed_roundtrip(family, axis):
    from mxq import block
    V = torch.from_numpy(config2_like(256, 320, 3 + axis)).cuda()
    q = getattr(block, family)
    for fmt, (e, m) in FMTS.items():
        kw = {"scale_floor": 2.0 ** -23} if family == "mxgemmini" else {}
        P, X = q.quantize(V, fmt, axis=axis, **kw)
        codes, scales = q.quantize_packed(V, fmt, axis=axis, **kw)
        assert codes.dtype == torch.uint8 and scales.dtype == torch.uint8
        Pu, Xu = block.unpack(codes, scales, fmt)
        assert_bits(Pu.cpu().numpy(), P.cpu().numpy(), f"{family} {fmt} {axis} P")
        assert_bits(Xu.cpu().numpy(), X.cpu().numpy(), f"{family} {fmt} {axis} X")
        # every byte is the code's OCP bit pattern
        enc = ocp_encoder(e, m)
        want = np.vectorize(enc.__getitem__)(P.cpu().numpy().view(np.uint32).astype(np.int64)).astype(np.uint8)
        if e + m == 3:
            want = (want[..., 0::2] | (want[..., 1::2] << 4)).astype(np.uint8)
        assert np.array_equal(codes.cpu().numpy(), want), f"{family} {fmt} {axis} bytes"
        xb = X.cpu().numpy().view(np.uint32)
        want_x = np.where(xb == 0x00400000, 0, xb >> 23).astype(np.uint8)
        assert np.array_equal(scales.cpu().numpy(), want_x), f"{family} {fmt} {axis} scale bytes"
        D = block.dequantize_packed(codes, scales, fmt, axis=axis)
        assert_bits(D.cpu().numpy(), block.dequantize(P, X, axis=axis).cpu().numpy(), f"{family} {fmt} dequantize")


def test_packed_specials():
    from mxq import block
    V = torch.from_numpy(config2_like(64, 64, 9)).cuda()
    inf = V.clone()
    inf[5, 7] = float("inf")                             # the block's scale becomes Inf: no E8M0 byte holds it
    for fmt in ("MXFP8_E4M3", "MXFP8_E5M2"):
        with pytest.raises(ValueError, match="power of two"):
            block.mxgemmini.quantize_packed(inf, fmt, axis=1, scale_floor=2.0 ** -23)
    nan = V.clone()
    nan[3, 3] = float("nan")                             # a NaN scale is 0xFF; a NaN code fits E4M3, not FP6
    with pytest.raises(ValueError, match="cannot hold"):
        block.ocp.quantize_packed(nan, "MXFP6_E3M2", axis=0)
    codes, scales = block.ocp.quantize_packed(nan, "MXFP8_E4M3", axis=0)
    Pu, Xu = block.unpack(codes, scales, "MXFP8_E4M3")
    P, X = block.ocp.quantize(nan, "MXFP8_E4M3", axis=0)
    assert_bits(Pu.cpu().numpy(), P.cpu().numpy(), "E4M3 with NaN: codes")
    assert_bits(Xu.cpu().numpy(), X.cpu().numpy(), "E4M3 with NaN: scales")
    assert int(scales[0, 3]) == 0xFF
    zero = V.clone()
    zero[:32, 0] = 0.0                                   # an all-zero block: the default floor 1e-38 is its scale
    with pytest.raises(ValueError, match="power of two"):
        block.mxgemmini.quantize_packed(zero, "MXFP8_E4M3", axis=0)
    codes, scales = block.mxgemmini.quantize_packed(zero, "MXFP8_E4M3", axis=0, scale_floor=2.0 ** -127)
    assert int(scales[0, 0]) == 0                        # 2^-127
