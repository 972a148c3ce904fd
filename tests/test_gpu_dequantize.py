"""block.dequantize, block.unpack and block.dequantize_packed on the GPU, on both kernel paths: the float4 kernels
(rows of 4-aligned runs, 16-byte aligned buffers) and the general per-element ones (ragged extents, odd block sizes,
buffers that start off a 16-byte boundary). dequantize is checked against float32 products computed here with
numpy (the host's own multiply: P * each scale repeated block_size times, cut to P's length), with NaN, Inf, zero
and subnormal codes and scales; the compact form's kernels against the float32 path."""
import numpy as np
import pytest
import torch

from _util import assert_bits

pytestmark = pytest.mark.gpu


def specials(rng, shape):
    """float32 values of every class: normals over a wide range, subnormals, zeros of both signs, Inf, NaN."""
    v = (rng.standard_normal(shape) * 2.0 ** rng.integers(-30, 30, shape)).astype(np.float32)
    pick = rng.random(shape)
    v[pick < 0.02] = np.float32(np.inf)
    v[(pick >= 0.02) & (pick < 0.04)] = np.float32(-np.inf)
    v[(pick >= 0.04) & (pick < 0.06)] = np.float32(0.0)
    v[(pick >= 0.06) & (pick < 0.08)] = np.float32(-0.0)
    sub = (pick >= 0.08) & (pick < 0.10)
    v[sub] = (rng.integers(1, 1 << 23, int(sub.sum())).astype(np.uint32)).view(np.float32)
    nan = (pick >= 0.10) & (pick < 0.12)
    v[nan] = (np.uint32(0x7fc00001) | (rng.integers(0, 2, int(nan.sum())).astype(np.uint32) << 31)).view(np.float32)
    return v


def expected(P, X, axis, block):
    L = P.shape[axis]
    with np.errstate(all="ignore"):                      # Inf x 0 and overflow are data here
        return P * np.repeat(X, block, axis=axis).take(np.arange(L), axis=axis)


# (shape, axis, block): the first four take the float4 kernels, the rest the general ones
LAYOUTS = [((64, 96), 0, 32), ((64, 96), 1, 32), ((8, 40, 12), 1, 32), ((5, 44), 1, 4),
           ((8, 40, 6), 1, 16), ((5, 36), 1, 6), ((3, 7, 5), 2, 32), ((6, 34), 1, 32)]


@pytest.mark.parametrize("shape,axis,block", LAYOUTS)
def test_dequantize_layouts(shape, axis, block):
    from mxq import block as blk
    rng = np.random.default_rng(sum(shape) + axis + block)
    P = specials(rng, shape)
    xs = list(shape)
    xs[axis] = -(-shape[axis] // block)
    X = specials(rng, tuple(xs))
    D = blk.dequantize(torch.from_numpy(P).cuda(), torch.from_numpy(X).cuda(), axis=axis, block_size=block)
    assert_bits(D.cpu().numpy(), expected(P, X, axis, block), f"dequantize {shape} axis {axis} block {block}")


def test_dequantize_unaligned_buffers():
    """Buffers that start 4 bytes past a 16-byte boundary go through the general kernel, with the same result."""
    from mxq import block as blk
    rng = np.random.default_rng(11)
    P, X = specials(rng, (64, 96)), specials(rng, (2, 96))
    base = torch.empty(64 * 96 + 1, device="cuda")
    p = base[1:].view(64, 96)
    p.copy_(torch.from_numpy(P))
    assert p.data_ptr() % 16 != 0
    D = blk.dequantize(p, torch.from_numpy(X).cuda(), axis=0)
    assert_bits(D.cpu().numpy(), expected(P, X, 0, 32), "unaligned dequantize")


FMTS = ["MXFP8_E4M3", "MXFP8_E5M2", "MXFP6_E3M2", "MXFP6_E2M3", "MXFP4"]


# (shape of V, axis, padded shape): the compact quantizer needs rows of 4-aligned runs, so a ragged V is quantized
# inside a zero-padded one (zeros change no block's maximum) and its codes and scales are cut out of the result
# ((5, 48), 1): rows of a ragged last block (the scale index by division); the two large ones take the grid-stride
# loops of the float4 kernels more than once round
COMPACT = [((4, 64, 12), 1, None), ((6, 64), 1, None), ((64, 8), 0, None), ((3, 34), 1, (3, 64)),
           ((2, 40, 6), 1, (2, 40, 8)), ((5, 48), 1, None), ((1024, 2048), 1, None), ((1200, 2000), 1, None),
           ((2048, 1024), 0, None)]


@pytest.mark.parametrize("shape,axis,padded", COMPACT)
def test_compact_layouts(shape, axis, padded):
    """unpack gives back quantize's (P, X) and dequantize_packed equals dequantize, on layouts of both kernel paths
    (4-aligned runs; ragged code and scale counts; inner extents that are not a multiple of 4)."""
    from mxq import block as blk
    rng = np.random.default_rng(len(shape) * 7 + axis)
    v = (rng.standard_normal(shape) * 2.0 ** rng.uniform(-8, 8, shape)).astype(np.float32)
    vp = np.zeros(padded or shape, np.float32)
    vp[tuple(slice(0, n) for n in shape)] = v
    V, Vp = torch.from_numpy(v).cuda(), torch.from_numpy(vp).cuda()
    for fmt in FMTS:
        P, X = blk.mxgemmini.quantize(V, fmt, axis=axis, scale_floor=2.0 ** -23)
        codes, scales = blk.mxgemmini.quantize_packed(Vp, fmt, axis=axis, scale_floor=2.0 ** -23)
        cut = list(shape)
        if fmt == "MXFP4":
            cut[-1] //= 2
        codes = codes[tuple(slice(0, n) for n in cut)].contiguous()
        scales = scales[tuple(slice(0, n) for n in X.shape)].contiguous()
        Pu, Xu = blk.unpack(codes, scales, fmt)
        assert_bits(Pu.cpu().numpy(), P.cpu().numpy(), f"{fmt} {shape} unpack P")
        assert_bits(Xu.cpu().numpy(), X.cpu().numpy(), f"{fmt} {shape} unpack X")
        D = blk.dequantize_packed(codes, scales, fmt, axis=axis)
        assert_bits(D.cpu().numpy(), blk.dequantize(P, X, axis=axis).cpu().numpy(), f"{fmt} {shape} dequantize_packed")
