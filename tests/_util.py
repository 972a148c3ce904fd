"""Shared helpers for the tests: bit-exact comparison with NaN-aware semantics, and golden fixture loading."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
_cache = {}


def golden(name):
    """Load tests/golden/<name>.npz once per session."""
    if name not in _cache:
        _cache[name] = dict(np.load(os.path.join(GOLDEN, name + ".npz"), allow_pickle=False))
    return _cache[name]


def as_np(x):
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.asarray(x)


def bits_equal(a, b):
    """True when a and b are bit-identical, except that a NaN only has to meet a NaN (its sign and payload are
    the host's NaN propagation, not a value). Integer arrays compare exactly."""
    a, b = as_np(a), as_np(b)
    if a.shape != b.shape:
        return False
    if a.dtype.kind != "f":
        return bool(np.array_equal(a, b))
    if a.dtype != b.dtype:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    ua = a.view(np.uint32 if a.dtype == np.float32 else np.uint64)
    ub = b.view(np.uint32 if b.dtype == np.float32 else np.uint64)
    return bool(np.array_equal(ua[~na], ub[~nb]))


def assert_bits(a, b, what=""):
    a, b = as_np(a), as_np(b)
    if bits_equal(a, b):
        return
    msg = f"{what}: shape {a.shape} vs {b.shape}, dtype {a.dtype} vs {b.dtype}"
    if a.shape == b.shape and a.dtype == b.dtype and a.dtype.kind == "f":
        ua = a.view(np.uint32 if a.dtype == np.float32 else np.uint64).reshape(-1)
        ub = b.view(np.uint32 if b.dtype == np.float32 else np.uint64).reshape(-1)
        bad = np.nonzero((ua != ub) & ~(np.isnan(a.reshape(-1)) & np.isnan(b.reshape(-1))))[0]
        msg += f"; {bad.size} of {a.size} differ, first at {bad[:5].tolist()}: " \
               f"{[hex(int(x)) for x in ua[bad[:5]]]} vs {[hex(int(x)) for x in ub[bad[:5]]]}"
    elif a.shape == b.shape:
        bad = np.nonzero(a.reshape(-1) != b.reshape(-1))[0]
        msg += f"; {bad.size} differ, first at {bad[:5].tolist()}"
    raise AssertionError(msg)


def nan_block_mask(V, axis, block_size=32):
    """Elements of V whose block (block_size along axis) holds a NaN. block.mxquant's codes there depend on the
    NaN payload torch's amax kernel returns, which differs between tensor layouts in the reference itself
    (0x7fc00000 for one, 0xffffffff for another), so they are excluded from bit comparisons."""
    V = as_np(V)
    axis = axis % V.ndim
    Vt = np.moveaxis(np.isnan(V), axis, -1)
    L = Vt.shape[-1]
    pad = (-L) % block_size
    Vp = np.concatenate([Vt, np.zeros(Vt.shape[:-1] + (pad,), bool)], -1)
    blk = Vp.reshape(*Vp.shape[:-1], -1, block_size).any(-1, keepdims=True)
    full = np.broadcast_to(blk, blk.shape[:-1] + (block_size,)).reshape(*Vp.shape[:-1], -1)[..., :L]
    return np.moveaxis(full, -1, axis)


def assert_bits_where(a, b, keep, what=""):
    """assert_bits on the elements where `keep` is True."""
    a, b = as_np(a), as_np(b)
    assert a.shape == b.shape, f"{what}: shape {a.shape} vs {b.shape}"
    assert_bits(a[keep], b[keep], what)
