"""mxq_block_lut_quantize_static, the block.lut entry point whose scratch is a static device array (it allocates
nothing), against mxq_block_lut_quantize with a workspace on the same inputs: bit for bit, on two calls in a row
(every call shares the array), both axes and two groupings; and a size whose scratch exceeds the array is refused
before any device work. The file sorts last so it also runs after every other GPU test."""
import ctypes

import numpy as np
import pytest
import torch

from _util import assert_bits

pytestmark = pytest.mark.gpu


def _operand(rows, cols, seed):
    """config 4's distribution: column j ~ N(0, sigma_j^2), sigma_j = 2^U[-8, 8]."""
    rng = np.random.default_rng(seed)
    V = rng.standard_normal((rows, cols)) * 2.0 ** rng.uniform(-8, 8, (1, cols))
    return torch.from_numpy(V.astype(np.float32)).cuda()


def _call(name, V, axis, group, workspace=None):
    from mxq import _lib
    from mxq.block import mxgemmini
    spec = mxgemmini.spec("MXFP6_E3M2", "rne", 2.0 ** -23)
    rows, cols = V.shape
    P = torch.full_like(V, float("nan"))
    xshape = [rows, cols]
    xshape[axis] = (xshape[axis] + 31) // 32
    X = torch.full(xshape, float("nan"), dtype=torch.float32, device=V.device)
    st = torch.full((1,), 7, dtype=torch.int32, device=V.device)
    args = [_lib.ptr(V), _lib.ptr(P), _lib.ptr(X), rows, cols, axis, 32, ctypes.byref(spec), group, 50]
    if workspace is not None:
        args += [_lib.ptr(workspace), workspace.numel()]
    _lib.run(name, V.device, *args, _lib.ptr(st))
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    return P.cpu().numpy(), X.cpu().numpy()


@pytest.mark.parametrize("axis,group", [(0, 1), (1, 3)])
def test_static_scratch_matches_workspace(axis, group):
    from mxq import _lib
    V = _operand(512, 384, 12 + axis)
    need = _lib.lib().mxq_block_lut_workspace(512, 384, axis, group)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    want_P, want_X = _call("mxq_block_lut_quantize", V, axis, group, ws)
    for call in range(2):
        P, X = _call("mxq_block_lut_quantize_static", V, axis, group)
        assert_bits(P, want_P, f"P, call {call + 1}")
        assert_bits(X, want_X, f"X, call {call + 1}")


def test_static_scratch_refuses_oversize():
    from mxq import _lib
    from mxq.block import mxgemmini
    spec = mxgemmini.spec("MXFP6_E3M2", "rne", 2.0 ** -23)
    with pytest.raises(ValueError, match="static scratch"):
        _lib.run("mxq_block_lut_quantize_static", torch.device("cuda", 0), None, None, None, 4096, 4096, 0, 32,
                 ctypes.byref(spec), 1, 50, None)
