"""LUT host-side pieces without a GPU: the format tables the library builds (values, fixed points, finder-safe
values) against the reference's, and the argument checks of the lut API."""
import numpy as np
import pytest
import torch

import test_oracle_golden as g


def test_format_tables_match_reference():
    import mxq_host_tables
    g.test_lut_format_tables(mxq_host_tables)


def test_lut_argument_errors():
    import mxq
    P = torch.zeros(4, 6)
    with pytest.raises(ValueError, match="not a LUT format"):
        mxq.lut.tables(P, "MXFP4", group=1, max_iters=5)
    with pytest.raises(ValueError, match="non-negative integer"):
        mxq.lut.tables(P, "MXFP8_E4M3", group=-1, max_iters=5)
    with pytest.raises(ValueError, match="max_iters"):
        mxq.lut.tables(P, "MXFP8_E4M3", group=1, max_iters=-2)
    with pytest.raises(ValueError, match="K×n"):
        mxq.lut.pick(torch.zeros(3), torch.zeros(1, 16), group=0)
    with pytest.raises(ValueError, match="tables with width"):
        mxq.lut.pick(P, torch.zeros(2, 16), group=0)
    with pytest.raises(ValueError, match="2-D with axis 0 or 1"):
        mxq.block.lut.quantize(torch.zeros(2, 2, 2), "MXFP8_E4M3", 0, 32, rounding_mode="rne", scale_floor=1.0,
                               group=1, max_iters=1)
    assert mxq.lut.values("E3M2").dtype == torch.float32 and mxq.lut.SIZE == 16
