"""Element quantization to float(e, m) (mxq/element_quant/float_em.py:50-134): `rounding_mode` picks the rule
(ties_away | rne | truncate), `grid` the representable values:

    qtorch   qtorch 0.2.0 float_quantize: top exponent reserved, one binade of fake subnormals, saturating
    ieee     IEEE-like with true subnormals, overflow to Inf (the lane accumulators; (8, 7) is bf16)
    ocp      the OCP element formats only: ieee's subnormals, normals in the top exponent, saturate at max_norm

Input is float32 (any other dtype is cast) or float64 (rounded from float64 directly); output float32.
(8, 23) is float32 itself. One libmxq_b200 kernel per call (mxq_float_em_f32 / _f64).
"""
import torch

from .. import _lib
from ..rounding import mode_code
from .formats import FORMATS

__all__ = ["quantize", "bias", "GRIDS"]

GRIDS = ("qtorch", "ieee", "ocp")


def bias(e: int) -> int:
    """Exponent bias of a float with e exponent bits: 2^(e-1) - 1."""
    return (1 << (e - 1)) - 1


def quantize(z: torch.Tensor, e: int, m: int, rounding_mode: str = "ties_away", grid: str = "qtorch") -> torch.Tensor:
    if rounding_mode not in ("ties_away", "rne", "truncate"):
        raise ValueError(f"rounding_mode must be one of ('ties_away', 'rne', 'truncate'), got {rounding_mode!r}")
    if grid not in GRIDS:
        raise ValueError(f"grid must be one of {GRIDS}, got {grid!r}")
    if (e, m) != (8, 23) and not (1 <= e <= 8 and 1 <= m <= 22):
        raise ValueError(f"unsupported widths e={e}, m={m}")
    if grid == "ocp" and (e, m) != (8, 23) and not any((f.e, f.m) == (e, m) for f in FORMATS.values()):
        raise ValueError(f"grid='ocp' is defined only for the OCP element formats, not (e={e}, m={m})")
    home = _lib.home(z)
    dev = _lib.device_for(z)
    f64 = z.dtype == torch.float64
    x = _lib.on(z, dev, torch.float64 if f64 else torch.float32)
    out = torch.empty(x.shape, dtype=torch.float32, device=dev)
    _lib.run("mxq_float_em_f64" if f64 else "mxq_float_em_f32", dev, _lib.ptr(x), _lib.ptr(out), x.numel(), e, m,
             mode_code(rounding_mode), GRIDS.index(grid))
    return _lib.back(out, home)
