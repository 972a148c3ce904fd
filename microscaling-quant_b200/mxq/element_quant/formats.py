"""The OCP MX element formats shared by every block quantizer (mxq/element_quant/formats.py:13-51).

One row per format: exponent and mantissa widths, the OCP emax and max_norm, and the microxcaling name. "FP32"
(or None) is the pass-through and resolves to None. The values are the OCP Microscaling v1.0 specification's.
"""
from dataclasses import dataclass
from typing import Optional, Union

__all__ = ["Format", "FORMATS", "get"]


@dataclass(frozen=True)
class Format:
    name: str
    e: int
    m: int
    emax: int
    max_norm: float
    ocp: str


FORMATS = {f.name: f for f in (
    Format("MXFP8_E4M3", 4, 3, 8, 448.0, "fp8_e4m3"),
    Format("MXFP8_E5M2", 5, 2, 15, 57344.0, "fp8_e5m2"),
    Format("MXFP6_E3M2", 3, 2, 4, 28.0, "fp6_e3m2"),
    Format("MXFP6_E2M3", 2, 3, 2, 7.5, "fp6_e2m3"),
    Format("MXFP4", 2, 1, 2, 6.0, "fp4_e2m1"),
)}

# accepted alternative spellings -> FORMATS key
_ALIASES = {}
for _canon, _names in (("MXFP8_E4M3", ("FP8_E4M3", "E4M3", "MX_E4M3")), ("MXFP8_E5M2", ("FP8_E5M2", "E5M2", "MX_E5M2")),
                       ("MXFP6_E3M2", ("FP6_E3M2", "E3M2")), ("MXFP6_E2M3", ("FP6_E2M3", "E2M3")),
                       ("MXFP4", ("FP4", "FP4_E2M1", "E2M1", "MXFP4_E2M1"))):
    for _n in _names:
        _ALIASES[_n] = _canon


def get(fmt: Union[str, Format, None]) -> Optional[Format]:
    """A format name (case-insensitive, aliases allowed) or Format -> Format; "FP32" / None -> None."""
    if fmt is None or isinstance(fmt, Format):
        return fmt
    key = fmt.strip().upper()
    if key == "FP32":
        return None
    key = _ALIASES.get(key, key)
    if key not in FORMATS:
        raise ValueError(f"Unknown format '{fmt}'. Known: {sorted(FORMATS)} + FP32")
    return FORMATS[key]
