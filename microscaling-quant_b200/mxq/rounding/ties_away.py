"""Round to nearest, ties away from zero (qtorch's nearest), in the two forms of mxq/rounding/ties_away.py:5-10.

    bits(bits, drop, mask, half)   int64 float32 bit patterns rounded with the given drop / mask / half (ints or
                                   int64 tensors, broadcast); the int64 result keeps any carry past bit 31
                                   (round_bits reduces it to 32 bits)
    integer(k)                     an integer-valued float32 / float64 tensor rounded to an integer

Both run on the device (mxq_round_pattern, mxq_round_int_*)."""
import torch


def bits(bits: torch.Tensor, drop, mask, half) -> torch.Tensor:
    from . import _pattern
    return _pattern(bits, drop, mask, half, "ties_away")


def integer(k: torch.Tensor) -> torch.Tensor:
    from . import round_int
    return round_int(k, "ties_away")
