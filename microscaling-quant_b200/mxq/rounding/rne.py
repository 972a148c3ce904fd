"""Round to nearest, ties to even (IEEE default). The two forms of mxq/rounding/rne.py: `bits` on an int64 pattern with
the (drop, mask, half) of a kept width, `integer` on an integer-valued float. Both run as libmxq_b200 kernels;
`bits` returns the pattern reduced to 32 bits, as round_bits does."""
import torch


def bits(bits: torch.Tensor, drop, mask, half) -> torch.Tensor:
    from . import round_bits
    keep = 23 - drop if isinstance(drop, int) else (23 - torch.as_tensor(drop))
    return round_bits(bits, keep, "rne")


def integer(k: torch.Tensor) -> torch.Tensor:
    from . import round_int
    return round_int(k, "rne")
