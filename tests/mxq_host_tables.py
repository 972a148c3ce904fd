"""The library's host-side LUT format tables behind the oracle's name (lut_format_tables), for a CPU golden check."""
import mxq

LUT_FORMATS = ("MXFP6_E3M2", "MXFP6_E2M3", "MXFP8_E5M2", "MXFP8_E4M3")


def lut_format_tables(fmt):
    v, fx, s = mxq.lut.formats._tables(fmt)
    return v.numpy(), fx.numpy(), s.numpy()
