"""mxq.lut — MX-Gemmini's look-up tables (placeholder until the LUT kernels land)."""
