"""mxq.microxcaling — OCP MX element formats (placeholder)."""
