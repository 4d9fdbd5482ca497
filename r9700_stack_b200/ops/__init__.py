"""Python entry points for the sm_100a kernel library (``torch.ops.r9k``)."""
