"""The reference's own CUDA kernel, built unmodified by baseline/Makefile
(measurement and parity pinning only; never on the product path)."""
