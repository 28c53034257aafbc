"""Data transforms: split/rANS codec and fp8 packing (GPU kernels + CPU oracle)."""
