"""openTPU's quantized linear layer on NVIDIA B200.

A from-scratch sm_100a implementation of the reference's weight-quantized linear layer (its
MM / QACT numerics, MX weight formats, int8 per-row and 4-bit group-32 weights) behind a C ABI
(include/otq.h, libotq.so) with torch-level operators in `opentpu_b200.linear`.
"""
__version__ = "0.1.0"
