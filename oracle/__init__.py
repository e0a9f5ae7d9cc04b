"""CPU oracle for the quantized linear layer -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy, the arithmetic that openTPU defines for its matrix unit:
the fp32 rules (flush-to-zero, round-to-nearest-even, openTPU's own reciprocal sequence), the
activation quantizer QACT, the MX weight formats and their quantizers, the exact-integer MM
instruction and the float64 emulation the reference's model goldens use.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm may
import it, and only as the checker or as the timed CPU baseline. The product
(`opentpu_b200`) never imports it: the GPU path has no CPU fallback.

Parity status: pinned. Every function here is checked bit for bit against vectors produced by
running the reference itself (`tests/golden/make_golden.py` imports the reference package and
runs its ISA simulator); see `tests/test_oracle.py`.
"""
