"""CPU oracle for the KinoMLX denoise-step path -- TEST INFRASTRUCTURE ONLY.

A PyTorch-CPU restatement of the reference's formulas (KinoMLX 0.0.3, MLX on Apple GPUs), with
the fp32/bf16 rounding boundaries the reference documents, one function per reference function,
each citing the file:line it follows. The reference itself cannot run here (it needs MLX and
Python >= 3.15), so this restatement is the checker.

Pinning: the restatement is checked against the known-answer tests and golden values that the
reference's own tests hold for this path (tests/test_oracle_pins.py): the Klein schedule
midpoints, the Euler rounding order, the float64 RoPE grid, the LTX sigma pins, the tile
intervals and trapezoid masks, and the split-RoPE self-test recipe. Block- and model-level
outputs have no golden vectors in the reference (its real-checkpoint parity fixtures are not
shipped), so parity at that level is anchored on these op-level pins only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this package;
the product (kinomlx_b200) never does.
"""
