"""CPU oracle for tilec.ext.matrix_mul -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may
import this package, and only as the checker or the timed CPU baseline.  The product
path (tilec_b200) never imports it and has no CPU fallback.

Three oracles, all computing C = x1 @ x2 for fp32 row-major operands:

* ``mm_tiled``  -- plain-C restatement of the reference kernel tilec/ext.py:13-24 with
  its 64x64x16 launch (ext.py:54,62): masked loads with other=0.0, fp32 dot per BK
  block added to the accumulator, masked store (oracle/mm_tiled.c).
* ``mm_torch``  -- the reference test's own oracle expression ``x1 @ x2``
  (tests/test_matmul.py:40), evaluated in torch fp32 on the CPU.
* ``mm_f64``    -- fp64-accumulating reference that both fp32 oracles are checked
  against (relative Frobenius error about 3e-7 on N(0,1) data).

Parity pin: the reference ships no golden vectors and its Metal path cannot run here
(no Rust toolchain, no MLIR, no Apple GPU).  tests/golden/make_golden.py executes the
reference's own kernel text (_matmul_tiled from tilec/ext.py) under a numpy model of
the tile-language builtins and commits its outputs; tests/test_oracle.py pins
``mm_tiled`` to those vectors (bit-exact on exactly representable inputs).
"""
from .oracle import mm_tiled, mm_f64, mm_torch, rel_frob, lib_path, build  # noqa: F401
