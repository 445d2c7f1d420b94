"""CPU oracle for the weight-only quantized GEMV path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference's own torch "dequantise then matmul"
path and its NVFP4 codec, so the CUDA kernels can be checked against it:

* ``oracle.numerics`` -- bf16 round-to-nearest-even, e4m3 / e2m1 decode and encode;
* ``oracle.nvfp4``    -- NVFP4 pack/unpack, ModelOpt quantiser, dequantiser, the 128x4
  block-scale swizzle, and the NVFP4 GEMV;
* ``oracle.w8a16``    -- the W8A16 GEMV (int8 / fp8 weights, per-row scales), its fused
  gate_up SiLU form and the greedy argmax;
* ``oracle.moe``      -- the routed-MoE layer (server and checkpoint row orders), with an
  optional always-on shared expert;
* ``oracle.router``   -- the router projection and the softmax top-k routing table.

Parity pins: the functions are checked against golden vectors produced by the
reference's own Python code (``tests/golden/make_golden.py``, fixtures in
``tests/golden/``) and against the known answers of its CPU tests.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this package, and only as the checker or the timed CPU baseline.  The product
(``flash_next_rtxpro6000_b200``) never imports it.
"""

from . import moe, numerics, nvfp4, router, w8a16  # noqa: F401
