"""CPU oracle for the quantized-linear hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic of the reference
(xiro2416/inspark_proper_format) for every operation the CUDA library
implements: norm→quantize, W8A8 FP8 / INT8 SmoothQuant / NVFP4 scaled GEMMs,
the CFM gated-up SwiGLU epilogue and the BigVGAN alias-free Snake FIR.  Each
function cites the reference file:line it follows (paths relative to the
reference project root).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or as the timed CPU baseline.  The product path
(``inspark_proper_format_b200``) never imports it and has no CPU fallback.

Parity pinning: the restatements are checked against golden vectors that were
produced by running the reference's own PyTorch modules (see
``tests/golden/make_golden.py``).  The NVFP4 quantizer restates NVIDIA ModelOpt
0.47's published NVFP4 scheme, which is not part of the reference tree; its
parity against ModelOpt itself is unpinned (no ModelOpt in this environment and
no golden vectors for it in the reference).
"""
