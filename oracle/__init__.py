"""CPU oracle for the quantized-linear hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product package imports this directory. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only as the checker or as the timed CPU
restatement of the reference's torch path.

Parity status:
  * fusions (adaln, rms_rope, swiglu), FP8 W8A8 quantization, the RoPE table and the NVFP4 *decode* side (LUT,
    nibble order, scale layout, dequant formula, global-scale formulas) are pinned against the reference's own
    code run in the build container (fixtures under ``tests/golden/``);
  * the NVFP4 *encoder* rounding lives in TensorFold v0.6.1 (a submodule absent from the reference checkout), so
    it is "parity unpinned": ``oracle/nvfp4.py`` states the rounding this build adopts and the GPU kernels are
    bit-exact against that statement.
"""
