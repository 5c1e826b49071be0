"""CPU oracle for the W8A16 / W4A16 quantized linear layer.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this module;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
(and ``bench.py --impl reference``) may use it, and only as the checker or as the
timed CPU baseline -- never as the thing measured on the GPU.

The functions restate, in numpy, the reference implementation of the path:

* ``quant_oracle.quantize_int8`` / ``dequantize_int8``  -- reference
  ``learning/10_cuda_decode/activation_int8.py:24-64``.
* ``quant_oracle.quantize_int4`` / ``dequantize_int4``  -- reference
  ``learning/09_int4/quantization.py:35-71``.
* ``quant_oracle.linear``        -- the reference's oracle expression
  ``(dequantize(packed) @ x.float()).bfloat16()``
  (``profiling/decode_stage2_benchmark.py:55``,
  ``learning/10_cuda_decode/test_cuda_decode.py:30-31``), generalised to M rows.
* ``quant_oracle.swiglu``        -- the model-ordered SwiGLU epilogue of
  ``learning/10_cuda_decode/warp_gemv.cu:46-50``.
* ``quant_oracle.quantize_int8_rowwise`` / ``quantize_int4_asym`` -- restatements
  of the BASELINE.json weight formats (per-row bf16 scale; asymmetric 4-bit with
  bf16 scale and zero-point per 128-group), which have no reference function.

Parity pin: ``tests/golden/reference_vectors.npz`` holds outputs of the
reference's own Python functions, generated in the build container by
``tests/golden/make_golden.py``; ``tests/test_oracle.py`` checks this oracle
against them.
"""
