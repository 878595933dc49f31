"""CPU oracle for the quantized dequant-GEMM family -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference modules of
lilian-muyaoli/kernelbench-harbor that the CUDA library replaces.  It is the
checker and nothing else: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product path (``kernelbench_harbor_b200``) never imports it and has no CPU
fallback.

Modules
-------
w4a16      numpy restatement of QUANT_REF (generate_tasks.py:45-74): packer,
           bit-exact unpack, fp16 dequant in the reference's op order, fp32
           ground truth (common/kb_verifier.py:194-196 convention).
w8a8       numpy restatement of W8A8_REF (generate_tasks.py:198-215) plus the
           the benchmark's SmoothQuant input preparation (alpha = 0.5 smoothing,
           1 % outlier channels, per-token int8 activations).
mxfp8      OCP-MX v1.0 e4m3 + E8M0 block quantiser and block-scaled GEMM; there
           is no reference module for this config (parity: see its header).
moe        routing of MOE_REF / FUSED_QMOE_REF (generate_tasks.py:171-178,
           368-378) and the composite W4A16 top-2 MoE FFN.
reference_port
           torch-CPU restatement of the reference ``Model.forward`` op sequence,
           used only as the timed CPU baseline.
lora, silu_fp8
           numpy restatements of LORA_REF / multi_lora_qgemm and FUSED_SILU_REF.

Parity pinning: the numpy restatements are checked against golden vectors
produced by the reference modules themselves (``tests/golden/make_golden.py``
imports the reference task files and runs them on CPU with seeded inputs).
"""
