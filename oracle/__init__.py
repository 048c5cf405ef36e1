"""CPU oracle for the decode MoE path -- TEST INFRASTRUCTURE, not product code.

This package restates, on the CPU, the arithmetic of the reference's decode hot path so that the CUDA
kernels can be checked against it.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and its ``--impl reference`` arm) may import it, and only as the checker or as the timed
CPU baseline.  The product path never calls into this package and has no CPU fallback.

Modules
-------
``router_ref``  router GEMM -> bf16 logits -> fp32 softmax -> top-k (ties to the lower expert id) -> renormalise
                (reference ``serve/qwenfast/qf_router.cu:3-6, 84-86, 103-155``).
``moe_ref``     W4A16 routed experts with the kernel's bf16 rounding points, the fp32 "truth" of
                ``serve/qwenfast/test_a16moe.py:139-148``, and the shared expert of
                ``serve/qwenfast/test_a16moe.py:68-73`` (bf16 weights as in the synthetic configs).
``w8_ref``      group-128 INT8 weight quantisation (``serve/overlays/sglang/srt/qwenfast.py:301-315``), the
                W8A16 product of ``qf_w8g.cu`` and the W8A8 per-token / per-channel product (exact int64
                accumulators).

Parity status
-------------
* Pinned against the reference's own Python: ``tests/golden/make_golden.py`` extracts the reference functions
  ``w8_quant`` (qwenfast.py), ``route``, ``w8q``, ``shared_ref`` and ``truth`` (test_a16moe.py) from their
  source files, runs them on seeded inputs in the build container and stores the outputs under
  ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this package against them.
* The W8A8 arithmetic (per-token activation scale, int32 accumulation) has no counterpart in the reference; it
  follows the benchmark definition only, so that part is "parity unpinned" by the reference.
"""
