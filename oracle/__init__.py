"""CPU oracle for the Tiny_Infra decode/prefill hot path.

TEST INFRASTRUCTURE ONLY. This package restates, in numpy float32, the algorithms of the
reference project (Unica2804/Tiny_Infra) for the continuous-batching hot path:

* ``oracle.kernels`` -- the three CUDA kernels (``src/attention.cu``, ``src/fused_rope.cu``,
  ``src/fused_swiglu.cu``), RMSNorm (``models/qwen_25.py:24-36``), the RoPE table
  (``engine/scheduler.py:36-48``) and the prefill attention of ``models/qwen_25.py:89-104``.
* ``oracle.cache`` -- the paged block allocator ``engine/cache_manager.py``.
* ``oracle.model`` -- the Qwen2 forward of ``models/qwen_25.py``.
* ``oracle.sampler`` -- ``_sample_next_token`` of ``engine/scheduler.py:104-156``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm may import it,
and only as the checker or as the timed CPU baseline.  The product package
(``tiny_infra_b200``) never imports it; the product has no CPU fallback.

Pinning: the oracle is checked against golden vectors in ``tests/golden/`` that were produced
by importing the reference's own Python modules (``tests/golden/make_golden.py``) and by running
the reference's own CUDA kernels compiled from its sources into ``oracle/_ref``
(``oracle/build_ref.py``, ``tests/golden/make_kernel_golden.py``).
"""
