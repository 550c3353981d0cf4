"""CPU oracle for the resident decode step -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain torch fp32 on the CPU, the arithmetic of the reference project's decode step
(sott0n/tt-qwen-resident, ``qwen36_resident/model.py:219-292`` ``torch_step``), its seeded random weights and
decode state (``model.py:151-216``), its on-device sampling rules (``qwen36_resident/kernels/sampling.hpp``)
and the paged-KV indexing that this build uses for the KV cache.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import it, and there
only as the checker (or the timed CPU baseline). The product path (``tt_qwen_resident_b200``) never imports,
calls or links anything here: it runs the CUDA kernels of ``libqres.so`` and fails loudly without them.

Pinning: ``tests/golden/make_golden.py`` imports the reference's own ``torch_step`` (with a stub ``ttnn``
module) in the build container and records its outputs as fixtures; ``tests/test_oracle_golden.py`` checks
this restatement against them.
"""
