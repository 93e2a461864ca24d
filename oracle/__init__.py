"""CPU oracle for the quantized MoE expert path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the algorithms of LLaDA_Quant's quantized
MoE expert path so that the CUDA kernels of ``llada_quant_b200`` can be
checked against them.  It is imported only by ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``.  The product path never imports it and has no CPU
fallback: every public op of ``llada_quant_b200`` raises when the CUDA library
is missing.

Pinning: the restatement is checked against golden vectors produced by the
reference package itself (``tests/golden/make_golden.py`` imports
``LLaDA_Quant`` and records its outputs), see ``tests/test_oracle_golden.py``.
The routed expert FFN (``fused_moe``) lives in an external repository that is
not part of the reference tree, so its semantics are restated from the
reference's description of that kernel (file:line cited in ``moe.py``); that
boundary is "parity unpinned" beyond the reference's own dense-expert tests.
"""
