"""CPU oracle for the Qwen3.5-MoE block-verify path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the arithmetic of the reference's host
oracle ``reference/fused_ops.py`` and of the layer composition in
``model/qwen35_moe_dflash/fused/model.py``.  It exists to check the CUDA
library, never to replace it: only ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py`` may import it.  The product path
(``qwen35_dflash_b200``) never imports this package and has no CPU fallback.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own
``fused_ops`` functions, its ``FusedTargetModel``/``FusedTargetSession`` and
``torch.topk`` on seeded inputs and stores their outputs as fixtures under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this package
against every one of them.
"""
