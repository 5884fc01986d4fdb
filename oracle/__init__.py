"""CPU oracle for the Qwen3-30B-A3B sparse-MoE block and its norms.

TEST INFRASTRUCTURE ONLY. This package restates, in numpy, the arithmetic of
the reference's PyTorch CPU paths (Goomelo/nki-moe) so that the CUDA product
path can be checked against it.  Only ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` may import it; the product package
``nki_moe_b200`` never does, and fails loudly when its CUDA library is absent.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own CPU code
(``NKIMoESimple``, ``NKIMoEExpertMLP._fallback_forward``,
``NKIMoELayer._pytorch_forward``, ``NKIRMSNorm._fallback_forward``) and HF
``transformers`` 5.5 (RMSNorm, rotate-half RoPE) and commits their outputs as
fixtures; ``tests/test_oracle_golden.py`` checks this oracle against them.
"""

from .moe_oracle import *  # noqa: F401,F403
