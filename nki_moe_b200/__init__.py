"""B200 (sm_100a) implementation of the Qwen3-30B-A3B sparse-MoE block and
the norms that feed it, behind the Python interface of Goomelo/nki-moe's
kernel modules (``nki_custom_rmsnorm``, ``nki_moe_integrated``,
``nki_moe_kernel``, ``nki_moe_expert``).

``install_reference_aliases()`` registers those four module names in
``sys.modules`` so that a model file written against the reference
(``from nki_custom_rmsnorm import NKIRMSNorm``,
``from nki_moe_integrated import NKIMoEWrapper, enable_nki_moe``) imports
this package instead.
"""

from __future__ import annotations

import importlib
import sys

__version__ = "0.1.0"

REFERENCE_MODULES = ("nki_custom_rmsnorm", "nki_moe_integrated", "nki_moe_kernel", "nki_moe_expert")


def install_reference_aliases() -> None:
    for name in REFERENCE_MODULES:
        sys.modules[name] = importlib.import_module(f"{__name__}.{name}")


def lib_path() -> str:
    from ._lib import LIB_PATH
    return LIB_PATH
