"""anetransformers_b200 -- B200 (sm_100a) speculative-decode hot path for Mistral-architecture Q4_0 models.

A drop-in for the reference's (m0at/ANEtransformers) dequant.h / metal_matvec.h / speculative.h path:
the kernels live in libspecdec_b200.so behind the C ABI of include/specdec_b200.h; this package is the
Python mirror of that interface plus the GGUF reader / synthetic-model writer.
"""
from . import _lib, gguf  # noqa: F401
from ._lib import SpecDecError, lib  # noqa: F401

__all__ = ["gguf", "dequant", "engine", "lib", "SpecDecError"]
