"""B200 (sm_100a) implementation of the Qwen3.5 fused inference hot path.

Drop-in for the reference's ``qwen35_fused`` package: ``ppu_b200.kernels`` mirrors
``qwen35_fused.kernels``; ``ppu_b200.engine`` runs the whole text decoder (prefill + greedy
decode) through the C ABI in ``include/qwen35_b200.h``.
"""

from .config import FusionConfig, Qwen35Dims  # noqa: F401

__all__ = ["FusionConfig", "Qwen35Dims"]
