"""CPU oracle for the Qwen3.5 fused inference hot path.

TEST INFRASTRUCTURE ONLY. This package restates, in plain PyTorch on the CPU,
the arithmetic of the reference project's fused operators (qwen35_fused/kernels.py,
qwen35_fused/validate_kernels.py) and of the Hugging Face eager Qwen3.5 modules they
replace. Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the checker or the
timed CPU baseline. The product package ``ppu_b200`` never imports it.

Parity is pinned by golden vectors generated from the reference's own torch reference
functions (validate_kernels.reference_*) and from the installed Transformers eager
modules; see ``tests/golden/make_golden.py``.
"""

from . import ops  # noqa: F401
from . import a8w8  # noqa: F401
