"""B200 (sm_100a) Llama decode step behind the C ABI of include/lcr_b200.h.

``checkpoint`` holds the model geometry and the seeded random-init weights;
``runtime`` binds liblcr_b200.so (``Model`` mirrors the reference's Model,
the ``lcr_*`` entry points its src/kernels.cuh launchers).
"""
from . import checkpoint  # noqa: F401
