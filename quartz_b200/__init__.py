"""quartz_b200: the B200-native (sm_100a) fused int8 weight-only matmul path.

Drop-in for quartz's ``quartz.kernels`` numpy entry points
(``quartz_b200.kernels``), a torch-tensor device API (``quartz_b200.device``),
and ``install()`` to route an installed quartz package to these kernels.
The CUDA work is done by libquartz_b200.so (C ABI in include/quartz_b200.h).
"""

from .drop_in import install  # noqa: F401
