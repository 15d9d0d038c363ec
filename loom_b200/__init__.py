"""loom_b200: a B200-native (sm_100a) CUDA compute backend for Loom's quantized
Mixture-of-Experts forward path, behind Loom's compute-backend seam.

The product is the C ABI library ``loom_b200/lib/libloom_cuda.so``
(include/loom_cuda.h). ``loom_b200.backend`` mirrors the seam in Python;
``loom_b200.device`` drives the device-resident API.
"""
from ._lib import LoomCudaError  # noqa: F401
