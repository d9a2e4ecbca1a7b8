"""Cortex decoder forward hot path on NVIDIA B200 (sm_100a).

Drop-in for the reference package's ``cortex.models``, ``cortex.kernels`` and
``cortex.quantization.calibrate`` call surface; the compute runs in the
hand-written CUDA kernels of ``libcortex_b200.so`` (C ABI: include/cortex_b200.h).
"""

__version__ = "0.1.0"
