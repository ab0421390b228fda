"""B200-native batched AVBD environment step (drop-in for duck_gym's CudaBatch).

``CudaBatch`` is the reference-compatible Python API over the C ABI in
``include/duck_b200.h``; ``biped`` generates the seeded synthetic biped.
"""

from .cuda_batch import CudaBatch, fp32_peak_tflops, library

__all__ = ["CudaBatch", "fp32_peak_tflops", "library"]
