"""B200-native batched small-matrix exponential with a structured Frechet backward.

Drop-in for the ``flash_hypercons`` Python surface: ``matrix_exp``, ``use_backend`` and the
``flash_hypercons::_matrix_exp`` / ``flash_hypercons::_frechet`` operators.  The operators run
hand-written sm_100a kernels through the C ABI of ``include/fhx.h``; there is no CPU fallback
inside the operators (CPU and other ineligible tensors are routed to native PyTorch before they
reach them, exactly as in the original package).
"""

from ._native import load_extension as _load_extension

_C = _load_extension()

from .ops.matrix_exp import matrix_exp, matrix_exp_and_grad, mix_streams, use_backend  # noqa: E402

__version__ = "0.1.0"
__all__ = ["matrix_exp", "matrix_exp_and_grad", "mix_streams", "use_backend"]
