"""Drop-in import name of the original package: ``import flash_hypercons as fh``.

Re-exports the B200-native implementation in ``flash_hyperconnections_b200``.
"""

from flash_hyperconnections_b200 import __version__, _C, matrix_exp, use_backend  # noqa: F401

__all__ = ["matrix_exp", "use_backend"]
