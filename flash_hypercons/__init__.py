"""Drop-in import name of the original package: ``import flash_hypercons as fh``.

Re-exports the B200-native implementation in ``flash_hyperconnections_b200``.  The original
package's module paths resolve to the same module objects: ``flash_hypercons.ops``,
``flash_hypercons.ops.matrix_exp`` (with its private helpers ``_eligible``, ``_native``,
``_MatrixExpMode``) and ``flash_hypercons._C``.
"""

import sys as _sys

from flash_hyperconnections_b200 import __version__, _C, matrix_exp, matrix_exp_and_grad, mix_streams, ops, use_backend  # noqa: F401
from flash_hyperconnections_b200.ops import matrix_exp as _matrix_exp_module

_sys.modules[__name__ + "._C"] = _C
_sys.modules[__name__ + ".ops"] = ops
_sys.modules[__name__ + ".ops.matrix_exp"] = _matrix_exp_module

__all__ = ["matrix_exp", "use_backend"]
