"""Loading of the in-tree native libraries.

Import fails loudly when they are missing: the operators have no Python or CPU fallback.
Build them with ``python flash_hyperconnections_b200/build.py`` (or ``__graft_entry__.build()``).
"""

from __future__ import annotations

import ctypes
import importlib
import pathlib

_PKG = pathlib.Path(__file__).resolve().parent
LIBFHX_PATH = _PKG / "libfhx.so"
TORCH_EXT_PATH = _PKG / "_C.so"


def load_extension():
    """Import the operator-registration module ``_C`` (registers the flash_hypercons ops)."""
    import torch  # noqa: F401  (loads libtorch / libc10 before the extension)

    if not TORCH_EXT_PATH.exists() or not LIBFHX_PATH.exists():
        raise ImportError(
            f"flash_hyperconnections_b200: native libraries missing ({TORCH_EXT_PATH.name}, {LIBFHX_PATH.name}); "
            "build them with `python flash_hyperconnections_b200/build.py`"
        )
    return importlib.import_module(f"{__package__}._C")


def load_cabi() -> ctypes.CDLL:
    """Open ``libfhx.so`` for direct C-ABI calls (tests, benchmarks, other languages' stubs)."""
    if not LIBFHX_PATH.exists():
        raise OSError(f"{LIBFHX_PATH} missing; build it with `python flash_hyperconnections_b200/build.py`")
    lib = ctypes.CDLL(str(LIBFHX_PATH))
    i64, i32, vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p
    lib.fhx_matrix_exp.argtypes = [vp, i64, i64, i64, i32, vp, i64, i32, i32, vp]
    lib.fhx_matrix_exp.restype = i32
    lib.fhx_frechet.argtypes = [vp, i64, i64, i64, i32, vp, i64, i64, i64, i32, vp, i64, i32, i32, vp]
    lib.fhx_frechet.restype = i32
    sz = ctypes.c_size_t
    lib.fhx_workspace_bytes.argtypes = [i64, i32]
    lib.fhx_workspace_bytes.restype = sz
    lib.fhx_matrix_exp_ws.argtypes = [vp, i64, i64, i64, i32, vp, i64, i32, i32, vp, sz, vp]
    lib.fhx_matrix_exp_ws.restype = i32
    lib.fhx_frechet_ws.argtypes = [vp, i64, i64, i64, i32, vp, i64, i64, i64, i32, vp, i64, i32, i32, vp, sz, vp]
    lib.fhx_frechet_ws.restype = i32
    lib.fhx_frechet_grouped.argtypes = [vp, i64, i64, i64, i32, vp, i64, i64, i64, i32, vp, i64, i32, i32, vp, sz, vp]
    lib.fhx_frechet_grouped.restype = i32
    lib.fhx_launch_count.argtypes = []
    lib.fhx_launch_count.restype = ctypes.c_uint64
    lib.fhx_matrix_exp_noalloc.argtypes = [vp, i64, i64, i64, i32, vp, i64, i32, i32, vp]
    lib.fhx_matrix_exp_noalloc.restype = i32
    lib.fhx_matrix_exp_frechet.argtypes = [vp, i64, i64, i64, i32, vp, i64, i64, i64, i32, vp, i32, vp, i64, i32, i32,
                                           vp, sz, vp]
    lib.fhx_matrix_exp_frechet.restype = i32
    lib.fhx_stream_mix.argtypes = [vp, i64, i64, i64, i32, i32, vp, i64, i64, i32, vp, i64, i32, i64, vp]
    lib.fhx_stream_mix.restype = i32
    lib.fhx_stream_mix_backward.argtypes = [vp, i64, i64, i64, i32, i32, vp, i64, i64, i32, vp, i64, i64, vp, vp,
                                            i64, i32, i64, vp, ctypes.c_size_t, vp]
    lib.fhx_stream_mix_workspace_bytes.argtypes = [i64, i32]
    lib.fhx_stream_mix_workspace_bytes.restype = ctypes.c_size_t
    lib.fhx_stream_mix_backward.restype = i32
    lib.fhx_status_string.argtypes = [i32]
    lib.fhx_status_string.restype = ctypes.c_char_p
    lib.fhx_abi_version.argtypes = []
    lib.fhx_abi_version.restype = i32
    lib.fhx_last_cuda_error.argtypes = []
    lib.fhx_last_cuda_error.restype = i32
    lib.fhx_last_cuda_error_string.argtypes = []
    lib.fhx_last_cuda_error_string.restype = ctypes.c_char_p
    return lib
