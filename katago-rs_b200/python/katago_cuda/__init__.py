"""Python binding of the katago-rs B200 backend (libkatago_cuda.so, C ABI in include/katago_cuda.h).

The binding is a thin ctypes layer used by the tests and the benchmark; the product is the shared library. Loading
fails loudly if the library has not been built: there is no Python or CPU fallback for the forward pass.
"""

from .api import (  # noqa: F401
    PRECISION_AUTO,
    PRECISION_BF16,
    PRECISION_F16,
    PRECISION_F32,
    Context,
    Handle,
    KcError,
    Model,
    device_count,
    lib,
    library_path,
)
