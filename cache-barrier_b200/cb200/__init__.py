"""cb200 — B200 (sm_100a) kernels for the cache-barrier quantized-GEMM hot path.

Import the torch-facing ops from :mod:`cb200.ops`; the C ABI they call is
declared in ``include/cb200.h`` and implemented in ``csrc/`` (built into
``libcb200.so`` by ``cb200.build.build()``).
"""

from . import _lib  # noqa: F401
from . import build  # noqa: F401  (module: cb200.build.build() compiles the library)
from .build import LIB_PATH  # noqa: F401
