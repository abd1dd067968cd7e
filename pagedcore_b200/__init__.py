"""B200-native paged KV-cache hot path with PagedCore's Python API.

Importing the package loads the native library (C++ block ledger + sm_100a
kernels); it fails if ``libpagedkv.so`` has not been built.
"""

from pagedcore_b200._lib import LIBRARY_PATH, lib  # noqa: F401  (loads the native library)

__all__ = ["LIBRARY_PATH", "lib"]
