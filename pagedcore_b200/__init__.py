"""B200-native paged KV-cache hot path with PagedCore's Python API.

The native library (C++ block ledger + sm_100a kernels) is loaded by
``pagedcore_b200._lib`` on first use of any module that needs it; that import
fails if ``libpagedkv.so`` has not been built (``python -m pagedcore_b200.build``).
"""
