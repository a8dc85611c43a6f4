"""Python host binding of the B200-native GWP-0.5 MoT engine (libwam_b200.so).

The product is the C ABI in include/wam_b200.h; this package binds it with
ctypes for the tests and the benchmark.
"""
from ._lib import LIB_PATH, check, last_error, load  # noqa: F401
