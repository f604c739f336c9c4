"""Whether libscree_b200.so is present next to the package."""

from .._lib import LIB_PATH

NATIVE_AVAILABLE = LIB_PATH.exists()
