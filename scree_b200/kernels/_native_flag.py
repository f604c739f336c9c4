"""Whether libscree_b200.so is present next to the package and loads."""

from .._lib import load as _load


def _loads() -> bool:
    try:
        _load()
    except OSError:
        return False
    except ImportError:
        return False
    return True


NATIVE_AVAILABLE = _loads()
