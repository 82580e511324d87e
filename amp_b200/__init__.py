"""amp_b200 -- B200-native (sm_100a) kernels for AMP's data-parallel hot path.

The compute lives in ``libamp_b200.so`` (C ABI in ``include/amp_b200.h`` and
``include/amp_plugin.h``); this package is the host-side mirror of the
reference's launcher API over torch device tensors.
"""
from ._lib import AmpError, LIB_PATH, lib  # noqa: F401

__all__ = ["AmpError", "LIB_PATH", "lib"]
