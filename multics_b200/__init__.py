"""B200-native (sm_100a) hierarchical group attention for Multics.

Host code mirrors the reference's Python API; all compute runs in
``libhier_b200.so`` (C ABI in include/hier_b200.h).
"""

from . import _lib  # noqa: F401

__version__ = "0.1.0"
