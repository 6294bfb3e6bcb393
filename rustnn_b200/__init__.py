"""rustnn_b200: B200 (sm_100a) backend for rustnn's dense-contraction path.

The compute lives in ``librnn_b200.so`` (hand-written tcgen05/TMEM kernels
behind the C ABI in ``include/rnn_b200.h``); this package is the thin
Python host layer over it.
"""
from ._lib import LIB_PATH, RnnError, lib  # noqa: F401

__all__ = ["LIB_PATH", "RnnError", "lib"]
