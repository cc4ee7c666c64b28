"""Crash reporting for native faults.

``install_crash_handler()`` enables Python's ``faulthandler`` (Python stacks of
every thread) and the native reporter of ``flodl_b200._native`` (faulting
address plus the native frames as ``module +offset``, which ``addr2line -e
<module> <offset>`` resolves for the in-tree extension modules). The process
still terminates with the original signal.
"""
from __future__ import annotations

import faulthandler

from .._ext import native


def install_crash_handler() -> None:
    faulthandler.enable()
    native().install_crash_handler()
