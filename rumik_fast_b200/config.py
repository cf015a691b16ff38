"""Launch settings shared by the Python wrappers.

PDL (programmatic dependent launch) is on by default: a kernel may be scheduled while the previous kernel on
the stream finishes, and it waits for it (griddepcontrol.wait) before reading activations or writing
outputs, so stream order semantics are unchanged.

Weight prefetch is off by default. When on, a GEMV starts streaming its weights into shared memory BEFORE
that wait, which hides the kernel-boundary bubble in a chain of GEMVs. It is only correct when the weights
are not written by the kernel that runs immediately before the GEMV on the same stream - true for inference
weights loaded once (the decode loop of an engine), not for a kernel that has just produced the weights.
The same switch lets the decode attention read the position and the K/V rows of the slots before it ahead of
its wait (only q and the token's own slot come from the launch before it in a decode step).
"""
import contextlib

from . import _lib

PDL = True
PREFETCH_WEIGHTS = False


def set_weight_prefetch(on: bool):
    global PREFETCH_WEIGHTS
    PREFETCH_WEIGHTS = bool(on)


@contextlib.contextmanager
def weight_prefetch(on: bool = True):
    """Temporarily enable (or disable) weight prefetch across kernel boundaries."""
    global PREFETCH_WEIGHTS
    old = PREFETCH_WEIGHTS
    PREFETCH_WEIGHTS = bool(on)
    try:
        yield
    finally:
        PREFETCH_WEIGHTS = old


def flags():
    f = 0
    if PDL:
        f |= _lib.FLAG_PDL
        if PREFETCH_WEIGHTS:
            f |= _lib.FLAG_PREFETCH_WEIGHTS
    return f
