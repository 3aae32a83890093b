"""Scoped, verified attribute patches for the research adapters.

The reference's research contexts swap a callable in a host module for the
duration of a `with` block and refuse to restore it if somebody else changed
it meanwhile (rdna2_ops/int8_gemm.py:265-271, 324-330).  This package does
that through one helper: `scoped_patch(owner, {name: replacement}, label)`
installs every replacement, yields, and on exit first checks that each
attribute still holds the object it installed -- raising RuntimeError and
leaving the foreign value in place if not -- before putting the saved
originals back.
"""
from __future__ import annotations

from contextlib import contextmanager


class CandidateStats(dict):
    """The statistics dict the research contexts yield: hits, fallbacks and
    a per-shape "(M, N, K)" hit count."""

    def __init__(self):
        super().__init__(hits=0, fallbacks=0, shapes={})

    def hit(self, m, n, k):
        self["hits"] += 1
        key = str((m, n, k))
        self["shapes"][key] = self["shapes"].get(key, 0) + 1

    def fallback(self):
        self["fallbacks"] += 1


@contextmanager
def scoped_patch(owner, replacements, label):
    saved = {name: getattr(owner, name) for name in replacements}
    for name, fn in replacements.items():
        setattr(owner, name, fn)
    try:
        yield
    finally:
        foreign = [name for name, fn in replacements.items() if getattr(owner, name) is not fn]
        if foreign:
            raise RuntimeError(f"{label} changed during the research context: {', '.join(foreign)}")
        for name, fn in saved.items():
            setattr(owner, name, fn)
