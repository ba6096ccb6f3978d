"""Per-phase device time of the library's launches (C ABI ``yabt_phase_*``).

Every launch group of the library runs inside a named phase (tree set-up,
histogram, reduce, exchange, scan, finalize, partition, plan, finish, leaf
models, interaction detector, margin update, binning, collectives), which
always opens an NVTX range for profilers. ``start()`` records a CUDA event
pair around each phase range on the launching stream; ``read()`` sums them.
Recording adds event records between launches, so phases are measured in a
pass of their own, never inside a timed region.
"""

from __future__ import annotations

import contextlib
import ctypes

from . import _lib

COLLECTIVE = 13      # PH_COLLECTIVE of the C enum: host-issued collectives


def names() -> list[str]:
    lib = _lib.load()
    out = []
    for p in range(int(lib.yabt_phase_count())):
        buf = ctypes.create_string_buffer(32)
        _lib.check(lib.yabt_phase_name(p, buf, 32), "yabt_phase_name")
        out.append(buf.value.decode())
    return out


def start(max_ranges: int = 1 << 16) -> None:
    """Record phase ranges on the current device from now on (clears earlier ones)."""
    _lib.check(_lib.load().yabt_phase_timing(int(max_ranges)), "yabt_phase_timing")


def stop() -> None:
    _lib.check(_lib.load().yabt_phase_timing(0), "yabt_phase_timing")


def read() -> dict[str, dict]:
    """{phase: {"ms": summed device time, "ranges": count}} of the recorded ranges."""
    lib = _lib.load()
    n = int(lib.yabt_phase_count())
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_longlong * n)()
    _lib.check(lib.yabt_phase_read(ms, cnt, n), "yabt_phase_read")
    return {name: {"ms": ms[i], "ranges": int(cnt[i])} for i, name in enumerate(names()) if cnt[i]}


@contextlib.contextmanager
def host_phase(phase: int = COLLECTIVE, stream=None):
    """Time host-issued work on ``stream`` (default: torch's current stream) as ``phase``."""
    lib = _lib.load()
    _lib.check(lib.yabt_phase_push(int(phase), _lib.stream_ptr(stream)), "yabt_phase_push")
    try:
        yield
    finally:
        lib.yabt_phase_pop()
