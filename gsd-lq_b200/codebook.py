"""A2 hexagonal-lattice codebooks.

A GSD-LQ code is one byte that indexes a table of 2-D lattice points.  The
table for radius R lists every A2 point ``(r0 + r1/2, r1*sqrt(3)/2)`` with
integers ``|r0|, |r1|, |r0+r1| <= R``, r0 the outer loop and r1 the inner one,
computed in float64 and rounded once to float32
(gsd_lq_v2/gsd_lq_cpu_runtime.py:111-118; the same generator is duplicated at
gsd_lq_v2/run_gpu_native_chat.py:26-33).  R=6 gives 127 points, R=8 gives 217.

The engine's kernels do not multiply by the float table directly: they use the
integer lattice coordinates (r0, r1), which are exact in bf16, and move the
irrational sqrt(3)/2 factor onto the activation side (see ``csrc/hexmv.cuh``).
``lattice_coords`` gives that integer form of the same table.
"""
from __future__ import annotations

import functools

import numpy as np

RADII = (6, 8)


@functools.lru_cache(maxsize=None)
def _enumerate(radius: int) -> tuple[tuple[int, int], ...]:
    return tuple((r0, r1)
                 for r0 in range(-radius, radius + 1)
                 for r1 in range(-radius, radius + 1)
                 if abs(r0 + r1) <= radius)


def num_points(radius: int) -> int:
    return len(_enumerate(radius))


def xy_table(radius: int) -> np.ndarray:
    """float32 [n_pts, 2] table of lattice points, bit-identical to the reference's."""
    h = float(np.sqrt(3.0) / 2.0)
    pts = np.array([[r0 + 0.5 * r1, r1 * h] for r0, r1 in _enumerate(radius)], dtype=np.float64)
    return pts.astype(np.float32)


def lattice_coords(radius: int) -> np.ndarray:
    """int8 [n_pts, 2] integer coordinates (r0, r1) of each code."""
    return np.array(_enumerate(radius), dtype=np.int8)


@functools.lru_cache(maxsize=None)
def code_index_table(radius: int) -> np.ndarray:
    """int32 [2R+1, 2R+1] map (r0+R, r1+R) -> code index, -1 outside the hexagon."""
    t = np.full((2 * radius + 1, 2 * radius + 1), -1, dtype=np.int32)
    for i, (r0, r1) in enumerate(_enumerate(radius)):
        t[r0 + radius, r1 + radius] = i
    return t
