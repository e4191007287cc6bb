"""Column-parallel evaluation of the C oracle, and its tolerance checks.

Every column of the fan-out / fan-in ops is independent, so the sequential
oracle run on a block of columns gives exactly the same values as one
whole-array call. Large cases run the blocks on a thread pool (the oracle is a
ctypes call, which releases the GIL), sized by the host's cores and memory.
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np


def threads_for(bytes_per_block: int, blocks: int) -> int:
    try:
        import psutil

        avail = psutil.virtual_memory().available
    except Exception:  # pragma: no cover - psutil is in the image
        avail = 32 << 30
    by_mem = max(1, int(avail * 0.6) // max(1, bytes_per_block))
    return max(1, min(os.cpu_count() or 1, blocks, by_mem))


def run_blocks(work, emb: int, width: int, rows: int) -> None:
    """Call ``work(c0, c1)`` for column blocks of ``width``; each returns None
    or a failure message. Asserts that none failed."""

    blocks = [(c, min(emb, c + width)) for c in range(0, emb, width)]
    # per block in flight: ~4 float64 arrays of rows x width
    nthreads = threads_for(4 * rows * width * 8, len(blocks))
    with ThreadPoolExecutor(nthreads) as ex:
        fails = [f for f in ex.map(lambda b: work(*b), blocks) if f]
    assert not fails, "; ".join(fails[:4])


def col64(a: np.ndarray, c0: int, c1: int) -> np.ndarray:
    return np.ascontiguousarray(a[:, c0:c1], dtype=np.float64)


def sum_violations(got: np.ndarray, ref: np.ndarray, scale: np.ndarray, rtol: float, atol: float) -> str | None:
    """|got - ref| <= atol + rtol * max(|ref|, scale), scale = the row's sum of |terms|."""

    got = got.astype(np.float64)
    err = np.abs(got - ref)
    bound = atol + rtol * np.maximum(np.abs(ref), scale)
    bad = ~(err <= bound)
    if bad.any():
        return f"{int(bad.sum())} elements out of tolerance, worst excess {float((err - bound)[bad].max()):.3g}"
    return None


def close_violations(got: np.ndarray, ref: np.ndarray, rtol: float, atol: float) -> str | None:
    """allclose with matching infinities and NaN == NaN."""

    got = got.astype(np.float64)
    same_inf = np.isinf(ref) & (got == ref)
    both_nan = np.isnan(ref) & np.isnan(got)
    with np.errstate(invalid="ignore"):  # inf - inf at the matching infinities
        err = np.abs(got - ref)
        ok = same_inf | both_nan | (err <= atol + rtol * np.abs(ref))
    if not ok.all():
        return f"{int((~ok).sum())} elements out of tolerance"
    return None
