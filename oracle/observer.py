"""The amax observer of per-tensor / per-channel fake quantization, restated
in numpy.

Test infrastructure only (see ``oracle/__init__.py``).

Follows ``FusedAmaxObsFakeQuantize._update_amax_scale``
(``src/voyager_compiler/quantization/fake_quantize.py:494-527``):

* ``amax_cur`` = max of |x| over every axis (per-tensor) or every axis but
  ``ch_axis`` (per-channel, kept as size-1 dims); NaN propagates;
* the scale is computed from the history BEFORE ``amax_cur`` enters it:
  ``amax = max(history, axis=0)``;
* the history is rolled by -1 along axis 0 and row 0 overwritten with
  ``amax_cur`` (so the old row 1 is dropped and the old row 0 moves last);
* ``sf = amax / quant_max`` in float32 (the Python float rounded to float32
  first, as torch converts a scalar operand to the tensor's dtype), kept
  only where ``amax > 0`` and ``amax`` is finite, else the old scale;
* with ``force_scale_power_of_two``, ``sf = 2 ** ceil(log2(sf))`` with
  ``log2`` correctly rounded to float32 (torch's CPU float32 ``log2`` gives
  the correctly rounded value on every input the tests use, including the
  ones closest to powers of two).

The lazy sizing of the first call (history zeros, scale ones) is the
caller's ``fresh`` flag here.
"""

from typing import Optional, Tuple

import numpy as np


def amax_of(x_f32: np.ndarray, per_channel: bool, ch_axis: Optional[int]) -> np.ndarray:
    """float32 amax of |x| (keepdim for per-channel, 0-d for per-tensor)."""
    a = np.abs(x_f32.astype(np.float32))
    if per_channel:
        axis = ch_axis % a.ndim
        dims = tuple(i for i in range(a.ndim) if i != axis)
        return np.max(a, axis=dims, keepdims=True) if dims else a.copy()
    return np.asarray(np.max(a), dtype=np.float32)


def pow2_ceil(sf: np.ndarray) -> np.ndarray:
    """``torch.pow(2, torch.ceil(torch.log2(sf)))`` on float32."""
    sf = np.asarray(sf, dtype=np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        t = np.ceil(np.log2(sf.astype(np.float64)).astype(np.float32))
        return np.power(np.float64(2.0), t.astype(np.float64)).astype(np.float32)


def update_amax_scale(x_f32: np.ndarray, history: Optional[np.ndarray], scale: np.ndarray,
                      quant_max: float, *, per_channel: bool, ch_axis: Optional[int],
                      history_len: int, power_of_two: bool) -> Tuple[np.ndarray, np.ndarray]:
    """One observer step; returns the new (history, scale).  ``history`` None
    is the first call (lazily sized: zeros, and the scale ones)."""
    cur = amax_of(x_f32, per_channel, ch_axis)
    if history is None:
        history = np.zeros((history_len,) + cur.shape, dtype=np.float32)
        scale = np.ones(cur.shape, dtype=np.float32)
    history = history.astype(np.float32, copy=True)
    scale = np.asarray(scale, dtype=np.float32)
    amax = np.max(history, axis=0)  # NaN propagates, as torch.amax
    history = np.roll(history, -1, axis=0)
    history[0] = cur
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        sf = (amax.astype(np.float32) / np.float32(quant_max)).astype(np.float32)
    keep = (amax > 0) & np.isfinite(amax)
    sf = np.where(keep, sf, scale).astype(np.float32)
    if power_of_two:
        sf = pow2_ceil(sf)
    return history, sf.reshape(cur.shape)
