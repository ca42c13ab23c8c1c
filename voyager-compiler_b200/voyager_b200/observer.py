"""Per-tensor and per-channel amax observation on the device.

``FusedAmaxObsFakeQuantize`` mirrors the reference module of the same name
(``src/voyager_compiler/quantization/fake_quantize.py:440-537``): the same
constructor arguments, buffers (``scale``, ``amax_history``, the
``fake_quant_enabled`` / ``observer_enabled`` flags), lazy sizing on the
first input, and ``forward`` = observe, then fake-quantize against the
scale.  The observer step ``_update_amax_scale`` (``:494-527``) runs as
``vq_amax_observe`` (an amax reduction and a one-thread-per-channel history
and scale update); the fake quantization is this library's ``quantize``
followed by ``dequantize``, which is the reference's ``_fake_quant``
(``:121-133``: ``vmap(input / scale, qmap) * scale`` with the scale cast to
the input's dtype).  CUDA tensors only: there is no CPU path.
"""

import ctypes
from typing import Optional, Tuple

import torch

from voyager_b200 import ops
from voyager_b200.tables import get_quantization_map

PER_TENSOR_SYMMETRIC = "per_tensor_symmetric"
PER_CHANNEL_SYMMETRIC = "per_channel_symmetric"


def _scheme_name(qscheme) -> str:
    """The reference's ``QScheme`` member, its value string, or that string."""
    return str(getattr(qscheme, "value", qscheme))


def update_amax_scale(x: torch.Tensor, amax_history: torch.Tensor, scale: torch.Tensor,
                      quant_max: float, *, per_channel: bool, ch_axis: Optional[int] = None,
                      power_of_two: bool = False, reset: bool = False) -> None:
    """One observer step in place on ``amax_history`` [L, *C] and ``scale``
    [*C] (float32, on x's device, contiguous): ``_update_amax_scale``
    (``fake_quantize.py:494-527``) without the lazy sizing, which ``reset``
    stands for (history zero, scale one before the step)."""
    ops._check_cuda(x, "amax_observe")
    if amax_history.dtype != torch.float32 or scale.dtype != torch.float32:
        raise TypeError("amax_history and scale are float32")
    if not (amax_history.is_contiguous() and scale.is_contiguous()):
        raise ValueError("amax_history and scale must be contiguous")
    x = x.contiguous()
    axis = 0
    if per_channel:
        axis = ch_axis % x.ndim  # ZeroDivisionError on a 0-d input, as the reference
        channels = x.shape[axis]
    else:
        channels = 1
    if scale.numel() != channels or amax_history.numel() % max(channels, 1):
        raise ValueError(f"scale holds {scale.numel()} values for {channels} channels")
    length = amax_history.numel() // max(channels, 1)
    ws = torch.empty(max(channels, 1), dtype=torch.float32, device=x.device)
    st = ops.lib().vq_amax_observe(
        ctypes.byref(ops._vt(x)), 1 if per_channel else 0, axis, amax_history.data_ptr(), length,
        scale.data_ptr(), float(quant_max), 1 if power_of_two else 0, 1 if reset else 0,
        ws.data_ptr(), ops._stream(x.device))
    if st != 0:
        if x.numel() == 0:
            raise RuntimeError("amax(): the reduction of an empty tensor has no identity")
        raise RuntimeError(f"vq_amax_observe: {ops._lib.STATUS.get(st, st)}")


def fake_quant(input: torch.Tensor, qmap: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """``_fake_quant`` (``fake_quantize.py:121-133``): the scale cast to the
    input's dtype, then quantize and dequantize on this library's kernels."""
    scale = scale.to(input.dtype)
    codes = ops.quantize(input, scale, qmap=qmap)
    return ops.dequantize(codes, scale)


class FusedAmaxObsFakeQuantize(torch.nn.Module):
    """Fake-quantize against a scale observed from recent amaxes
    (``fake_quantize.py:440-537``)."""

    _lazily_sized = ("scale", "amax_history")

    def __init__(self, dtype: str, qscheme, quant_max: float, amax_history_len: int,
                 ch_axis: Optional[int] = None, force_scale_power_of_two: bool = False,
                 device=None, **unused) -> None:
        super().__init__()
        scheme = _scheme_name(qscheme)
        if scheme not in (PER_TENSOR_SYMMETRIC, PER_CHANNEL_SYMMETRIC):
            raise ValueError(f"{qscheme} is not fake-quantized by FusedAmaxObsFakeQuantize")
        self.dtype = dtype
        self.qscheme = qscheme
        self.quant_max = quant_max
        self.amax_history_len = amax_history_len
        self.ch_axis = ch_axis
        self.force_scale_power_of_two = force_scale_power_of_two
        self.is_per_channel = scheme == PER_CHANNEL_SYMMETRIC
        fk = {"device": device, "dtype": torch.float}
        self.register_buffer("fake_quant_enabled", torch.tensor([1], dtype=torch.uint8, device=device))
        self.register_buffer("observer_enabled", torch.tensor([1], dtype=torch.uint8, device=device))
        self.register_buffer("qmap", get_quantization_map(dtype, device), persistent=False)
        self.register_buffer("scale", torch.tensor([1.0], **fk))
        self.register_buffer("amax_history", torch.tensor([], **fk))
        self._frozen_flags: Optional[Tuple[bool, bool]] = None

    # -- the flags of torch's FakeQuantizeBase and the reference's freezing --
    def enable_fake_quant(self, enabled: bool = True) -> None:
        self.fake_quant_enabled[0] = 1 if enabled else 0

    def disable_fake_quant(self) -> None:
        self.enable_fake_quant(False)

    def enable_observer(self, enabled: bool = True) -> None:
        self.observer_enabled[0] = 1 if enabled else 0

    def disable_observer(self) -> None:
        self.enable_observer(False)

    def freeze_flags(self) -> None:
        self._frozen_flags = (bool(self.fake_quant_enabled[0]), bool(self.observer_enabled[0]))

    def fake_quant_on(self) -> bool:
        if self._frozen_flags is not None:
            return self._frozen_flags[0]
        return bool(self.fake_quant_enabled[0])

    def observer_on(self) -> bool:
        if self._frozen_flags is not None:
            return self._frozen_flags[1]
        return bool(self.observer_enabled[0])

    @torch.no_grad()
    def _update_amax_scale(self, x: torch.Tensor) -> None:
        """Fold ``x``'s amax into the history and recompute ``scale``
        (``fake_quantize.py:494-527``); the history and the scale take their
        shape from the first input."""
        if self.is_per_channel:
            axis = self.ch_axis % x.ndim
            shape = tuple(s if i == axis else 1 for i, s in enumerate(x.shape))
        else:
            shape = ()
        reset = self.amax_history.numel() == 0
        if reset:
            self.amax_history.resize_((self.amax_history_len,) + shape)
            self.scale.resize_(shape)
        update_amax_scale(x, self.amax_history, self.scale, self.quant_max,
                          per_channel=self.is_per_channel, ch_axis=self.ch_axis,
                          power_of_two=self.force_scale_power_of_two, reset=reset)

    def calculate_qparams(self):
        return self.scale

    def extra_repr(self):
        return (f"fake_quant_enabled={self.fake_quant_enabled}, "
                f"observer_enabled={self.observer_enabled}, dtype={self.dtype}, "
                f"qscheme={self.qscheme}, quant_max={self.quant_max}, ch_axis={self.ch_axis}, "
                f"amax_history_len={self.amax_history_len}, "
                f"force_scale_power_of_two={self.force_scale_power_of_two}")

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        for name in self._lazily_sized:
            key = prefix + name
            if key in state_dict:
                getattr(self, name).resize_(state_dict[key].shape)
            elif strict:
                missing_keys.append(key)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.observer_on():
            self._update_amax_scale(x)
        if not self.fake_quant_on():
            return x
        return fake_quant(x, self.qmap, self.scale)
