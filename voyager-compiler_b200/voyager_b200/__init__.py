"""voyager_b200 -- B200 (sm_100a) kernels for the reference's quantization
numerics hot path (Joejoedesu/voyager-compiler ``quantized_ops``).

``import voyager_b200`` loads ``libvoyager_b200.so`` and registers its CUDA
kernels on the ``quantized_ops`` torch.library ops (see ``voyager_b200.ops``).
"""

from voyager_b200 import _lib
from voyager_b200.tables import get_quantization_map, index_table, rounder_for  # noqa: F401

__all__ = ["get_quantization_map", "index_table", "rounder_for", "ops", "register", "lib",
           "check_errors"]

lib = _lib.load()

from voyager_b200 import ops  # noqa: E402
from voyager_b200.ops import register  # noqa: E402

register()


def check_errors(device=None, clear: bool = True) -> None:
    """Raise ``VqError`` if a tcgen05 or barrier kernel of this library gave
    up a bounded wait on ``device`` (default: the current one) since the
    last check.  Kernels never trap: a wait that runs out records a code and
    the launch ends with an incomplete result, so call this after a batch of
    work (it synchronises the current stream).  ``clear`` resets the word."""
    import ctypes

    import torch

    from voyager_b200.ops import _stream

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    code = ctypes.c_int32(0)
    with torch.cuda.device(dev):
        _lib.check(lib.vq_device_errors(ctypes.byref(code), 1 if clear else 0, _stream(dev)),
                   "vq_device_errors")
    if code.value:
        raise _lib.VqError(f"a bounded device wait gave up on {dev} (code {code.value}): "
                           "the results of that launch are incomplete")
