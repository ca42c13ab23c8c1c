"""voyager_b200 -- B200 (sm_100a) kernels for the reference's quantization
numerics hot path (Joejoedesu/voyager-compiler ``quantized_ops``).

``import voyager_b200`` loads ``libvoyager_b200.so`` and registers its CUDA
kernels on the ``quantized_ops`` torch.library ops (see ``voyager_b200.ops``).
"""

from voyager_b200 import _lib
from voyager_b200.tables import get_quantization_map, index_table, rounder_for  # noqa: F401

__all__ = ["get_quantization_map", "index_table", "rounder_for", "ops", "register", "lib"]

lib = _lib.load()

from voyager_b200 import ops  # noqa: E402
from voyager_b200.ops import register  # noqa: E402

register()
