"""ctypes binding of the C ABI in ``include/voyager_b200.h``.

The shared object is built in-tree (``voyager_b200/libvoyager_b200.so``, see
``voyager_b200.build``).  Loading it needs no GPU; the entry points that
launch kernels need one.  If the library is missing the import fails loudly:
there is no fallback implementation.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libvoyager_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

VQ_MAX_DIMS = 8
VQ_STEP_MAX = 64

# vq_dtype
VQ_BF16, VQ_F32, VQ_F16, VQ_I64, VQ_U8, VQ_I32 = 0, 1, 2, 3, 4, 5
# vq_rounder_kind
VQ_R_IDENTITY, VQ_R_MINIFLOAT, VQ_R_INT, VQ_R_POSIT, VQ_R_STEP, VQ_R_TABLE = range(6)
KIND_NAMES = {0: "identity", 1: "minifloat", 2: "int", 3: "posit", 4: "step", 5: "table"}

STATUS = {
    0: "ok", 1: "invalid argument", 2: "unsupported dtype or layout",
    3: "alignment requirement not met", 4: "CUDA runtime error",
    5: "shapes do not broadcast", 6: "required pointer is NULL",
    7: "bounded device wait timed out", 8: "problem exceeds the fixed scratch area",
}

VQ_NOALLOC_SCRATCH_BYTES = 16 << 20


class VqTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * VQ_MAX_DIMS),
    ]


class VqRounder(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("ebits", ctypes.c_int32),
        ("mbits", ctypes.c_int32),
        ("is_signed", ctypes.c_int32),
        ("min_exp", ctypes.c_int32),
        ("max_norm", ctypes.c_float),
        ("qmin", ctypes.c_float),
        ("qmax", ctypes.c_float),
        ("nbits", ctypes.c_int32),
        ("es", ctypes.c_int32),
        ("nan_bits", ctypes.c_uint32),
        ("nsteps", ctypes.c_int32),
        ("step_keys", ctypes.c_uint16 * VQ_STEP_MAX),
        ("step_vals", ctypes.c_uint16 * (VQ_STEP_MAX + 1)),
        ("pad_", ctypes.c_uint16),
        ("table", ctypes.c_void_p),
        ("hw", ctypes.c_int32),
        ("pad2_", ctypes.c_int32),
        ("table8", ctypes.c_void_p),
        ("palette", ctypes.c_void_p),
    ]

    def describe(self) -> str:
        k = KIND_NAMES.get(self.kind, "?")
        if self.kind == VQ_R_MINIFLOAT:
            hw = {1: ", hw e4m3", 2: ", hw e5m2", 3: ", hw e2m1"}.get(self.hw, "")
            return (f"minifloat(e{self.ebits}m{self.mbits}, "
                    f"{'signed' if self.is_signed else 'unsigned'}, max={self.max_norm:g}{hw})")
        if self.kind == VQ_R_INT:
            return f"int[{self.qmin:g},{self.qmax:g}]"
        if self.kind == VQ_R_POSIT:
            return f"posit({self.nbits},{self.es})"
        if self.kind == VQ_R_STEP:
            return f"step({self.nsteps})"
        return k


P = ctypes.POINTER
_SIGNATURES = {
    "vq_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "vq_version": (ctypes.c_char_p, []),
    "vq_rounder_from_table": (ctypes.c_int, [ctypes.c_void_p, P(VqRounder)]),
    "vq_rounder_eval_host": (ctypes.c_uint16, [P(VqRounder), ctypes.c_uint16]),
    "vq_pow2_scale_host": (ctypes.c_uint32, [ctypes.c_uint32, ctypes.c_int32, ctypes.c_int32]),
    "vq_quantize": (ctypes.c_int, [P(VqTensor), P(VqTensor), P(VqTensor), ctypes.c_int64,
                                   P(VqRounder), P(VqTensor), ctypes.c_void_p]),
    "vq_dequantize": (ctypes.c_int, [P(VqTensor), P(VqTensor), P(VqTensor), ctypes.c_int64,
                                     P(VqRounder), P(VqRounder), P(VqTensor), ctypes.c_void_p]),
    "vq_calculate_mx_qparam": (ctypes.c_int, [P(VqTensor), P(ctypes.c_int64), ctypes.c_int32,
                                              ctypes.c_int64, ctypes.c_float, ctypes.c_int32,
                                              ctypes.c_int32, P(VqRounder), P(VqTensor),
                                              ctypes.c_void_p]),
    "vq_quantize_mx": (ctypes.c_int, [P(VqTensor), P(VqRounder), P(ctypes.c_int64), ctypes.c_int32,
                                      ctypes.c_int64, ctypes.c_float, ctypes.c_int32, ctypes.c_int32,
                                      P(VqRounder), P(VqTensor), P(VqTensor), ctypes.c_void_p]),
    "vq_mx_pack_sizes": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                        P(ctypes.c_int64), P(ctypes.c_int64), P(ctypes.c_int64)]),
    "vq_mx_pack": (ctypes.c_int, [P(VqTensor), P(VqTensor), ctypes.c_int64, ctypes.c_int32,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "vq_gemm_mxf8": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                    ctypes.c_void_p, ctypes.c_void_p]),
    "vq_linear_mxf8_noalloc": (ctypes.c_int, [P(VqTensor), P(VqTensor), ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    "vq_quantize_mx_packed": (ctypes.c_int, [P(VqTensor), P(VqRounder), ctypes.c_int32,
                                             P(VqTensor), P(VqTensor), ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p]),
    "vq_attn_mxf8": (ctypes.c_int, [ctypes.c_void_p] * 6 + [ctypes.c_int64] * 6
                     + [ctypes.c_float, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]
                     + [ctypes.c_int64] * 3 + [ctypes.c_void_p, ctypes.c_void_p]),
    "vq_rmsnorm_quantize_mx": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_float, P(VqRounder),
                                              ctypes.c_int32] + [ctypes.c_void_p] * 5),
    "vq_rope_quantize_qk": (ctypes.c_int, [ctypes.c_void_p] + [ctypes.c_int64] * 3
                            + [ctypes.c_void_p] * 2 + [ctypes.c_int64] * 3
                            + [P(VqRounder), ctypes.c_int32] + [ctypes.c_void_p] * 9),
    "vq_quantize_vt": (ctypes.c_int, [ctypes.c_void_p] + [ctypes.c_int64] * 5
                       + [P(VqRounder), ctypes.c_int32] + [ctypes.c_void_p] * 5),
    "vq_swiglu_quantize_mx": (ctypes.c_int, [ctypes.c_void_p] + [ctypes.c_int64] * 4
                              + [P(VqRounder), ctypes.c_int32] + [ctypes.c_void_p] * 5),
    "vq_gemm_mxf8_ex": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3
                        + [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                           ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]),
    "vq_tp_barrier": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                     ctypes.c_int32, ctypes.c_uint32, ctypes.c_void_p,
                                     ctypes.c_void_p]),
    "vq_mx_pack_batched": (ctypes.c_int, [P(VqTensor), P(VqTensor), ctypes.c_int64,
                                          ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "vq_gemm_mxf8_batched": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 5
                             + [ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                ctypes.c_void_p]),
    "vq_gemm_dq": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_void_p, ctypes.c_void_p]),
    "vq_gemm_dq_ex": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
                                     ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p,
                                     ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                     ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "vq_tp_barrier_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_void_p, ctypes.c_uint64,
                                         ctypes.c_void_p, ctypes.c_void_p]),
    "vq_stream_probe": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                       ctypes.c_int64, ctypes.c_void_p]),
    "vq_gemm_dq_splits": (ctypes.c_int32, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int64]),
    "vq_dq_pack_sizes": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int32, P(ctypes.c_int64), P(ctypes.c_int64)]),
    "vq_dq_pack": (ctypes.c_int, [P(VqTensor), ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_void_p]),
    "vq_dq_pack_scales": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_void_p, ctypes.c_void_p]),
    "vq_dq_patterns": (ctypes.c_int, [P(VqTensor), ctypes.c_void_p, ctypes.c_void_p]),
    "vq_dq_decode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p]),
    "vq_transpose_bf16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
    "vq_nvf4_pack_sizes": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                          P(ctypes.c_int64), P(ctypes.c_int64)]),
    "vq_nvf4_pack": (ctypes.c_int, [P(VqTensor), P(VqTensor), ctypes.c_int32, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "vq_gemm_nvf4": (ctypes.c_int, [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3
                     + [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                        ctypes.c_void_p]),
    "vq_tp_barrier_ex": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64,
                                        ctypes.c_void_p, ctypes.c_void_p]),
    "vq_linear_mxf8_noalloc_status": (ctypes.c_int, [P(ctypes.c_int32), ctypes.c_void_p]),
    "vq_device_errors": (ctypes.c_int, [P(ctypes.c_int32), ctypes.c_int32, ctypes.c_void_p]),
    "vq_tp_copy_multicast": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                            ctypes.c_void_p]),
    "vq_tp_sumsq": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                   ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]),
    "vq_tp_norm_quantize": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                           ctypes.c_void_p, ctypes.c_float, P(VqRounder),
                                           ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_void_p]),
    "vq_tp_quantize": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int64, P(VqRounder), ctypes.c_int32,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]),
    "vq_tp_swiglu_quantize": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_int64, P(VqRounder),
                                             ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_void_p]),
    "vq_w4_packed_bytes": (ctypes.c_int64, [ctypes.c_int64, ctypes.c_int64]),
    "vq_w4_pack_weights": (ctypes.c_int, [P(VqTensor), P(VqTensor), ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p]),
    "vq_w4a8_workspace_bytes": (ctypes.c_int64, [ctypes.c_int64, ctypes.c_int64]),
    "vq_w4a8_linear_small": (ctypes.c_int, [P(VqTensor), P(VqTensor), ctypes.c_void_p,
                                            ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p]),
    "vq_rounder_check_hw": (ctypes.c_int, [P(VqRounder), ctypes.c_void_p, ctypes.c_void_p]),
    "vq_quantize_affine_qparams": (ctypes.c_int, [P(VqTensor), P(ctypes.c_int64), ctypes.c_int32,
                                                  ctypes.c_int64, ctypes.c_float, ctypes.c_float,
                                                  P(VqRounder), P(VqTensor), P(VqTensor),
                                                  ctypes.c_void_p]),
    "vq_amax_observe": (ctypes.c_int, [P(VqTensor), ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                       ctypes.c_float, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_void_p, ctypes.c_void_p]),
    "vq_outlier_threshold_bits": (ctypes.c_uint32, [ctypes.c_double, ctypes.c_int32]),
    "vq_filter_outlier_workspace_bytes": (ctypes.c_size_t, [P(VqTensor)]),
    "vq_filter_outlier": (ctypes.c_int, [P(VqTensor), ctypes.c_double, ctypes.c_int64,
                                         ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]),
    "vq_quantize_mx_masked": (ctypes.c_int, [P(VqTensor), P(VqRounder), ctypes.c_int64,
                                             ctypes.c_float, ctypes.c_int32, ctypes.c_int32,
                                             P(VqRounder), ctypes.c_double, P(VqTensor),
                                             P(VqTensor), ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p]),
    "vq_spmm_csr": (ctypes.c_int, [P(VqTensor), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                   P(VqTensor), P(VqTensor), ctypes.c_void_p, ctypes.c_void_p]),
    "vq_slice_csr": (ctypes.c_int, [P(VqTensor), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                    ctypes.c_int32, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p]),
    "vq_transpose": (ctypes.c_int, [P(VqTensor), P(VqTensor), ctypes.c_void_p]),
    "vq_codebook_lookup": (ctypes.c_int, [P(VqTensor), P(ctypes.c_int64), ctypes.c_int32,
                                          ctypes.c_void_p, ctypes.c_int64, P(VqTensor),
                                          ctypes.c_void_p]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load the library and declare every exported signature."""
    global _lib
    if _lib is not None and path == LIB_PATH:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(the CUDA path has no fallback)"
        )
    lib = ctypes.CDLL(path)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    if path == LIB_PATH:
        _lib = lib
    return lib


def exported_symbols():
    return list(_SIGNATURES)


class VqError(RuntimeError):
    pass


def check(status: int, what: str):
    if status != 0:
        msg = STATUS.get(status, f"status {status}")
        exc = ValueError if status in (1, 2, 3, 5, 6, 8) else VqError
        raise exc(f"{what}: {msg}")
