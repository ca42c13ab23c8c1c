"""Generate the golden fixtures by running the REFERENCE's own Python ops.

Run in the build container, where the reference checkout is readable:

    python tests/golden/make_golden.py --reference-src DIR

DIR is the reference checkout's ``src`` directory (or set
``VOYAGER_REFERENCE_SRC``).

It imports ``voyager_compiler.ops`` and ``get_quantization_map`` from the
reference source tree with three shims (the reference's top-level package
``__init__`` pulls in codegen and torchao, torchao is not installed, and the
installed torch rejects ``torch.compile(recompile_limit=...)``):

1. stub package modules ``voyager_compiler`` and
   ``voyager_compiler.quantization`` whose ``__path__`` points at the sources;
2. a stub ``torchao.quantization.pt2e`` with ``FakeQuantizeBase``;
3. ``torch.compile`` replaced by the identity while the ops import (the CPU
   path never runs the compiled function).

Outputs (all under ``tests/golden/``):

* ``tables.npz`` -- exhaustive 65,536-entry tables per dtype (bf16 bits) and
  the int64 index table ``convert_pt2e`` swaps in for ``lut4``;
* ``scale_maps.npz`` -- exhaustive bf16 amax -> block scale maps;
* ``ops_small.npz`` + ``ops_small.json`` -- small seeded op cases with edge
  values (inputs, arguments, reference outputs);
* ``full_checksums.json`` -- sha256 of the reference's outputs on the
  full-size configurations (and of their inputs).
"""

import argparse
import hashlib
import importlib.util
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
# the input generators only (importing the voyager_b200 package would
# register its own quantized_ops namespace before the reference's)
_spec = importlib.util.spec_from_file_location(
    "voyager_b200_synth", os.path.join(ROOT, "voyager-compiler_b200", "voyager_b200", "synth.py"))
synth = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(synth)

TABLE_DTYPES = [
    None, "fp4_e2m1", "fp6_e2m3", "fp6_e3m2", "fp8_e4m3", "fp8_e5m2",
    "fp8_e3m4", "fp7_e4m3", "fp8_e5m3", "fp5_e2m2", "int8", "int4", "int6",
    "uint8", "uint4", "int16", "posit8_1", "posit8_0", "posit8_2", "posit6_1",
    "posit16_1", "lut4", "lut3", "lut4_to_fp8_e4m3", "lut4_to_int8",
]


def load_reference(src):
    sys.path.insert(0, src)
    for name, sub in [
        ("voyager_compiler", "voyager_compiler"),
        ("voyager_compiler.quantization", "voyager_compiler/quantization"),
    ]:
        m = types.ModuleType(name)
        m.__path__ = [os.path.join(src, sub)]
        sys.modules[name] = m
    ta = types.ModuleType("torchao")
    ta.__path__ = []
    taq = types.ModuleType("torchao.quantization")
    taq.__path__ = []
    tap = types.ModuleType("torchao.quantization.pt2e")
    tap.__path__ = []

    class FakeQuantizeBase(torch.nn.Module):
        pass

    tap.FakeQuantizeBase = FakeQuantizeBase
    tap.ObserverOrFakeQuantize = object
    sys.modules.update(
        {"torchao": ta, "torchao.quantization": taq, "torchao.quantization.pt2e": tap}
    )
    orig = torch.compile
    torch.compile = lambda fn=None, **kw: fn
    try:
        import voyager_compiler.ops  # noqa: F401
        from voyager_compiler.quantization.fake_quantize import get_quantization_map
    finally:
        torch.compile = orig
    return get_quantization_map


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float32:
        return t.numpy().copy()
    if t.dtype in (torch.int64, torch.int32):
        return t.numpy().copy()
    raise TypeError(t.dtype)


def to_t(a: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(a).reshape(np.shape(a))  # keep 0-d as 0-d
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(a.copy())


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def edge_values_bf16(rng, n):
    """A bf16 array mixing normals, ties, zeros of both signs, infinities,
    NaN, subnormals and huge values."""
    x = synth.f32_to_bf16_bits(rng.standard_normal(n).astype(np.float32))
    specials = np.array(
        [0x0000, 0x8000, 0x7F80, 0xFF80, 0xFFFF, 0x7FC0, 0x0001, 0x8001,
         0x007F, 0x0080, 0x7F7F, 0xFF7F, 0x3E80, 0xBE80, 0x3FA0, 0xBFA0,
         0x3F20, 0x4020, 0x4060, 0x40A0],
        dtype=np.uint16,
    )
    pos = rng.choice(n, size=min(n // 8, 4 * len(specials)), replace=False)
    x[pos] = specials[np.arange(len(pos)) % len(specials)]
    return x


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("VOYAGER_REFERENCE_SRC"),
                    help="the reference checkout's src directory")
    ap.add_argument("--skip-full", action="store_true")
    ap.add_argument("--schemas-only", action="store_true",
                    help="only record the op schemas (schemas.json)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("give --reference-src (or set VOYAGER_REFERENCE_SRC)")
    torch.set_num_threads(os.cpu_count())
    gqm = load_reference(args.reference_src)
    Q = torch.ops.quantized_ops

    # -- 0. the op schemas, as torch parses the reference's definitions ----
    schemas = {}
    for full in sorted(torch._C._dispatch_get_all_op_names()):
        if not full.startswith("quantized_ops::"):
            continue
        name = full.split("::", 1)[1].split(".", 1)[0]
        schemas[name] = str(getattr(Q, name).default._schema)
    with open(os.path.join(HERE, "schemas.json"), "w") as f:
        json.dump(schemas, f, indent=1, sort_keys=True)
    if args.schemas_only:
        return

    # -- 1. tables ---------------------------------------------------------
    tables = {}
    for d in TABLE_DTYPES:
        tables["identity" if d is None else d] = to_np(gqm(d))
    lut4 = gqm("lut4")
    tables["lut4_index"] = to_np(torch.searchsorted(torch.unique(lut4), lut4).to(torch.int64))
    np.savez_compressed(os.path.join(HERE, "tables.npz"), **tables)

    # -- 2. exhaustive scale maps -----------------------------------------
    allb = to_t(np.arange(65536, dtype=np.uint32).astype(np.uint16)).view(65536, 1)
    maps = {}
    for qmax in (6.0, 448.0, 57344.0, 127.0, 7.5, 1.0, 4096.0):
        s = Q.calculate_mx_qparam(allb, [-1], 1, qmax, True)
        maps[f"pow2_bf16_{qmax:g}"] = to_np(s).reshape(-1)
    for qmax, sq in ((6.0, "fp8_e4m3"), (448.0, None), (6.0, None), (1.0, None),
                     (6.0, "fp8_e5m2"), (127.0, "int8")):
        s = Q.calculate_mx_qparam(allb, [-1], 1, qmax, False,
                                  None if sq is None else gqm(sq))
        maps[f"amax_bf16_{qmax:g}_{sq}"] = to_np(s).reshape(-1)
    # float32 inputs: every bf16-exact value plus neighbours around each
    # power of two (where log2 rounding decides the exponent).
    rng = np.random.Generator(np.random.PCG64(7))
    e = np.arange(-149, 128)
    near = []
    for k in e:
        p = np.float32(2.0 ** float(k)) if k > -150 else np.float32(0)
        if not np.isfinite(p) or p == 0:
            continue
        u = np.array([p], dtype=np.float32).view(np.uint32)[0]
        u = int(u)
        near += [u - 3, u - 2, u - 1, u, u + 1, u + 2]
    near = np.array(near, dtype=np.int64)
    near = near[(near >= 0) & (near < 0x7F800000)].astype(np.uint32)
    rand = rng.integers(0, 0x7F800000, size=20000, dtype=np.uint32)
    f32 = np.concatenate([near, rand, np.array([0, 0x7F800000, 0x7FC00000], np.uint32)])
    f32v = f32.view(np.float32)
    maps["f32_inputs"] = f32v
    xt = torch.from_numpy(f32v.copy()).view(-1, 1)
    for qmax in (448.0, 6.0, 1.0):
        maps[f"pow2_f32_{qmax:g}"] = to_np(Q.calculate_mx_qparam(xt, [-1], 1, qmax, True)).reshape(-1)
        maps[f"amax_f32_{qmax:g}"] = to_np(Q.calculate_mx_qparam(xt, [-1], 1, qmax, False)).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "scale_maps.npz"), **maps)

    # -- 3. small op cases -------------------------------------------------
    cases, arrays = [], {}

    def add(name, op, inputs, kwargs, outputs):
        idx = len(cases)
        entry = {"name": name, "op": op, "inputs": [], "kwargs": {}, "outputs": []}
        for i, a in enumerate(inputs):
            key = f"c{idx}_in{i}"
            if a is None:
                entry["inputs"].append(None)
            else:
                arrays[key] = a
                entry["inputs"].append(key)
        for k, v in kwargs.items():
            if isinstance(v, np.ndarray):
                key = f"c{idx}_kw_{k}"
                arrays[key] = v
                entry["kwargs"][k] = {"array": key}
            elif isinstance(v, str) and v.startswith("table:"):
                entry["kwargs"][k] = {"table": v[6:]}
            else:
                entry["kwargs"][k] = v
        for i, o in enumerate(outputs):
            key = f"c{idx}_out{i}"
            arrays[key] = to_np(o)
            entry["outputs"].append(key)
        cases.append(entry)

    def tbl(spec):
        if spec is None:
            return None
        if spec == "lut4_index":
            return torch.from_numpy(tables["lut4_index"])
        return gqm(None if spec == "identity" else spec)

    def run(name, op, inputs, **kw):
        tin = [None if a is None else to_t(a) for a in inputs]
        tkw = {}
        for k, v in kw.items():
            if isinstance(v, np.ndarray):
                tkw[k] = to_t(v)
            elif isinstance(v, str) and v.startswith("table:"):
                tkw[k] = tbl(v[6:])
            else:
                tkw[k] = v
        fn = getattr(Q, op)
        out = fn(*tin, **tkw)
        outs = list(out) if isinstance(out, (tuple, list)) else [out]
        add(name, op, inputs, kw, outs)

    rng = np.random.Generator(np.random.PCG64(123))
    xb = edge_values_bf16(rng, 64 * 128).reshape(64, 128)
    for qd, qmax, sq, bs, pow2 in [
        ("fp4_e2m1", 6.0, "fp8_e4m3", 16, False),
        ("fp8_e4m3", 448.0, None, 32, True),
        ("fp8_e5m2", 57344.0, None, 32, True),
        ("fp4_e2m1", 6.0, None, 32, True),
        ("int8", 127.0, None, 32, False),
        ("posit8_1", 4096.0, None, 16, False),
        ("lut4", 1.0, None, 64, False),
        ("fp6_e2m3", 7.5, "fp8_e4m3", 16, False),
        ("fp8_e4m3", 448.0, "fp8_e5m2", 8, False),
    ]:
        run(f"qmx_bf16_{qd}_{bs}_{pow2}_{sq}", "quantize_mx", [xb],
            qmap=f"table:{qd}", axes=[-1], block_size=bs, quant_max=qmax,
            force_scale_power_of_two=pow2,
            scale_qmap=None if sq is None else f"table:{sq}")
    # ragged last block and short rows
    xr = edge_values_bf16(rng, 33 * 50).reshape(33, 50)
    run("qmx_ragged_nvfp4", "quantize_mx", [xr], qmap="table:fp4_e2m1", axes=[-1],
        block_size=16, quant_max=6.0, force_scale_power_of_two=False,
        scale_qmap="table:fp8_e4m3")
    run("qmx_ragged_mxfp8", "quantize_mx", [xr], qmap="table:fp8_e4m3", axes=[-1],
        block_size=32, quant_max=448.0, force_scale_power_of_two=True)
    xs = edge_values_bf16(rng, 7 * 5).reshape(7, 5)
    run("qmx_short_rows", "quantize_mx", [xs], qmap="table:fp4_e2m1", axes=[-1],
        block_size=16, quant_max=6.0, force_scale_power_of_two=False,
        scale_qmap="table:fp8_e4m3")
    # blocks along a non-last axis, 3-D, 2-D blocks
    x3 = edge_values_bf16(rng, 2 * 64 * 24).reshape(2, 64, 24)
    run("qmx_axis_m2", "quantize_mx", [x3], qmap="table:fp8_e4m3", axes=[-2],
        block_size=32, quant_max=448.0, force_scale_power_of_two=True)
    run("qmx_3d_last", "quantize_mx", [x3], qmap="table:fp4_e2m1", axes=[-1],
        block_size=8, quant_max=6.0, force_scale_power_of_two=False,
        scale_qmap="table:fp8_e4m3")
    run("qmx_2d_blocks", "quantize_mx", [x3], qmap="table:int8", axes=[-2, -1],
        block_size=8, quant_max=127.0, force_scale_power_of_two=False)
    # float32 inputs (C2 shapes in miniature)
    wf = (rng.standard_normal((48, 256)) * 0.02).astype(np.float32)
    wf.reshape(-1)[:6] = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-42]
    run("qmx_f32_nf4_index", "quantize_mx", [wf], qmap="table:lut4_index",
        axes=[-1], block_size=64, quant_max=1.0, force_scale_power_of_two=False)
    run("qmx_f32_nf4_value", "quantize_mx", [wf], qmap="table:lut4",
        axes=[-1], block_size=64, quant_max=1.0, force_scale_power_of_two=False)
    run("qmx_f32_mxfp8", "quantize_mx", [wf], qmap="table:fp8_e4m3",
        axes=[-1], block_size=32, quant_max=448.0, force_scale_power_of_two=True)
    wc = np.abs(wf[np.isfinite(wf)]).max()
    s0 = np.array(wc / 4096.0, dtype=np.float32).reshape(())
    run("q_f32_posit8_per_tensor", "quantize", [wf, s0], qmap="table:posit8_1")
    sc = (np.nanmax(np.where(np.isfinite(wf), np.abs(wf), 0), axis=1, keepdims=True)
          / np.float32(127.0)).astype(np.float32)
    sc[sc == 0] = 1.0
    run("q_f32_int8_per_channel", "quantize", [wf, sc], qmap="table:int8")
    run("q_bf16_scalar_f32", "quantize", [xb, np.array(0.0123456, np.float32).reshape(())],
        qmap="table:fp8_e4m3")
    run("q_bf16_one_elem_f32", "quantize", [xb, np.array([0.0123456], np.float32)],
        qmap="table:fp8_e4m3")
    run("q_f32_scalar_bf16", "quantize", [wf, synth.f32_to_bf16_bits(np.array([0.00123], np.float32)).reshape(())],
        qmap="table:int8")
    sb = synth.f32_to_bf16_bits((np.abs(rng.standard_normal((64, 1))) + 0.1).astype(np.float32))
    run("q_bf16_per_channel_bf16", "quantize", [xb, sb], qmap="table:int8")
    sf = (np.abs(rng.standard_normal((64, 1))) + 0.1).astype(np.float32)
    run("q_bf16_per_channel_f32", "quantize", [xb, sf], qmap="table:fp4_e2m1")
    zp = synth.f32_to_bf16_bits(np.round(rng.standard_normal((64, 1)) * 3).astype(np.float32))
    run("q_bf16_zero_point", "quantize", [xb, sb, zp], qmap="table:uint8")
    s_blk = synth.f32_to_bf16_bits((np.abs(rng.standard_normal((64, 8))) + 0.05).astype(np.float32))
    run("q_bf16_blocks", "quantize", [xb, s_blk], axes=[-1], block_size=16,
        qmap="table:fp4_e2m1")
    run("q_bf16_identity", "quantize", [xb, sb], qmap="table:identity")
    # dequantize
    s_mx, c_mx = Q.quantize_mx(to_t(xb), gqm("fp4_e2m1"), [-1], 16, 6.0, False, gqm("fp8_e4m3"))
    run("dq_nvfp4", "dequantize", [to_np(c_mx), to_np(s_mx)], axes=[-1], block_size=16)
    s_r, c_r = Q.quantize_mx(to_t(xr), gqm("fp4_e2m1"), [-1], 16, 6.0, False, gqm("fp8_e4m3"))
    run("dq_ragged", "dequantize", [to_np(c_r), to_np(s_r)], axes=[-1], block_size=16)
    run("dq_per_channel_zp", "dequantize", [xb, sb, zp])
    run("dq_qmaps", "dequantize", [xb, sb], input_qmap="table:int8",
        output_qmap="table:fp8_e4m3")
    run("dq_f32_scalar", "dequantize", [wf, s0])
    # calculate_mx_qparam alone
    run("mxq_bf16_nvfp4", "calculate_mx_qparam", [xb], axes=[-1], block_size=16,
        quant_max=6.0, force_scale_power_of_two=False, scale_qmap="table:fp8_e4m3")
    run("mxq_f32_pow2", "calculate_mx_qparam", [wf], axes=[-1], block_size=32,
        quant_max=448.0, force_scale_power_of_two=True)
    # vmap
    run("vmap_bf16_e2m1", "vmap", [xb, tables["fp4_e2m1"]])
    # quantize_affine (group-wise affine)
    run("qaffine_bf16_uint4", "quantize_affine", [xb], qmap="table:uint4", axes=[-1],
        block_size=32, quant_min=0.0, quant_max=15.0)
    run("qaffine_f32_int8", "quantize_affine", [wf], qmap="table:uint8", axes=[-1],
        block_size=64, quant_min=0.0, quant_max=255.0)
    # GEMMs (reference output is its bf16 GEMM)
    a = synth.f32_to_bf16_bits(rng.standard_normal((32, 128)).astype(np.float32))
    w = synth.f32_to_bf16_bits((rng.standard_normal((48, 128)) * 0.02).astype(np.float32))
    sa, ca = Q.quantize_mx(to_t(a), gqm("fp8_e4m3"), [-1], 32, 448.0, True)
    sw, cw = Q.quantize_mx(to_t(w), gqm("fp8_e4m3"), [-1], 32, 448.0, True)
    run("linear_mxfp8", "linear_mx", [to_np(ca), to_np(cw), None],
        input_scale=to_np(sa), weight_scale=to_np(sw), block_size=32)
    bias = synth.f32_to_bf16_bits(rng.standard_normal(48).astype(np.float32))
    run("linear_mxfp8_bias", "linear_mx", [to_np(ca), to_np(cw), bias],
        input_scale=to_np(sa), weight_scale=to_np(sw), block_size=32)
    cwt = np.ascontiguousarray(to_np(cw).T)
    swt = np.ascontiguousarray(to_np(sw).T)
    run("matmul_mxfp8_ck", "matmul_mx", [to_np(ca), cwt],
        input_scale=to_np(sa), weight_scale=swt, block_size=32)

    # fused-attention op (sdpa_mx): MXFP8 q / k (blocks along head_dim),
    # v (blocks along the keys), probabilities quantized to MXFP8
    def mx_operand(shape, axis, sd=1.0):
        x = synth.f32_to_bf16_bits((rng.standard_normal(shape) * sd).astype(np.float32))
        s, c = Q.quantize_mx(to_t(x), gqm("fp8_e4m3"), [axis], 32, 448.0, True)
        return to_np(c), to_np(s)

    for name, (B, H, HKV, S, causal) in {
        "sdpa_mxfp8_causal": (1, 2, 2, 256, True),
        "sdpa_mxfp8_full": (1, 2, 2, 128, False),
        "sdpa_mxfp8_gqa_causal": (1, 4, 2, 128, True),
    }.items():
        cq, sq_ = mx_operand((B, H, S, 128), -1, 2.0)
        ck, sk = mx_operand((B, HKV, S, 128), -1, 2.0)
        cv, sv = mx_operand((B, HKV, S, 128), -2)
        run(name, "sdpa_mx", [cq, ck, cv], is_causal=causal, enable_gqa=HKV != H,
            query_scale=sq_, key_scale=sk, value_scale=sv, block_size=32,
            probs_qmap="table:fp8_e4m3", probs_quant_max=448.0,
            force_scale_power_of_two=True)

    # outlier CSR side-stream: filter_outlier, quantize_mx_outlier,
    # slice_csr_tensor, spmm_csr and linear_mx / matmul_mx with A_data
    def spiky(shape, frac=0.02, mult=50.0, sd=1.0):
        x = (rng.standard_normal(shape) * sd).astype(np.float32)
        n = x.size
        pos = rng.choice(n, size=max(1, int(n * frac)), replace=False)
        x.reshape(-1)[pos] *= mult
        return x

    def bf(x):
        return synth.f32_to_bf16_bits(x.astype(np.float32))

    xo = bf(spiky((2, 3, 40, 64)))
    xo.reshape(-1)[:16] = [0x0000, 0x8000, 0x7F80, 0xFF80, 0x7FC0, 0xFFFF, 0x4270, 0xC270,
                           0x406D, 0xC06D, 0x406E, 0x0001, 0x8001, 0x7F7F, 0xFF7F, 0x3F80]
    run("filter_outlier_bf16_batched", "filter_outlier", [xo], threshold=3.7, max_pct=0.05)
    run("filter_outlier_overflow", "filter_outlier", [bf(spiky((64, 128)))], threshold=0.5,
        max_pct=0.01)
    xf = spiky((33, 70))
    xf.reshape(-1)[:8] = [0.0, -0.0, np.inf, -np.inf, np.nan, 2.0, -2.0, 2.0000002]
    run("filter_outlier_f32_ragged", "filter_outlier", [xf], threshold=2.0, max_pct=0.1)
    xz = bf(spiky((8, 24)))
    xz.reshape(-1)[:6] = [0x0000, 0x8000, 0x0000, 0x7FC0, 0x3F80, 0xBF80]
    run("filter_outlier_negative_threshold", "filter_outlier", [xz], threshold=-1.0,
        max_pct=1.0)
    run("filter_outlier_empty_stream", "filter_outlier", [bf(spiky((4, 16)))], threshold=1e9,
        max_pct=0.0)

    xn = bf(spiky((64, 256), frac=0.01))
    run("quantize_mx_outlier_nvfp4", "quantize_mx_outlier", [xn],
        qmap="table:fp4_e2m1", axes=[-1], block_size=16, quant_max=6.0, force_scale_power_of_two=False,
        scale_qmap="table:fp8_e4m3", threshold=6.0, max_pct=0.02)
    run("quantize_mx_outlier_mxfp8_offset", "quantize_mx_outlier",
        [bf(spiky((3, 64, 128), frac=0.01))], qmap="table:fp8_e4m3", axes=[-1], block_size=32,
        quant_max=448.0, force_scale_power_of_two=True, threshold=3.0, max_pct=0.01,
        indptr_offset=7)
    run("quantize_mx_outlier_int8_axis0", "quantize_mx_outlier",
        [bf(spiky((64, 48)))], qmap="table:int8", axes=[-2], block_size=32, quant_max=127.0,
        threshold=2.5, max_pct=0.05)
    run("quantize_mx_outlier_f32", "quantize_mx_outlier",
        [spiky((32, 96))], qmap="table:fp8_e4m3", axes=[-1], block_size=32, quant_max=448.0,
        force_scale_power_of_two=True, threshold=4.0, max_pct=0.03)

    d0, i0, p0, _ = (to_np(t) for t in Q.filter_outlier(to_t(xn), 2.0, 0.05))
    run("slice_csr_rows", "slice_csr_tensor", [d0, i0, p0], dim=0, start=8, end=40)
    run("slice_csr_rows_truncated", "slice_csr_tensor", [d0, i0, p0], dim=0, start=0,
        end=64, size_factor=0.5)
    run("slice_csr_cols", "slice_csr_tensor", [d0, i0, p0], dim=1, start=32, end=96,
        size_factor=0.5)
    run("slice_csr_cols_neg_dim_truncated", "slice_csr_tensor", [d0, i0, p0], dim=-1,
        start=100, end=256, size_factor=0.25)

    # spmm_csr: KC weight with MXFP8 codes and block scales; CK batched B;
    # codebook-decoded B
    xa = bf(spiky((48, 256), frac=0.03))
    da, ia, pa, _ = (to_np(t) for t in Q.filter_outlier(to_t(xa), 3.0, 0.05))
    wkc = bf(rng.standard_normal((96, 256)) * 0.05)
    sw_, cw_ = Q.quantize_mx(to_t(wkc), gqm("fp8_e4m3"), [-1], 32, 448.0, True)
    run("spmm_csr_kc_mxfp8", "spmm_csr", [da, ia, pa, to_np(cw_)], B_scale=to_np(sw_),
        block_size=32, weight_layout="kc")
    xb3 = bf(spiky((2, 32, 64), frac=0.05))
    db, ib, pb, _ = (to_np(t) for t in Q.filter_outlier(to_t(xb3), 2.5, 0.1))
    run("spmm_csr_ck_batched", "spmm_csr", [db, ib, pb, bf(rng.standard_normal((2, 64, 40)))],
        weight_layout="ck")
    code = bf(np.linspace(-1.0, 1.0, 16).astype(np.float32))
    bidx = bf(rng.integers(0, 16, size=(256, 24)).astype(np.float32))
    run("spmm_csr_ck_codebook", "spmm_csr", [da, ia, pa, bidx], B_code=code,
        weight_layout="ck")
    run("spmm_csr_f32_B", "spmm_csr", [da, ia, pa, rng.standard_normal((24, 256)).astype(
        np.float32)], weight_layout="kc")

    # the GEMMs with the side-stream
    a_d, a_i, a_p, a_s, a_c = (to_np(t) for t in Q.quantize_mx_outlier(
        to_t(bf(spiky((128, 256), frac=0.01))), gqm("fp8_e4m3"), [-1], 32, 448.0, True,
        None, None, 4.0, 0.02))
    run("linear_mx_outlier_mxfp8", "linear_mx", [a_c, to_np(cw_)], input_scale=a_s,
        weight_scale=to_np(sw_), block_size=32, A_data=a_d, A_indices=a_i, A_indptr=a_p)
    wck = np.ascontiguousarray(to_np(cw_).T)
    swck = np.ascontiguousarray(to_np(sw_).T)
    sck, cck = Q.quantize_mx(to_t(np.ascontiguousarray(wkc.T)), gqm("fp8_e4m3"), [-2], 32,
                             448.0, True)
    run("matmul_mx_outlier_ck", "matmul_mx", [a_c, to_np(cck)], input_scale=a_s,
        weight_scale=to_np(sck), block_size=32, A_data=a_d, A_indices=a_i, A_indptr=a_p)

    # codebooks: region grids ([*counts, k], one table per region) and the
    # midpoint rounding of a bfloat16 codebook
    def levels(shape):
        v = np.sort(rng.standard_normal(shape).astype(np.float32), axis=-1)
        return v

    xq = bf(rng.standard_normal((2, 4, 8, 32)))
    half = np.array(0.5, dtype=np.float32)
    run("quantize_region_per_head_f32", "quantize", [xq, half], qmap=levels((1, 4, 1, 1, 16)))
    cbb = bf(levels((1, 4, 1, 1, 16)))
    cbt = to_t(cbb)
    bnd = to_np((cbt[..., :-1] + cbt[..., 1:]) / 2)
    run("quantize_region_per_head_bf16_index", "quantize", [xq, half], qmap=cbb,
        output_code=bnd)
    run("quantize_region_per_head_bf16", "quantize", [xq, half], qmap=cbb)
    xg = rng.standard_normal((8, 64)).astype(np.float32)
    sg = (np.abs(xg).max(axis=1, keepdims=True) / np.float32(2)).astype(np.float32)
    run("quantize_region_channel_groups", "quantize", [xg, sg], qmap=levels((1, 4, 8)))
    tie_cb = bf(np.array([-2.0, -1.0, 0.0, 1.0, 1.0234375, 1.5, 2.0], dtype=np.float32))
    xt = bf(np.concatenate([np.array([1.015625, 1.0078125, 1.01171875, -1.5, 1.25, 1.2578125],
                                     dtype=np.float32), rng.standard_normal(58).astype(np.float32)
                            ]).reshape(8, 8))
    run("quantize_codebook_bf16_midpoint_tie", "quantize", [xt, np.array(1.0, dtype=np.float32)],
        qmap=tie_cb)
    idx_a = bf(rng.integers(0, 16, size=(1, 2, 16, 32)).astype(np.float32))
    other = bf(rng.standard_normal((1, 2, 32, 16)) * 0.1)
    run("matmul_mx_region_code", "matmul_mx", [idx_a, other],
        input_code=bf(levels((1, 2, 1, 1, 16))))
    idx_w = bf(rng.integers(0, 8, size=(24, 64)).astype(np.float32))
    xa = bf(rng.standard_normal((16, 64)))
    run("linear_mx_region_weight_code", "linear_mx", [xa, idx_w],
        weight_code=levels((4, 1, 8)))

    np.savez_compressed(os.path.join(HERE, "ops_small.npz"), **arrays)
    with open(os.path.join(HERE, "ops_small.json"), "w") as f:
        json.dump(cases, f, indent=1)

    if args.skip_full:
        return

    # -- 4. full-size checksums --------------------------------------------
    sums = {"torch": torch.__version__, "numpy": np.__version__}
    x1 = synth.c1_input()
    sums["c1_input"] = sha(x1)
    s1, c1 = Q.quantize_mx(to_t(x1), gqm("fp4_e2m1"), [-1], 16, 6.0, False, gqm("fp8_e4m3"))
    d1 = Q.dequantize(c1, s1, None, [-1], 16)
    sums["c1_scale"], sums["c1_codes"], sums["c1_deq"] = sha(to_np(s1)), sha(to_np(c1)), sha(to_np(d1))
    w2 = synth.c2_weight()
    sums["c2_input"] = sha(w2)
    wt = torch.from_numpy(w2)
    s_nf, c_nf = Q.quantize_mx(wt, torch.from_numpy(tables["lut4_index"]), [-1], 64, 1.0, False)
    sums["c2_nf4_scale"], sums["c2_nf4_codes"] = sha(to_np(s_nf)), sha(to_np(c_nf))
    s_p = (wt.abs().amax() / 4096.0)
    sums["c2_posit8_scale"] = sha(to_np(s_p))
    sums["c2_posit8_codes"] = sha(to_np(Q.quantize(wt, s_p, qmap=gqm("posit8_1"))))
    s_i = wt.abs().amax(dim=1, keepdim=True) / 127.0
    sums["c2_int8_scale"] = sha(to_np(s_i))
    sums["c2_int8_codes"] = sha(to_np(Q.quantize(wt, s_i, qmap=gqm("int8"))))
    a3, w3 = synth.c3_operands()
    sums["c3_a_input"], sums["c3_w_input"] = sha(a3), sha(w3)
    for tag, arr in (("c3_a", a3), ("c3_w", w3)):
        s, c = Q.quantize_mx(to_t(arr), gqm("fp8_e4m3"), [-1], 32, 448.0, True)
        sums[f"{tag}_scale"], sums[f"{tag}_codes"] = sha(to_np(s)), sha(to_np(c))
    with open(os.path.join(HERE, "full_checksums.json"), "w") as f:
        json.dump(sums, f, indent=1)


if __name__ == "__main__":
    main()
