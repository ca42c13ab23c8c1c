"""Golden vectors for the amax observer, made by the REFERENCE's own module.

Run in the build container, where the reference checkout is readable:

    python tests/golden/make_observer_golden.py --reference-src DIR

It loads the reference the way ``make_golden.py`` does (same shims), builds
``FusedAmaxObsFakeQuantize`` (``src/voyager_compiler/quantization/
fake_quantize.py:440-537``) for each case and calls its
``_update_amax_scale`` on a seeded sequence of inputs, recording the
history and the scale after every call.  Outputs ``observer.npz`` (inputs
as bf16 bits or float32, histories, scales) and ``observer.json`` (the
cases' arguments).
"""

import argparse
import importlib.util
import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(HERE, "make_golden.py"))
mg = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(mg)


def pow2_edges() -> np.ndarray:
    """Positive float32 values at and next to powers of two, where the
    float32 rounding of log2 decides the ceiling."""
    vals = []
    for e in range(-149, 128):
        for k in list(range(0, 24)) + [2 ** j for j in range(5, 23)]:
            v = np.float32(np.ldexp(np.float64(1 + k * 2.0 ** -23), e))
            if v > 0 and np.isfinite(v):
                vals.append(v)
        for k in (1, 2, 3, 7):
            v = np.float32(np.ldexp(np.float64(2 - k * 2.0 ** -23), e))
            if v > 0 and np.isfinite(v):
                vals.append(v)
    return np.unique(np.array(vals, dtype=np.float32))


CASES = [
    # name, shape, dtype, per_channel, ch_axis, L, quant_max, pow2, calls
    ("tensor_f32", [64, 96], "f32", False, None, 1, 127.0, False, 4),
    ("tensor_bf16_nan_zero", [33, 70], "bf16", False, None, 3, 448.0, True, 6),
    ("chan0_f32", [48, 40], "f32", True, 0, 2, 127.0, False, 4),
    ("chan1_bf16", [20, 37], "bf16", True, 1, 4, 6.0, True, 5),
    ("chanlast_f32", [3, 5, 64], "f32", True, -1, 5, 57344.0, False, 7),
    ("chan1_f32_runs", [4, 6, 40], "f32", True, 1, 3, 15.0, True, 4),
    ("chan1_bf16_odd", [4, 6, 33], "bf16", True, 1, 2, 0.1, False, 4),
    ("tensor_0d", [], "f32", False, None, 2, 7.0, True, 4),
    ("chan0_inf", [16, 24], "f32", True, 0, 3, 127.0, True, 4),
    ("tensor_tiny", [8, 8], "f32", False, None, 1, 3.0, True, 3),
]


def inputs_for(name, shape, dtype, calls, rng):
    xs = []
    for k in range(calls):
        x = (rng.standard_normal(shape) * (2.0 ** rng.integers(-6, 7))).astype(np.float32)
        if name == "tensor_bf16_nan_zero" and k == 2:
            x.reshape(-1)[5] = np.nan
        if name == "tensor_bf16_nan_zero" and k == 3:
            x[...] = 0.0
        if name == "chan0_inf" and k == 1:
            x[3, 7] = np.inf
            x[5, 2] = -np.inf
        if name == "chan0_inf" and k == 2:
            x[9, 0] = np.nan
        if name == "tensor_tiny":
            x = (x * np.float32(2.0 ** -140)).astype(np.float32)  # subnormals
        if dtype == "bf16":
            xs.append(mg.synth.f32_to_bf16_bits(x))
        else:
            xs.append(x)
    return xs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("VOYAGER_REFERENCE_SRC"))
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("give --reference-src (or set VOYAGER_REFERENCE_SRC)")
    mg.load_reference(args.reference_src)
    from voyager_compiler.quantization.fake_quantize import FusedAmaxObsFakeQuantize
    from voyager_compiler.quantization.qspec import QScheme

    rng = np.random.default_rng(20261202)
    out, meta = {}, []
    cases = list(CASES)
    edges = pow2_edges()
    cases.append(("pow2_edges", [int(edges.size), 1], "f32", True, 0, 1, 1.0, True, 2))
    cases.append(("pow2_edges_q", [int(edges.size), 1], "f32", True, 0, 1, 0.1, True, 2))
    for ci, (name, shape, dtype, per_ch, axis, L, qmax, pow2, calls) in enumerate(cases):
        if name.startswith("pow2_edges"):
            xs = [edges.reshape(-1, 1).copy(), edges.reshape(-1, 1).copy()]
        else:
            xs = inputs_for(name, shape, dtype, calls, rng)
        scheme = QScheme.PER_CHANNEL_SYMMETRIC if per_ch else QScheme.PER_TENSOR_SYMMETRIC
        fq = FusedAmaxObsFakeQuantize("int8", scheme, qmax, L, ch_axis=axis,
                                      force_scale_power_of_two=pow2)
        for k, x in enumerate(xs):
            xt = mg.to_t(x)
            fq._update_amax_scale(xt)
            out[f"c{ci}_x{k}"] = x
            out[f"c{ci}_h{k}"] = mg.to_np(fq.amax_history)
            out[f"c{ci}_s{k}"] = mg.to_np(fq.scale)
        meta.append({"name": name, "shape": shape, "dtype": dtype, "per_channel": per_ch,
                     "ch_axis": axis, "history_len": L, "quant_max": qmax, "pow2": pow2,
                     "calls": len(xs)})
    np.savez_compressed(os.path.join(HERE, "observer.npz"), **out)
    with open(os.path.join(HERE, "observer.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(f"{len(meta)} cases, {sum(m['calls'] for m in meta)} calls")


if __name__ == "__main__":
    main()
