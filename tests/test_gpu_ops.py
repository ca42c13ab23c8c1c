"""CUDA kernels against the reference's golden outputs and the CPU oracle.

Every case calls the ops through ``torch.ops.quantized_ops`` (the drop-in
boundary), which dispatches to ``libvoyager_b200.so``.  Codes and scales
must be bit-exact (any NaN equals any NaN); GEMMs within rel-L2 1e-3 of the
oracle's dequantize-then-matmul rounded to the output dtype."""

import hashlib
import math

import numpy as np
import pytest
import torch

import _golden as G
import oracle
from _tt import to_dev, to_np
from oracle.numerics import quantization_map

pytestmark = pytest.mark.gpu

Q = None


@pytest.fixture(scope="module", autouse=True)
def _setup():
    global Q
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401  (registers the CUDA kernels)

    Q = torch.ops.quantized_ops
    yield


def _kwargs_dev(kw):
    return {k: (to_dev(v) if isinstance(v, np.ndarray) else v) for k, v in kw.items()}


CASES = G.small_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_golden_case(case):
    ins, kw, outs = G.resolve_case(case)
    fn = getattr(Q, case["op"])
    dins = [to_dev(a) for a in ins]
    r = fn(*dins) if case["op"] == "vmap" else fn(*dins, **_kwargs_dev(kw))
    got = list(r) if isinstance(r, (tuple, list)) else [r]
    assert len(got) == len(outs)
    for g, w in zip(got, outs):
        g = to_np(g)
        assert g.shape == w.shape and g.dtype == w.dtype, (g.shape, w.shape, g.dtype, w.dtype)
        if case["op"] in ("linear_mx", "matmul_mx"):
            want = getattr(oracle, case["op"])(*ins, **kw)
            assert G.rel_l2(g, want) < 1e-3
        elif case["op"] == "sdpa_mx":
            # float32 sums in another order and a hardware exp: the same
            # bound as tests/test_gpu_attention.py, against the reference
            assert G.rel_l2(g, w) < 1e-3
        else:
            bad = G.bit_mismatches(g, w)
            assert len(bad) == 0, f"{len(bad)} mismatches, first at {bad[:5]}"


TABLES = [k for k in G.tables() if k != "lut4_index"]


@pytest.mark.parametrize("name", TABLES)
def test_table_every_pattern(name):
    """quantize of all 65,536 bf16 patterns (scale 1) through each table,
    and quantize_mx / vmap through the same rounder."""
    t = G.tables()[name]
    x = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    one = np.array(1.0, dtype=np.float32).reshape(())
    got = to_np(Q.quantize(to_dev(x), to_dev(one), qmap=to_dev(t)))
    want = oracle.quantize(x, one, qmap=t)
    assert len(G.bit_mismatches(got, want)) == 0
    got_v = to_np(Q.vmap(to_dev(x), to_dev(t)))
    assert len(G.bit_mismatches(got_v, t)) == 0


@pytest.mark.parametrize("qmax", [6.0, 448.0, 57344.0, 127.0, 1.0, 4096.0])
def test_pow2_scale_every_amax(qmax):
    x = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    # fast path: rows of 8 copies, block 8 along the last dim
    xr = np.repeat(x[:, None], 8, axis=1)
    got = to_np(Q.calculate_mx_qparam(to_dev(xr), [-1], 8, qmax, True)).reshape(-1)
    assert len(G.bit_mismatches(got, G.scale_maps()[f"pow2_bf16_{qmax:g}"])) == 0
    # generic path: block 1
    got1 = to_np(Q.calculate_mx_qparam(to_dev(x.reshape(-1, 1)), [-1], 1, qmax, True)).reshape(-1)
    assert len(G.bit_mismatches(got1, G.scale_maps()[f"pow2_bf16_{qmax:g}"])) == 0


def test_pow2_scale_f32_inputs():
    x = G.scale_maps()["f32_inputs"]
    for qmax in (448.0, 6.0, 1.0):
        got = to_np(Q.calculate_mx_qparam(to_dev(x.reshape(-1, 1)), [-1], 1, qmax, True)).reshape(-1)
        assert len(G.bit_mismatches(got, G.scale_maps()[f"pow2_f32_{qmax:g}"])) == 0
        xr = np.ascontiguousarray(np.repeat(x[:, None], 4, axis=1))
        got4 = to_np(Q.calculate_mx_qparam(to_dev(xr), [-1], 4, qmax, True)).reshape(-1)
        assert len(G.bit_mismatches(got4, G.scale_maps()[f"pow2_f32_{qmax:g}"])) == 0


def test_amax_scale_every_amax():
    x = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    xr = np.repeat(x[:, None], 16, axis=1)
    e4m3 = G.tables()["fp8_e4m3"]
    got = to_np(Q.calculate_mx_qparam(to_dev(xr), [-1], 16, 6.0, False, to_dev(e4m3))).reshape(-1)
    assert len(G.bit_mismatches(got, G.scale_maps()["amax_bf16_6_fp8_e4m3"])) == 0


# ---------------------------------------------------------------------------
# seeded random cases against the oracle (shapes, layouts, dtypes)
# ---------------------------------------------------------------------------
def _rand(shape, dtype, seed, std=1.0):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = (rng.standard_normal(shape) * std).astype(np.float32)
    if x.size > 10:
        flat = x.reshape(-1)
        flat[rng.choice(x.size, max(1, x.size // 200), replace=False)] *= 50
    if dtype == "bf16":
        from voyager_b200.synth import f32_to_bf16_bits

        return f32_to_bf16_bits(x)
    return x


MX_SHAPES = [
    ((1, 16), [-1], 16), ((3, 48), [-1], 16), ((17, 1000), [-1], 32), ((5, 7, 64), [-1], 64),
    ((256, 4096), [-1], 16), ((64, 96), [-2], 32), ((2, 64, 40), [-2], 32),
    ((33, 50), [-1], 16), ((9, 5), [-1], 16), ((16, 24), [-2, -1], 8), ((40, 96), [-1], 96),
    ((8, 1024), [-1], 256), ((4, 2048), [-1], 512),
]
FORMATS = [
    ("fp4_e2m1", 6.0, "fp8_e4m3", False), ("fp8_e4m3", 448.0, None, True),
    ("fp8_e5m2", 57344.0, None, True), ("int8", 127.0, None, False),
    ("lut4", 1.0, None, False), ("posit8_1", 4096.0, None, False),
]


@pytest.mark.parametrize("shape,axes,bs", MX_SHAPES)
@pytest.mark.parametrize("fmt", FORMATS, ids=[f[0] for f in FORMATS])
@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_quantize_mx_random(shape, axes, bs, fmt, dtype):
    qd, qmax, sqd, pow2 = fmt
    x = _rand(shape, dtype, seed=hash((shape, bs, qd, dtype)) & 0xFFFF)
    qm = quantization_map(qd)
    sq = None if sqd is None else quantization_map(sqd)
    ws, wc = oracle.quantize_mx(x, qm, axes, bs, qmax, pow2, sq)
    gs, gc = Q.quantize_mx(to_dev(x), to_dev(qm), axes, bs, qmax, pow2,
                           None if sq is None else to_dev(sq))
    assert len(G.bit_mismatches(to_np(gs), ws)) == 0
    assert len(G.bit_mismatches(to_np(gc), wc)) == 0
    # dequantize round trip
    wd = oracle.dequantize(wc, ws, None, axes, bs)
    gd = Q.dequantize(gc, gs, None, axes, bs)
    assert len(G.bit_mismatches(to_np(gd), wd)) == 0


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("sdtype", ["bf16", "fp32"])
@pytest.mark.parametrize("layout", ["scalar0d", "one", "row", "col", "full", "blocks"])
def test_quantize_broadcast(dtype, sdtype, layout):
    x = _rand((24, 64), dtype, seed=5)
    rng = np.random.Generator(np.random.PCG64(9))
    shapes = {"scalar0d": (), "one": (1,), "row": (24, 1), "col": (64,), "full": (24, 64),
              "blocks": (24, 4)}
    s = (np.abs(rng.standard_normal(shapes[layout])) + 0.05).astype(np.float32)
    if sdtype == "bf16":
        from voyager_b200.synth import f32_to_bf16_bits

        s = f32_to_bf16_bits(s).reshape(shapes[layout])
    bs = 16 if layout == "blocks" else None
    qm = quantization_map("int8")
    want = oracle.quantize(x, s, None, None, bs, qm)
    got = to_np(Q.quantize(to_dev(x), to_dev(s), None, None, bs, to_dev(qm)))
    assert got.dtype == want.dtype
    assert len(G.bit_mismatches(got, want)) == 0
    wd = oracle.dequantize(want, s, None, None, bs)
    gd = to_np(Q.dequantize(to_dev(want), to_dev(s), None, None, bs))
    assert len(G.bit_mismatches(gd, wd)) == 0


def test_empty_and_single():
    qm = quantization_map("fp4_e2m1")
    e = torch.empty((0, 16), dtype=torch.bfloat16, device="cuda")
    s, c = Q.quantize_mx(e, to_dev(qm), [-1], 16, 6.0)
    assert s.shape == (0, 1) and c.shape == (0, 16)
    x = _rand((1, 1), "bf16", 3)
    ws, wc = oracle.quantize_mx(x, qm, [-1], 16, 6.0)
    gs, gc = Q.quantize_mx(to_dev(x), to_dev(qm), [-1], 16, 6.0)
    assert len(G.bit_mismatches(to_np(gs), ws)) == 0 and len(G.bit_mismatches(to_np(gc), wc)) == 0


# ---------------------------------------------------------------------------
# full-size configurations against the reference's own checksums
# ---------------------------------------------------------------------------
def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_full_c1_nvfp4():
    from voyager_b200 import synth

    S = G.full_checksums()
    x = synth.c1_input()
    assert sha(x) == S["c1_input"]
    s, c = Q.quantize_mx(to_dev(x), to_dev(quantization_map("fp4_e2m1")), [-1], 16, 6.0, False,
                         to_dev(quantization_map("fp8_e4m3")))
    assert sha(to_np(s)) == S["c1_scale"] and sha(to_np(c)) == S["c1_codes"]
    assert sha(to_np(Q.dequantize(c, s, None, [-1], 16))) == S["c1_deq"]


def test_full_c2_weights():
    from voyager_b200 import synth

    S = G.full_checksums()
    w = synth.c2_weight()
    wd = to_dev(w)
    s, c = Q.quantize_mx(wd, to_dev(G.tables()["lut4_index"]), [-1], 64, 1.0, False)
    assert sha(to_np(s)) == S["c2_nf4_scale"] and sha(to_np(c)) == S["c2_nf4_codes"]
    sp = wd.abs().amax() / 4096.0
    assert sha(to_np(sp)) == S["c2_posit8_scale"]
    assert sha(to_np(Q.quantize(wd, sp, qmap=to_dev(quantization_map("posit8_1"))))) == S["c2_posit8_codes"]
    # the observer's per-channel scale, divided as the reference does on the
    # host (torch's CUDA scalar division multiplies by a reciprocal instead)
    si = to_dev((np.abs(w).max(axis=1, keepdims=True) / np.float32(127.0)).astype(np.float32))
    assert sha(to_np(si)) == S["c2_int8_scale"]
    assert sha(to_np(Q.quantize(wd, si, qmap=to_dev(quantization_map("int8"))))) == S["c2_int8_codes"]


def test_full_c3_quantize():
    from voyager_b200 import synth

    S = G.full_checksums()
    a, w = synth.c3_operands()
    e4m3 = to_dev(quantization_map("fp8_e4m3"))
    for tag, arr in (("c3_a", a), ("c3_w", w)):
        s, c = Q.quantize_mx(to_dev(arr), e4m3, [-1], 32, 448.0, True)
        assert sha(to_np(s)) == S[f"{tag}_scale"] and sha(to_np(c)) == S[f"{tag}_codes"]


# ---------------------------------------------------------------------------
# GEMMs
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("m,k,n", [(1, 64, 32), (32, 128, 48), (130, 256, 96), (256, 512, 384)])
def test_linear_mx_mxfp8(m, k, n):
    a = _rand((m, k), "bf16", 11)
    w = _rand((n, k), "bf16", 12, std=0.02)
    qm = quantization_map("fp8_e4m3")
    sa, ca = oracle.quantize_mx(a, qm, [-1], 32, 448.0, True)
    sw, cw = oracle.quantize_mx(w, qm, [-1], 32, 448.0, True)
    want = oracle.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
    got = to_np(Q.linear_mx(to_dev(ca), to_dev(cw), None, input_scale=to_dev(sa),
                            weight_scale=to_dev(sw), block_size=32))
    assert got.dtype == want.dtype and got.shape == want.shape
    assert G.rel_l2(got, want) < 1e-3


def test_matmul_mx_axes():
    a = _rand((2, 64, 96), "bf16", 21)
    b = _rand((2, 96, 80), "bf16", 22)
    qm = quantization_map("fp8_e4m3")
    sa, ca = oracle.quantize_mx(a, qm, [-1], 32, 448.0, True)
    sb, cb = oracle.quantize_mx(b, qm, [-2], 32, 448.0, True)
    want = oracle.matmul_mx(ca, cb, input_scale=sa, weight_scale=sb, block_size=32)
    got = to_np(Q.matmul_mx(to_dev(ca), to_dev(cb), input_scale=to_dev(sa),
                            weight_scale=to_dev(sb), block_size=32))
    assert G.rel_l2(got, want) < 1e-3


def test_codebook_quantize_and_decode():
    """1-D codebook quantize (encode, quantized.py:253-309) and the decode a
    converted graph's linear_mx does through ``weight_code``."""
    x = _rand((16, 128), "bf16", 31)
    lut = quantization_map("lut4")
    levels = np.unique(oracle.numerics.bf16_bits_to_f32(lut)).astype(np.float32)
    from voyager_b200.synth import f32_to_bf16_bits

    cb = f32_to_bf16_bits(levels)
    s = np.array(0.5, dtype=np.float32).reshape(())
    want = oracle.quantize(x, s, qmap=cb)
    got = to_np(Q.quantize(to_dev(x), to_dev(s), qmap=to_dev(cb)))
    assert len(G.bit_mismatches(got, want)) == 0
    mid = ((levels[:-1] + levels[1:]) / 2).astype(np.float32)
    want_i = oracle.quantize(x, s, qmap=cb, output_code=mid)
    got_i = to_np(Q.quantize(to_dev(x), to_dev(s), qmap=to_dev(cb), output_code=to_dev(mid)))
    assert len(G.bit_mismatches(got_i, want_i)) == 0


def test_hardware_rounders_verified():
    """The tensor-core formats take the hardware conversion path, kept only
    after matching all 65,536 table entries on this device."""
    from voyager_b200.tables import rounder_for

    for name, hw in (("fp8_e4m3", 1), ("fp8_e5m2", 2), ("fp4_e2m1", 3)):
        rd = rounder_for(to_dev(G.tables()[name]), torch.device("cuda", 0))
        assert rd.c.hw == hw, (name, rd.c.describe())


@pytest.mark.parametrize("bs", [32, 64])
def test_quantize_mx_e4m3_special_values(bs):
    """MXFP8 (E4M3 table, power-of-two scales) on blocks that leave the
    conversions' common case: zeros and -0, a quotient that rounds to a bf16
    zero (a tiny value beside a large one), a whole zero block, NaN and
    infinities, next to ordinary blocks.  Codes and scales bit-exact against
    the oracle; the GEMM operand written in the same pass equals
    vq_mx_pack's packing of the returned codes wherever the scale has a
    UE8M0 form."""
    from voyager_b200 import mxgemm
    from voyager_b200.synth import f32_to_bf16_bits

    rng = np.random.Generator(np.random.PCG64(77))
    x = rng.standard_normal((8, 256)).astype(np.float32)
    x[0, :4] = [0.0, -0.0, 3.0, -1.0]
    x[1, :3] = [3e4, -1e-35, 1e-35]
    x[2, :bs] = 0.0
    x[3, 5] = -0.0
    x[4, 7] = np.nan
    x[5, 9] = np.inf
    x[6, :bs] = -1e-36
    x[6, 1] = 2e3
    x[7, :3] = [3e4, -1e-40, 1e-40]  # quotients of 2^-139: a bf16 -0 and +0
    xb = f32_to_bf16_bits(x)
    qm = quantization_map("fp8_e4m3")
    ws, wc = oracle.quantize_mx(xb, qm, [-1], bs, 448.0, True)
    xs = to_dev(xb)
    gs, gc = Q.quantize_mx(xs, to_dev(qm), [-1], bs, 448.0, True)
    assert len(G.bit_mismatches(to_np(gs), ws)) == 0
    assert len(G.bit_mismatches(to_np(gc), wc)) == 0
    if bs == 32:
        entry = mxgemm._vouched_entry(gc, gs)
        if entry is not None and entry[1] is not None:
            pc, ps = entry[1]
            ok_rows = [r for r in range(8) if r not in (4, 5)]  # NaN / inf scales: no UE8M0
            rc, rs, _ = mxgemm._pack(gc.contiguous(), gs.contiguous(), 128, False)
            got = pc.view(-1, 256)[ok_rows]
            want = rc.view(-1, 256)[ok_rows]
            assert torch.equal(got, want)
