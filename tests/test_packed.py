"""The packed storage format (voyager_b200.packed) on the host: MXFP8 and
NVFP4 codes and scales from the oracle's quantize_mx round-trip exactly
through the packed bytes and through a file, the MXFP8 bytes sit where the
tensor cores' operand layout puts them (checked element by element against
the layout's formula), and values the formats cannot hold are refused."""

import numpy as np
import pytest

import oracle
from oracle.numerics import f32_to_bf16_bits, quantization_map


def _x(shape, seed, specials=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape).astype(np.float32) * 3
    if specials:
        flat = x.reshape(-1)
        flat[:6] = [0.0, -0.0, 1e-30, -1e-30, 3e4, -2.5]
    return f32_to_bf16_bits(x)


def _mxfp8(shape, seed, specials=True):
    return oracle.quantize_mx(_x(shape, seed, specials), quantization_map("fp8_e4m3"), [-1], 32,
                              448.0, True)


@pytest.mark.parametrize("shape", [(5, 96), (130, 200), (256, 128), (3, 4, 64), (1, 32)])
@pytest.mark.parametrize("row_multiple", [128, 256])
def test_mxfp8_round_trip(shape, row_multiple):
    from voyager_b200 import packed

    scale, codes = _mxfp8(shape, sum(shape))
    p = packed.pack_mxfp8(codes, scale, row_multiple)
    c, s = packed.unpack(p)
    K = shape[-1]
    assert np.array_equal(c, codes.reshape(-1, K)) and np.array_equal(s, scale.reshape(c.shape[0], -1))
    R = c.shape[0]
    RT = -(-R // row_multiple) * (row_multiple // 128)
    KT = -(-K // 128)
    assert p.codes.size == RT * 128 * KT * 128 and p.scales.size == KT * RT * 512


def test_mxfp8_layout_formula():
    """Every byte where the operand layout puts it: code (r, c) at
    r * Kp + c; the scale of (r, K block kb) in atom (kt, rt) at
    (r % 32) * 16 + (r / 32 % 4) * 4 + j; padding codes 0, padding scales 127."""
    from voyager_b200 import packed

    scale, codes = _mxfp8((150, 160), 3)
    p = packed.pack_mxfp8(codes, scale, 128)
    R, K = codes.shape
    RT, KT = 2, 2
    Kp = KT * 128
    cb = p.codes.reshape(RT * 128, Kp)
    for r in range(RT * 128):
        for c in range(0, Kp, 7):
            want = packed.E4M3_FROM_BF16[codes[r, c]] if (r < R and c < K) else 0
            assert cb[r, c] == want, (r, c)
    nkb = K // 32
    for r in range(RT * 128):
        for kb in range(KT * 4):
            kt, j, rt, rr = kb // 4, kb % 4, r // 128, r % 128
            byte = p.scales[(kt * RT + rt) * 512 + (rr % 32) * 16 + (rr // 32) * 4 + j]
            want = ((int(scale[r, kb]) >> 7) & 0xFF) if (r < R and kb < nkb) else 127
            assert byte == want, (r, kb)


@pytest.mark.parametrize("shape", [(7, 64), (33, 48), (2, 3, 32)])
def test_nvfp4_round_trip(shape):
    from voyager_b200 import packed

    x = _x(shape, 11, specials=False)
    scale, codes = oracle.quantize_mx(x, quantization_map("fp4_e2m1"), [-1], 16, 6.0, False,
                                      quantization_map("fp8_e4m3"))
    p = packed.pack_nvfp4(codes, scale)
    c, s = packed.unpack(p)
    K = shape[-1]
    assert np.array_equal(c, codes.reshape(-1, K)) and np.array_equal(s, scale.reshape(c.shape[0], -1))
    assert p.nbytes == c.shape[0] * (K // 2 + K // 16)


def test_file_round_trip_and_format(tmp_path):
    from voyager_b200 import packed

    scale, codes = _mxfp8((40, 96), 5)
    p = packed.pack_mxfp8(codes, scale, 256)
    path = str(tmp_path / "w.vqmx")
    packed.save(path, p)
    q = packed.load(path)
    assert q.header() == p.header()
    assert np.array_equal(q.codes, p.codes) and np.array_equal(q.scales, p.scales)
    raw = open(path, "rb").read()
    n = int.from_bytes(raw[4:8], "little")
    first = (8 + n + 63) // 64 * 64
    assert raw[:4] == b"VQMX" and raw[first:first + p.codes.nbytes] == p.codes.tobytes()
    # a damaged file is refused
    bad = str(tmp_path / "bad.vqmx")
    open(bad, "wb").write(b"XXXX" + raw[4:])
    with pytest.raises(ValueError):
        packed.load(bad)
    open(bad, "wb").write(raw[:-10])
    with pytest.raises(ValueError):
        packed.load(bad)


def test_fp32_dump_is_the_float_values(tmp_path):
    from voyager_b200 import packed

    scale, codes = _mxfp8((4, 64), 9)
    path = str(tmp_path / "codes.bin")
    packed.save_fp32_bin(path, codes)
    got = np.fromfile(path, dtype=np.float32)
    want = (codes.astype(np.uint32) << 16).view(np.float32).reshape(-1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_values_outside_the_formats_are_refused():
    from voyager_b200 import packed

    codes = np.full((1, 32), 0x3F80, dtype=np.uint16)   # 1.0
    scale = np.full((1, 1), 0x3F80, dtype=np.uint16)
    packed.pack_mxfp8(codes, scale)
    with pytest.raises(ValueError):
        packed.pack_mxfp8(np.full((1, 32), 0x3F81, dtype=np.uint16), scale)  # 1.0078: not E4M3
    with pytest.raises(ValueError):
        packed.pack_mxfp8(codes, np.full((1, 1), 0x3FC0, dtype=np.uint16))  # 1.5: not 2^k
    with pytest.raises(ValueError):
        packed.pack_mxfp8(codes, np.full((1, 2), 0x3F80, dtype=np.uint16))  # block count
    with pytest.raises(ValueError):
        packed.pack_nvfp4(np.full((1, 16), 0x4100, dtype=np.uint16),      # 8.0: not E2M1
                          np.full((1, 1), 0x3F80, dtype=np.uint16))
    # 2^-127 is exact in UE8M0 (byte 0); NaN codes store as the E4M3 NaN
    s = np.array([[0x0040]], dtype=np.uint16)
    c = np.full((1, 32), 0xFFFF, dtype=np.uint16)
    p = packed.pack_mxfp8(c, s)
    cc, ss = packed.unpack(p)
    assert np.array_equal(cc, c) and np.array_equal(ss, s)


def test_to_device_checks_the_operand_role():
    """The GEMM indexes scale atoms with RT = ceil(M / 128) for the
    activation and 2 ceil(N / 256) for the weight: each role takes its own
    row multiple (checked before anything touches a device)."""
    from voyager_b200 import packed

    scale, codes = _mxfp8((8, 64), 2)
    with pytest.raises(ValueError):
        packed.to_device(packed.pack_mxfp8(codes, scale, 128), "cpu", weight=True)
    with pytest.raises(ValueError):
        packed.to_device(packed.pack_mxfp8(codes, scale, 256), "cpu", weight=False)
    with pytest.raises(ValueError):
        packed.to_device(packed.pack_nvfp4(np.zeros((1, 16), np.uint16),
                                           np.full((1, 1), 0x3F80, np.uint16)), "cpu")
