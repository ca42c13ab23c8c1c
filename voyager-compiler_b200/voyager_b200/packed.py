"""Packed storage of MX-quantized tensors: codes and block scales at their
bit widths, for files and host-to-device transfer.

The reference keeps quantized tensors as float values -- bf16 codes and bf16
scales from ``quantize_mx`` -- and dumps every tensor as a float32 ``.bin``
file (``vc/codegen/transform/bufferize/emit.py:160-166``, ``np.tofile`` of
the float32 copy) with the logical dtype kept in node metadata
(``emit.py:325-331``).  Here the same values are stored in their formats:

  MXFP8  E4M3 codes, power-of-two scales, blocks of 32 along the last dim:
         codes as E4M3 bytes, row-major ``[RT * 128, Kp]`` (Kp = K rounded
         up to 128, zero filled; RT = the rows in whole chunks of
         ``row_multiple`` = 128 or 256), scales as UE8M0 bytes in the
         tensor cores' scale-factor atoms ``[KT][RT][512]``: byte
         ``(r % 32) * 16 + (r / 32 % 4) * 4 + j`` for row r and K block j of
         a 128-wide K tile, padding 127 (2^0).  This is the layout
         ``vq_mx_pack`` writes, so a loaded tensor reaches the GEMM with one
         copy and no repacking;
  NVFP4  E2M1 codes, E4M3 scales, blocks of 16: codes as nibbles, two per
         byte, even k in the low nibble, ``[R, ceil(K / 2)]``; scales as E4M3
         bytes ``[R, K / 16]``.

``pack_mxfp8`` / ``pack_nvfp4`` and ``unpack`` are exact inverses on the
values ``quantize_mx`` produces (NaN codes are the tables' NaN pattern
0xFFFF; E4M3 stores it as 0x7F).  ``save`` / ``load`` write a small
self-describing container: the magic ``VQMX``, a little-endian uint32 header
length, a JSON header, then the code and scale bytes, each starting on a
64-byte boundary.  ``save_fp32_bin`` writes the reference's float32 dump of
the codes for tools that read those.
"""

import json
import struct
from dataclasses import dataclass
from typing import Tuple

import numpy as np

MAGIC = b"VQMX"
VERSION = 1
NAN_BITS = 0xFFFF  # the NaN pattern of the value tables (a NaN code)


# ---------------------------------------------------------------------------
# element encodings
# ---------------------------------------------------------------------------
def _f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(NAN_BITS), r)


def _e4m3_values() -> np.ndarray:
    """float value of each E4M3 byte (sign, 4-bit exponent, 3-bit mantissa;
    S.1111.111 is NaN, no infinities)."""
    v = np.empty(256, dtype=np.float64)
    for b in range(256):
        s, e, m = b >> 7, (b >> 3) & 0xF, b & 7
        if e == 15 and m == 7:
            v[b] = np.nan
            continue
        mag = (m / 8.0) * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
        v[b] = -mag if s else mag
    return v


def _build_e4m3():
    vals = _e4m3_values()
    to_bf16 = np.empty(256, dtype=np.uint16)
    for b in range(256):
        to_bf16[b] = NAN_BITS if np.isnan(vals[b]) else \
            int(_f32_to_bf16_bits(np.array([vals[b]], dtype=np.float32))[0])
    from_bf16 = np.full(65536, -1, dtype=np.int16)
    for b in range(256):
        if not np.isnan(vals[b]):
            from_bf16[to_bf16[b]] = b
    # every NaN pattern (the tables give 0xFFFF) stores as E4M3 NaN
    pats = np.arange(65536, dtype=np.uint32)
    nan = (pats & 0x7FFF) > 0x7F80
    from_bf16[nan] = 0x7F
    return to_bf16, from_bf16


E4M3_TO_BF16, E4M3_FROM_BF16 = _build_e4m3()

# E2M1 magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6 as bf16; the sign is bit 3
_E2M1_MAG_BF16 = np.array([0x0000, 0x3F00, 0x3F80, 0x3FC0, 0x4000, 0x4040, 0x4080, 0x40C0],
                          dtype=np.uint16)
E2M1_TO_BF16 = np.concatenate([_E2M1_MAG_BF16, _E2M1_MAG_BF16 | 0x8000]).astype(np.uint16)
E2M1_FROM_BF16 = np.full(65536, -1, dtype=np.int16)
E2M1_FROM_BF16[E2M1_TO_BF16] = np.arange(16, dtype=np.int16)


def _encode(bits: np.ndarray, table: np.ndarray, what: str) -> np.ndarray:
    code = table[bits.astype(np.int64)]
    if (code < 0).any():
        bad = bits.reshape(-1)[(code < 0).reshape(-1)][:4]
        raise ValueError(f"{what}: values that the format does not hold, e.g. bf16 "
                         f"{[hex(int(b)) for b in bad]}")
    return code.astype(np.uint8)


def ue8m0_from_bf16(scale_bits: np.ndarray) -> np.ndarray:
    """UE8M0 bytes of power-of-two bf16 scales: the exponent field for
    normal scales, 0 for 2^-127 (the bf16 subnormal 0x0040); anything else
    (a sign, a mantissa, 2^-128 and below, infinity) has no UE8M0 form."""
    s = scale_bits.astype(np.uint32)
    e = (s >> 7) & 0xFF
    normal = ((s & 0x807F) == 0) & (e >= 1) & (e <= 254)
    sub = s == 0x0040
    if not (normal | sub).all():
        bad = scale_bits.reshape(-1)[~(normal | sub).reshape(-1)][:4]
        raise ValueError("MXFP8 scales must be powers of two in [2^-127, 2^127]; got bf16 "
                         f"{[hex(int(b)) for b in bad]}")
    return np.where(sub, 0, e).astype(np.uint8)


def ue8m0_to_bf16(b: np.ndarray) -> np.ndarray:
    b = b.astype(np.uint32)
    if (b == 255).any():
        raise ValueError("UE8M0 byte 255 (NaN) in a packed scale")
    return np.where(b == 0, 0x0040, b << 7).astype(np.uint16)


# ---------------------------------------------------------------------------
# the packed tensor
# ---------------------------------------------------------------------------
@dataclass
class PackedMX:
    fmt: str            # "mxfp8" or "nvfp4"
    rows: int           # R: the 2-D view [R, K], blocks along K
    cols: int           # K
    block_size: int     # 32 (mxfp8) or 16 (nvfp4)
    row_multiple: int   # mxfp8: rows padded to this (128 or 256); nvfp4: 1
    codes: np.ndarray   # uint8, flat
    scales: np.ndarray  # uint8, flat

    @property
    def nbytes(self) -> int:
        return int(self.codes.nbytes + self.scales.nbytes)

    def header(self) -> dict:
        return {"version": VERSION, "fmt": self.fmt, "rows": self.rows, "cols": self.cols,
                "block_size": self.block_size, "row_multiple": self.row_multiple,
                "codes_bytes": int(self.codes.nbytes), "scales_bytes": int(self.scales.nbytes)}


def _as_bits(t) -> np.ndarray:
    """bf16 bits (uint16) of a bf16 torch tensor or a uint16 array."""
    if isinstance(t, np.ndarray):
        if t.dtype != np.uint16:
            raise TypeError("numpy inputs are bf16 bit patterns (uint16)")
        return t
    import torch

    if t.dtype != torch.bfloat16:
        raise TypeError("codes and scales are bf16 tensors")
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _two_d(codes: np.ndarray, scale: np.ndarray, bs: int) -> Tuple[np.ndarray, np.ndarray]:
    if codes.ndim < 1:
        raise ValueError("codes need at least one dimension")
    K = codes.shape[-1]
    c2 = codes.reshape(-1, K)
    nkb = (K + bs - 1) // bs
    if scale.shape[-1] != nkb or scale.size != c2.shape[0] * nkb:
        raise ValueError(f"scales of shape {scale.shape} do not match codes {codes.shape} "
                         f"in blocks of {bs} along the last dim")
    return c2, scale.reshape(-1, nkb)


def pack_mxfp8(codes, scale, row_multiple: int = 128) -> PackedMX:
    """MXFP8 codes [.., K] and their power-of-two block-32 scales [.., K/32]
    -> E4M3 bytes and UE8M0 atoms in the GEMM operand layout.  Use
    ``row_multiple=256`` for a weight (the CTA-pair GEMM reads B in
    256-row tiles)."""
    if row_multiple not in (128, 256):
        raise ValueError("row_multiple is 128 or 256")
    c2, s2 = _two_d(_as_bits(codes), _as_bits(scale), 32)
    R, K = c2.shape
    RT = (R + row_multiple - 1) // row_multiple * (row_multiple // 128)
    KT = (K + 127) // 128
    Kp = KT * 128
    out = np.zeros((RT * 128, Kp), dtype=np.uint8)
    out[:R, :K] = _encode(c2, E4M3_FROM_BF16, "MXFP8 codes")
    sf = np.full((RT * 128, KT * 4), 127, dtype=np.uint8)
    sf[:R, :s2.shape[1]] = ue8m0_from_bf16(s2)
    # [rt, q, i, kt, j] -> [kt, rt, i, q, j]: row r = 128 rt + 32 q + i
    atoms = sf.reshape(RT, 4, 32, KT, 4).transpose(3, 0, 2, 1, 4).reshape(-1)
    return PackedMX("mxfp8", R, K, 32, row_multiple, out.reshape(-1), np.ascontiguousarray(atoms))


def pack_nvfp4(codes, scale) -> PackedMX:
    """NVFP4 codes [.., K] (E2M1 values) and their E4M3 block-16 scales
    [.., K/16] -> nibbles (even k low) and E4M3 bytes, row-major."""
    c2, s2 = _two_d(_as_bits(codes), _as_bits(scale), 16)
    R, K = c2.shape
    nib = _encode(c2, E2M1_FROM_BF16, "NVFP4 codes")
    if K % 2:
        nib = np.concatenate([nib, np.zeros((R, 1), dtype=np.uint8)], axis=1)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    sb = _encode(s2, E4M3_FROM_BF16, "NVFP4 scales")
    return PackedMX("nvfp4", R, K, 16, 1, packed.reshape(-1), sb.reshape(-1))


def unpack(p: PackedMX) -> Tuple[np.ndarray, np.ndarray]:
    """(codes, scales) as bf16 bit patterns, [R, K] and [R, K / block]:
    the values quantize_mx returned."""
    R, K = p.rows, p.cols
    if p.fmt == "mxfp8":
        RT = (R + p.row_multiple - 1) // p.row_multiple * (p.row_multiple // 128)
        KT = (K + 127) // 128
        codes = p.codes.reshape(RT * 128, KT * 128)[:R, :K]
        sf = p.scales.reshape(KT, RT, 32, 4, 4).transpose(1, 3, 2, 0, 4).reshape(RT * 128, KT * 4)
        return E4M3_TO_BF16[codes], ue8m0_to_bf16(sf[:R, :(K + 31) // 32])
    if p.fmt == "nvfp4":
        b = p.codes.reshape(R, (K + 1) // 2)
        nib = np.empty((R, b.shape[1] * 2), dtype=np.uint8)
        nib[:, 0::2], nib[:, 1::2] = b & 0xF, b >> 4
        return E2M1_TO_BF16[nib[:, :K]], E4M3_TO_BF16[p.scales.reshape(R, (K + 15) // 16)]
    raise ValueError(f"unknown packed format {p.fmt!r}")


# ---------------------------------------------------------------------------
# files
# ---------------------------------------------------------------------------
def _pad64(n: int) -> int:
    return (n + 63) // 64 * 64


def save(path: str, p: PackedMX) -> None:
    """Write the container: magic, uint32 header length, JSON header, then
    the code and scale bytes, each 64-byte aligned."""
    head = json.dumps(p.header(), sort_keys=True).encode()
    first = _pad64(len(MAGIC) + 4 + len(head))
    with open(path, "wb") as f:
        f.write(MAGIC + struct.pack("<I", len(head)) + head)
        f.write(b"\0" * (first - len(MAGIC) - 4 - len(head)))
        f.write(p.codes.tobytes())
        f.write(b"\0" * (_pad64(p.codes.nbytes) - p.codes.nbytes))
        f.write(p.scales.tobytes())


def load(path: str) -> PackedMX:
    with open(path, "rb") as f:
        data = f.read()
    if data[:4] != MAGIC:
        raise ValueError(f"{path}: not a packed MX tensor (magic {data[:4]!r})")
    (n,) = struct.unpack("<I", data[4:8])
    h = json.loads(data[8:8 + n].decode())
    if h.get("version") != VERSION:
        raise ValueError(f"{path}: container version {h.get('version')} (expected {VERSION})")
    o = _pad64(8 + n)
    cb, sb = h["codes_bytes"], h["scales_bytes"]
    o2 = o + _pad64(cb)
    if len(data) < o2 + sb:
        raise ValueError(f"{path}: truncated ({len(data)} bytes, need {o2 + sb})")
    codes = np.frombuffer(data, dtype=np.uint8, count=cb, offset=o).copy()
    scales = np.frombuffer(data, dtype=np.uint8, count=sb, offset=o2).copy()
    p = PackedMX(h["fmt"], h["rows"], h["cols"], h["block_size"], h["row_multiple"], codes,
                 scales)
    unpack(p)  # shape check: the byte counts must fit the recorded layout
    return p


def save_fp32_bin(path: str, codes) -> None:
    """The reference's tensor dump: the float32 values, raw (``np.tofile``)."""
    bits = _as_bits(codes).astype(np.uint32) << 16
    bits.view(np.float32).tofile(path)


# ---------------------------------------------------------------------------
# to the device
# ---------------------------------------------------------------------------
def to_device(p: PackedMX, device, weight: bool = False, verify: bool = True):
    """MXFP8: (codes, scale) bf16 tensors on ``device`` with the packed
    operand registered for the GEMM, so ``linear_mx`` / ``matmul_mx`` read
    the loaded bytes instead of packing again: as the weight operand
    (``weight=True``, which needs ``row_multiple=256``) or as an activation
    operand.  With ``verify`` the loaded bytes are compared once with the
    library's own packing of the same codes and a difference raises.
    Whatever ``verify``, operands the GEMM does not take (E4M3 NaN bytes,
    or zero UE8M0 bytes -- a 2^-127 block scale) are not registered: the
    ops then check and route them as they would any other operand."""
    import torch

    from voyager_b200 import mxgemm

    if p.fmt != "mxfp8":
        raise ValueError("to_device registers MXFP8 GEMM operands")
    # the GEMM indexes scale atoms with RT = ceil(M / 128) for the
    # activation and 2 ceil(N / 256) for the weight
    if weight and p.row_multiple != 256:
        raise ValueError("a weight operand is packed with row_multiple=256")
    if not weight and p.row_multiple != 128:
        raise ValueError("an activation operand is packed with row_multiple=128")
    c, s = unpack(p)
    dev = torch.device(device)
    codes = torch.from_numpy(c.view(np.int16).copy()).view(torch.bfloat16).to(dev)
    scale = torch.from_numpy(s.view(np.int16).copy()).view(torch.bfloat16).to(dev)
    pc = torch.from_numpy(p.codes).to(dev)
    ps = torch.from_numpy(p.scales).to(dev)
    if verify:
        rc, rs, ok = mxgemm._pack(codes, scale, p.row_multiple, True)
        if not ok:
            # NaN codes, or 2^-127 scales (exact in UE8M0, but the GEMM path
            # leaves such blocks to the dequantize route)
            raise ValueError("the GEMM does not take this operand (NaN codes or 2^-127 scales)")
        if not torch.equal(rc, pc) or not torch.equal(rs, ps):
            raise ValueError("the loaded operand differs from the library's packing")
    # a cheap host check, verified or not: NaN codes (0x7F / 0xFF) or a zero
    # scale byte keep the operand off the GEMM's fast path
    clean = not (np.any((p.codes & 0x7F) == 0x7F) or np.any(p.scales == 0))
    if weight:
        key = (codes._version, id(scale), scale._version)
        mxgemm._wcache.put(codes, key, (pc, ps, clean))
    elif clean:
        mxgemm.vouch(codes, scale, (pc, ps))
    return codes, scale
