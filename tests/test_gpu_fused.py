"""The decoder-graph fusions (voyager_b200.fused) against the unfused graph
on the GPU: the torch bf16 ops followed by this library's quantize_mx (whose
codes and scales are checked bit-exact against the reference elsewhere).

RoPE, the v transpose and SwiGLU round exactly as torch's CUDA kernels do,
so codes and scales must match bit for bit.  RMSNorm sums its squares in its
own order: a row's rsqrt can move by an ulp, so a few codes may differ; the
bound is 0.1 % of codes and rel-L2 1e-3 of the dequantized values.  The
packed operand must equal what vq_mx_pack makes of the returned codes."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    yield


def _table():
    from voyager_b200.tables import get_quantization_map

    return get_quantization_map("fp8_e4m3", "cuda")


def _qmx(x):
    return torch.ops.quantized_ops.quantize_mx(x.contiguous(), _table(), [-1], 32, 448.0, True)


def _same(a, b):
    return torch.equal(a.view(torch.int16), b.view(torch.int16))


def _check_packed(codes2d, scale2d):
    """The fused operand of codes2d equals vq_mx_pack's packing of it."""
    from voyager_b200 import mxgemm

    entry = mxgemm._vouched_entry(codes2d._base if codes2d._base is not None else codes2d,
                                  scale2d._base if scale2d._base is not None else scale2d)
    assert entry is not None and entry[1] is not None
    pc, ps = entry[1]
    R, C = codes2d.shape
    rc, rs, ok = mxgemm._pack(codes2d.contiguous(), scale2d.contiguous(), 128, True)
    assert ok
    cp = (C + 127) // 128 * 128
    got = pc.view(-1, cp)[:R]
    want = rc.view(-1, cp)[:R]
    assert torch.equal(got, want)
    # scale atoms: compare the bytes that hold real rows
    rt = (R + 127) // 128
    ga, wa = ps.view(cp // 128, rt, 512), rs.view(cp // 128, rt, 512)
    full = R // 128
    assert torch.equal(ga[:, :full], wa[:, :full])


def test_swiglu_bit_exact():
    from voyager_b200 import fused

    g = torch.Generator(device="cuda").manual_seed(1)
    F = 1376  # a TP shard of 11008: the packed operand pads to 1408
    gu = (torch.randn((300, 2 * F), generator=g, device="cuda") * 3).bfloat16()
    gu[0, :8] = torch.tensor([0.0, -0.0, 300.0, -300.0, 80.0, -80.0, 1e-30, -1e-30])
    s, c = fused.swiglu_quantize_mx(gu, F, _table())
    ws, wc = _qmx(torch.nn.functional.silu(gu[:, :F]) * gu[:, F:])
    assert _same(s, ws) and _same(c, wc)
    _check_packed(c, s)
    # infinities: the same codes and scales as the unfused graph (an infinite
    # block scale has no UE8M0 form, so no packed check)
    gu[1, :4] = torch.tensor([float("inf"), float("-inf"), float("nan"), 1.0])
    gu[2, F:F + 2] = torch.tensor([float("inf"), float("-inf")])
    s, c = fused.swiglu_quantize_mx(gu, F, _table())
    ws, wc = _qmx(torch.nn.functional.silu(gu[:, :F]) * gu[:, F:])
    assert _same(s, ws)
    nan = torch.isnan(c.float()) & torch.isnan(wc.float())
    assert torch.equal(c.view(torch.int16)[~nan], wc.view(torch.int16)[~nan])


def test_rope_and_vt_bit_exact():
    from voyager_b200 import fused
    from voyager_b200.decoder import apply_rope, rope_tables

    B, S, H = 2, 256, 3
    hl = H * 128
    g = torch.Generator(device="cuda").manual_seed(2)
    qkv = (torch.randn((B * S, 3 * hl + 64), generator=g, device="cuda") * 4).bfloat16()
    qkv = qkv[:, :3 * hl]  # a row stride wider than the three blocks
    cos, sin = rope_tables(S, 128, 10000.0, "cuda", torch.bfloat16)
    (sq, cq), (sk, ck) = fused.rope_quantize_qk(qkv, 0, hl, cos, sin, B, S, H, _table())
    sv, cv = fused.quantize_vt(qkv, 2 * hl, B, S, H, _table())
    q, k, v = (t.reshape(B, S, H, 128).transpose(1, 2) for t in qkv.split(hl, -1))
    wsq, wcq = _qmx(apply_rope(q, cos, sin))
    wsk, wck = _qmx(apply_rope(k, cos, sin))
    wsv, wcv = _qmx(v.transpose(-1, -2))
    assert _same(sq, wsq) and _same(cq, wcq)
    assert _same(sk, wsk) and _same(ck, wck)
    assert _same(sv, wsv) and _same(cv, wcv)
    _check_packed(cq.view(-1, 128), sq.view(-1, 4))
    _check_packed(cv.view(-1, S), sv.view(-1, S // 32))


def test_rmsnorm_close():
    from voyager_b200 import fused
    from voyager_b200.decoder import rms_norm

    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((513, 4096), generator=g, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(4096, generator=g, device="cuda")).bfloat16()
    s, c = fused.rmsnorm_quantize_mx(x, w, 1e-5, _table())
    ws, wc = _qmx(rms_norm(x, w, 1e-5))
    diff = (c.view(torch.int16) != wc.view(torch.int16)).float().mean().item()
    assert diff < 1e-3, diff
    deq = c.float() * s.float().repeat_interleave(32, -1)
    wdeq = wc.float() * ws.float().repeat_interleave(32, -1)
    assert ((deq - wdeq).norm() / wdeq.norm()).item() < 1e-3
    _check_packed(c, s)


def test_fused_decoder_matches_unfused():
    from _oracle_ops import rel_l2
    from voyager_b200.decoder import Decoder, DecoderConfig, init_weights

    cfg = DecoderConfig(layers=2, hidden=512, heads=4, ffn=1376)
    w = init_weights(cfg, 4, "cuda")
    x = torch.randn((2, 256, cfg.hidden), device="cuda").bfloat16()
    a = Decoder(cfg, w, fused=True)(x)
    b = Decoder(cfg, w, fused=False)(x)
    assert rel_l2(a, b) < 1e-2, rel_l2(a, b)


def test_rope_vt_rmsnorm_special_values():
    """Values that leave the conversions' common case: zeros, -0, a quotient
    that rounds to a bf16 zero (a tiny value beside a large one in the same
    block of 32), infinities and NaN.  Codes and scales stay bit-exact."""
    from voyager_b200 import fused
    from voyager_b200.decoder import apply_rope, rms_norm, rope_tables

    B, S, H = 1, 128, 2
    hl = H * 128
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = torch.randn((B * S, 3 * hl), generator=g, device="cuda").bfloat16()
    special = torch.tensor([0.0, -0.0, 3e4, -1e-38, 1e-38, -2.0, float("inf"), float("nan")])
    qkv[0, :8] = special.bfloat16()           # q of token 0, head 0
    qkv[1, hl + 64:hl + 70] = special[:6].bfloat16()  # k of token 1
    qkv[:8, 2 * hl + 5] = special.bfloat16()  # v: one dim over 8 tokens
    qkv[32:64, 2 * hl + 9] = 0.0              # v: a whole block of zeros
    qkv[64, 2 * hl + 11] = -0.0
    qkv[65, 2 * hl + 11] = 5e4                # v: a tiny quotient beside a large value
    qkv[66, 2 * hl + 11] = -1e-30
    cos, sin = rope_tables(S, 128, 10000.0, "cuda", torch.bfloat16)
    (sq, cq), (sk, ck) = fused.rope_quantize_qk(qkv, 0, hl, cos, sin, B, S, H, _table())
    sv, cv = fused.quantize_vt(qkv, 2 * hl, B, S, H, _table())
    q, k, v = (t.reshape(B, S, H, 128).transpose(1, 2) for t in qkv.split(hl, -1))

    def same_or_nan(a, b):
        nan = torch.isnan(a.float()) & torch.isnan(b.float())
        return torch.equal(a.view(torch.int16)[~nan], b.view(torch.int16)[~nan])

    for (s, c), ref in (((sq, cq), apply_rope(q, cos, sin)), ((sk, ck), apply_rope(k, cos, sin)),
                        ((sv, cv), v.transpose(-1, -2))):
        ws, wc = _qmx(ref)
        assert _same(s, ws) and same_or_nan(c, wc)
    # RMSNorm: zero and -0 entries, a tiny value beside a large one
    x = torch.randn((4, 256), generator=g, device="cuda").bfloat16()
    x[0, :32] = 0.0
    x[1, 0], x[1, 1], x[1, 2] = -0.0, 3e4, -1e-30
    w = torch.ones(256, device="cuda").bfloat16()
    s, c = fused.rmsnorm_quantize_mx(x, w, 1e-5, _table())
    ws, wc = _qmx(rms_norm(x, w, 1e-5))
    # the row statistic is summed in the kernel's own order (an ulp of rsqrt
    # may move a code elsewhere); the planted entries and the zero block's
    # scale must match exactly
    assert _same(c[0, :32], wc[0, :32]) and _same(s[0, :1], ws[0, :1])
    assert _same(c[1, :3], wc[1, :3]) and _same(s[1, :1], ws[1, :1])
    assert (c.view(torch.int16) != wc.view(torch.int16)).float().mean().item() < 1e-2
