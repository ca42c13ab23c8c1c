"""sdpa_mx on CUDA: the fused tcgen05 MXFP8 attention against the
reference's own outputs (golden fixtures) and the oracle, and the composite
path for what the fused kernel does not take.

Tolerance rel-L2 <= 1e-3 against the reference / oracle output (the GEMM
bound of this library): the scores are the same float32 dot products summed
in another order (a bf16 score moves by one ulp now and then), exp is the
hardware ex2 approximation (relative error ~1e-7 before the bf16 rounding of
each probability), and a probability that moves across an E4M3 rounding
boundary changes its code by one step.  Measured on a B200: at most 2.4e-5
against the reference's golden outputs and 7.3e-5 against the oracle (the
2048-key causal case included)."""

import numpy as np
import pytest
import torch

import _golden as G
import oracle
from _tt import to_dev, to_np
from oracle.numerics import quantization_map

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    yield


@pytest.fixture()
def fused_calls(monkeypatch):
    from voyager_b200 import attention

    n = {"fused": 0, "composite": 0}
    real_f, real_c = attention._fused, attention._composite

    def f(*a, **k):
        out = real_f(*a, **k)
        n["fused"] += out is not None
        return out

    def c(*a, **k):
        n["composite"] += 1
        return real_c(*a, **k)

    monkeypatch.setattr(attention, "_fused", f)
    monkeypatch.setattr(attention, "_composite", c)
    return n


def _call(ins, kw):
    t = [to_dev(a) for a in ins]
    k = {}
    for key, v in kw.items():
        k[key] = to_dev(v) if isinstance(v, np.ndarray) else v
    out = torch.ops.quantized_ops.sdpa_mx(*t, **k)
    torch.cuda.synchronize()
    return to_np(out)


SDPA = [c for c in G.small_cases() if c["op"] == "sdpa_mx"]


@pytest.mark.parametrize("case", SDPA, ids=[c["name"] for c in SDPA])
def test_fused_matches_reference_golden(case, fused_calls):
    ins, kw, outs = G.resolve_case(case)
    got = _call(ins, kw)
    assert fused_calls["fused"] == 1 and fused_calls["composite"] == 0
    assert got.shape == outs[0].shape
    assert G.rel_l2(got, outs[0]) < TOL, G.rel_l2(got, outs[0])


def _operands(B, H, HKV, SQ, SKV, seed, sd=2.0):
    rng = np.random.default_rng(seed)
    qm = quantization_map("fp8_e4m3")

    def mx(shape, axis, s=1.0):
        x = oracle.f32_to_bf16_bits((rng.standard_normal(shape) * s).astype(np.float32))
        return oracle.quantize_mx(x, qm, [axis], 32, 448.0, True)

    sq, cq = mx((B, H, SQ, 128), -1, sd)
    sk, ck = mx((B, HKV, SKV, 128), -1, sd)
    sv, cv = mx((B, HKV, SKV, 128), -2)
    kw = dict(query_scale=sq, key_scale=sk, value_scale=sv, block_size=32, probs_qmap=qm,
              probs_quant_max=448.0, force_scale_power_of_two=True, enable_gqa=HKV != H)
    return [cq, ck, cv], kw


@pytest.mark.parametrize("B,H,HKV,SQ,SKV,causal", [
    (2, 4, 4, 512, 512, True),    # many tiles, heaviest-first order
    (1, 2, 2, 128, 384, False),   # more keys than queries
    (1, 3, 3, 384, 256, True),    # more queries than keys (top-left causal)
    (3, 8, 2, 256, 256, True),    # grouped-query heads
])
def test_fused_matches_oracle(B, H, HKV, SQ, SKV, causal, fused_calls):
    ins, kw = _operands(B, H, HKV, SQ, SKV, seed=B * 100 + SQ)
    want = oracle.sdpa_mx(*ins, is_causal=causal, **kw)
    got = _call(ins, dict(kw, is_causal=causal))
    assert fused_calls["fused"] == 1
    assert G.rel_l2(got, want) < TOL, G.rel_l2(got, want)


def test_sharp_softmax_and_scale_argument(fused_calls):
    """Large scores (one key dominates most rows) and an explicit scale."""
    ins, kw = _operands(1, 2, 2, 256, 256, seed=5, sd=6.0)
    want = oracle.sdpa_mx(*ins, is_causal=True, scale=0.25, **kw)
    got = _call(ins, dict(kw, is_causal=True, scale=0.25))
    assert fused_calls["fused"] == 1
    assert G.rel_l2(got, want) < TOL, G.rel_l2(got, want)


def test_value_as_transposed_quantize_output_is_bitwise_same(fused_calls):
    """The decoder passes v as the transposed view of quantize_mx(v^T)
    (blocks along the keys either way): same result, packed buffers reused."""
    ins, kw = _operands(1, 2, 2, 256, 256, seed=9)
    Q = torch.ops.quantized_ops
    q, k, v = (to_dev(a) for a in ins)
    args = dict(query_scale=to_dev(kw["query_scale"]), key_scale=to_dev(kw["key_scale"]),
                block_size=32, probs_qmap=to_dev(kw["probs_qmap"]), probs_quant_max=448.0,
                force_scale_power_of_two=True)
    a = Q.sdpa_mx(q, k, v, is_causal=True, value_scale=to_dev(kw["value_scale"]), **args)
    table = to_dev(kw["probs_qmap"])
    # requantize v^T along its last axis: identical codes and scales
    deq = Q.dequantize(v, to_dev(kw["value_scale"]), None, [-2], 32)
    svt, cvt = Q.quantize_mx(deq.transpose(-1, -2).contiguous(), table, [-1], 32, 448.0, True)
    assert torch.equal(cvt.transpose(-1, -2).float(), v.float())
    b = Q.sdpa_mx(q, k, cvt.transpose(-1, -2), is_causal=True,
                  value_scale=svt.transpose(-1, -2), **args)
    torch.cuda.synchronize()
    assert fused_calls["fused"] == 2
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("what", ["short_seq", "float_mask", "no_probs_quant"])
def test_composite_path_matches_oracle(what, fused_calls):
    if what == "short_seq":
        ins, kw = _operands(1, 2, 2, 64, 64, seed=3)
        extra = dict(is_causal=True)
    else:
        ins, kw = _operands(1, 2, 2, 128, 128, seed=4)
        if what == "float_mask":
            rng = np.random.default_rng(1)
            m = oracle.f32_to_bf16_bits(np.where(rng.random((128, 128)) < 0.2, -1e4, 0.0)
                                        .astype(np.float32))
            extra = dict(attn_mask=m)
        else:
            kw = dict(kw, probs_qmap=None)
            extra = dict(is_causal=True)
    want = oracle.sdpa_mx(*ins[:3], extra.get("attn_mask"), 0.0, extra.get("is_causal", False),
                          **kw)
    t = [to_dev(a) for a in ins]
    kk = {k: (to_dev(v) if isinstance(v, np.ndarray) else v) for k, v in kw.items()}
    if "attn_mask" in extra:
        got = torch.ops.quantized_ops.sdpa_mx(*t, to_dev(extra["attn_mask"]), **kk)
    else:
        got = torch.ops.quantized_ops.sdpa_mx(*t, is_causal=True, **kk)
    torch.cuda.synchronize()
    assert fused_calls["fused"] == 0 and fused_calls["composite"] == 1
    assert G.rel_l2(to_np(got), want) < TOL, G.rel_l2(to_np(got), want)
