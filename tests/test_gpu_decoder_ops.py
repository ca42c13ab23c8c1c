"""Every quantized op inside one decoder layer at the C5 widths (hidden 4096,
32 heads of 128, ffn 11008; 256 tokens), checked on its actual inputs
against the oracle -- the layer as the converted graph runs it
(``quantize_pt2e.py:739-938``), with this library's fused kernels:

* ``linear_mx`` (q/k/v, gate/up; o_proj and down with the residual add in
  the GEMM epilogue) and ``sdpa_mx``: rel-L2 <= 1e-3 (float32 sums in
  another order);
* ``quantize_mx`` of the attention output: bit-exact, codes and scales;
* the fused quantizations: RoPE + ``quantize_mx`` of q and k, ``quantize_mx``
  of v^T and SwiGLU + ``quantize_mx`` bit-exact against ``quantize_mx`` of the
  unfused bf16 ops (torch on the same GPU);
* RMSNorm + ``quantize_mx``: the kernel sums the squares of a row in its own
  order, so a row's statistic can differ from torch's in the last bit and a
  value next to an E4M3 rounding boundary then takes the next code: at most
  0.5 % of the codes and of the scales differ, every other one is bit-exact.
"""

import numpy as np
import pytest
import torch

import _golden as G
import oracle
from _tt import to_np
from oracle.numerics import quantization_map

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    yield


def _c(t):
    return None if t is None else t.detach().clone()


def _same(got, want, what):
    bad = G.bit_mismatches(to_np(got), want)
    assert len(bad) == 0, f"{what}: {len(bad)} mismatches, first at {bad[:5]}"


@pytest.fixture(scope="module")
def recorded():
    """One layer's forward with every quantized op's inputs and outputs."""
    from voyager_b200 import fused, mxgemm
    from voyager_b200.decoder import Decoder, DecoderConfig, _CudaOps, init_weights

    rec = []
    mp = pytest.MonkeyPatch()

    class Rec(_CudaOps):
        def __init__(self):
            super().__init__()
            q = torch.ops.quantized_ops

            def quantize_mx(x, table, axes, bs, qmax, pow2=False):
                out = q.quantize_mx(x, table, axes, bs, qmax, pow2)
                rec.append(("quantize_mx", (_c(x), axes, bs, qmax, pow2), tuple(map(_c, out))))
                return out

            def linear_mx(x, w, bias=None, **kw):
                out = q.linear_mx(x, w, bias, **kw)
                rec.append(("linear_mx", (_c(x), _c(w), kw), _c(out)))
                return out

            def sdpa_mx(qq, kk, vv, **kw):
                out = q.sdpa_mx(qq, kk, vv, **kw)
                rec.append(("sdpa_mx", (_c(qq), _c(kk), _c(vv), kw), _c(out)))
                return out

            self.quantize_mx, self.linear_mx, self.sdpa_mx = quantize_mx, linear_mx, sdpa_mx

    def wrap(mod, name):
        real = getattr(mod, name)

        def f(*a, **k):
            out = real(*a, **k)
            rec.append((name, tuple(_c(x) if isinstance(x, torch.Tensor) else x for x in a),
                        {kk: _c(v) if isinstance(v, torch.Tensor) else v for kk, v in k.items()},
                        out))
            return out

        mp.setattr(mod, name, f)

    for n in ("rmsnorm_quantize_mx", "rope_quantize_qk", "quantize_vt", "swiglu_quantize_mx"):
        wrap(fused, n)
    wrap(mxgemm, "linear")
    try:
        cfg = DecoderConfig(layers=1)
        w = init_weights(cfg, 21, "cuda")
        x = torch.randn((1, 256, cfg.hidden), device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(4)).bfloat16()
        dec = Decoder(cfg, w, ops=Rec())
        dec(x)
        torch.cuda.synchronize()
        yield rec, cfg, dec
    finally:
        mp.undo()


def _qmap():
    return quantization_map("fp8_e4m3")


def test_the_layer_issues_the_converted_graph_ops(recorded):
    rec, cfg, _ = recorded
    names = [r[0] for r in rec]
    # linear_mx through the op for q/k/v and gate/up, the GEMM with its
    # residual add for o_proj and down
    assert names.count("linear_mx") == 2 and names.count("sdpa_mx") == 1
    assert names.count("rmsnorm_quantize_mx") == 2 and names.count("swiglu_quantize_mx") == 1
    assert names.count("rope_quantize_qk") == 1 and names.count("quantize_vt") == 1
    assert sum(1 for r in rec if r[0] == "linear" and r[2].get("residual") is not None) == 2


def test_linears_and_attention_match_the_oracle(recorded):
    rec, cfg, _ = recorded
    for r in rec:
        if r[0] == "linear_mx":
            (x, w, kw), out = r[1], r[2]
            want = oracle.linear_mx(to_np(x), to_np(w), None,
                                    input_scale=to_np(kw["input_scale"]),
                                    weight_scale=to_np(kw["weight_scale"]),
                                    block_size=kw["block_size"])
            assert G.rel_l2(to_np(out), want) < 1e-3
        elif r[0] == "linear" and r[2].get("residual") is not None:
            a, k, out = r[1], r[2], r[3]
            assert out is not None
            x, w, bias, sx, sw = a[:5]
            lin = oracle.linear_mx(to_np(x), to_np(w), None, input_scale=to_np(sx),
                                   weight_scale=to_np(sw), block_size=32)
            res = to_np(k["residual"])
            # the graph's residual add: bf16(bf16(linear) + residual)
            want = oracle.f32_to_bf16_bits(oracle.bf16_bits_to_f32(lin)
                                           + oracle.bf16_bits_to_f32(res))
            assert G.rel_l2(to_np(out), want) < 1e-3
        elif r[0] == "sdpa_mx":
            (q, k, v, kw), out = r[1], r[2]
            want = oracle.sdpa_mx(to_np(q), to_np(k), to_np(v), None, 0.0, kw["is_causal"],
                                  query_scale=to_np(kw["query_scale"]),
                                  key_scale=to_np(kw["key_scale"]),
                                  value_scale=to_np(kw["value_scale"]), block_size=32,
                                  probs_qmap=_qmap(), probs_quant_max=448.0,
                                  force_scale_power_of_two=True)
            assert G.rel_l2(to_np(out), want) < 1e-3


def test_quantize_mx_bit_exact(recorded):
    rec, _, _ = recorded
    n = 0
    for r in rec:
        if r[0] == "quantize_mx":
            (x, axes, bs, qmax, pow2), (s, c) = r[1], r[2]
            ws, wc = oracle.quantize_mx(to_np(x), _qmap(), axes, bs, qmax, pow2)
            _same(s, ws, "scale")
            _same(c, wc, "codes")
            n += 1
    assert n >= 1


def test_fused_rope_vt_swiglu_bit_exact(recorded):
    from voyager_b200.decoder import apply_rope

    rec, cfg, dec = recorded
    qm = _qmap()
    for r in rec:
        if r[0] == "rope_quantize_qk":
            qkv, q_off, k_off, cos, sin, batch, seq, heads = r[1][:8]
            (sq, cq), (sk, ck) = r[3]
            hd = cfg.head_dim
            for off, s, c in ((q_off, sq, cq), (k_off, sk, ck)):
                t = qkv[:, off:off + heads * hd].reshape(batch, seq, heads, hd).transpose(1, 2)
                ref = apply_rope(t, cos, sin).contiguous()
                ws, wc = oracle.quantize_mx(to_np(ref), qm, [-1], 32, 448.0, True)
                _same(s, ws, "rope scale")
                _same(c, wc, "rope codes")
        elif r[0] == "quantize_vt":
            qkv, v_off, batch, seq, heads = r[1][:5]
            s, c = r[3]
            hd = cfg.head_dim
            v = qkv[:, v_off:v_off + heads * hd].reshape(batch, seq, heads, hd).transpose(1, 2)
            vt = v.transpose(-1, -2).contiguous()
            ws, wc = oracle.quantize_mx(to_np(vt), qm, [-1], 32, 448.0, True)
            _same(s, ws, "v^T scale")
            _same(c, wc, "v^T codes")
        elif r[0] == "swiglu_quantize_mx":
            gu, cols = r[1][:2]
            s, c = r[3]
            act = torch.nn.functional.silu(gu[:, :cols]) * gu[:, cols:2 * cols]
            ws, wc = oracle.quantize_mx(to_np(act.contiguous()), qm, [-1], 32, 448.0, True)
            _same(s, ws, "swiglu scale")
            _same(c, wc, "swiglu codes")


def test_fused_rmsnorm_within_its_reduction_order(recorded):
    from voyager_b200.decoder import rms_norm

    rec, cfg, _ = recorded
    n = 0
    for r in rec:
        if r[0] != "rmsnorm_quantize_mx":
            continue
        x, w, eps = r[1][:3]
        s, c = r[3]
        ref = rms_norm(x, w, eps).contiguous()
        ws, wc = oracle.quantize_mx(to_np(ref), _qmap(), [-1], 32, 448.0, True)
        gs, gc = to_np(s), to_np(c)
        assert len(G.bit_mismatches(gs, ws)) <= 0.005 * ws.size
        assert len(G.bit_mismatches(gc, wc)) <= 0.005 * wc.size
        n += 1
    assert n == 2
