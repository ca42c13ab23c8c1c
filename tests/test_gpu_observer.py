"""The device amax observer against the reference's own outputs and the
oracle: ``FusedAmaxObsFakeQuantize._update_amax_scale``
(fake_quantize.py:494-527) through ``vq_amax_observe``, bit-exact."""

import numpy as np
import pytest
import torch

from oracle import observer as ob
from oracle import ops as oops
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits, quantization_map
from test_observer import DATA, META, as_f32, same_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    yield


def to_dev(x, dtype):
    if dtype == "bf16":
        return torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


@pytest.mark.parametrize("ci", range(len(META)), ids=[m["name"] for m in META])
def test_golden_sequence(ci):
    from voyager_b200.observer import FusedAmaxObsFakeQuantize

    m = META[ci]
    scheme = "per_channel_symmetric" if m["per_channel"] else "per_tensor_symmetric"
    fq = FusedAmaxObsFakeQuantize("int8", scheme, m["quant_max"], m["history_len"],
                                  ch_axis=m["ch_axis"], force_scale_power_of_two=m["pow2"],
                                  device="cuda")
    for k in range(m["calls"]):
        fq._update_amax_scale(to_dev(DATA[f"c{ci}_x{k}"], m["dtype"]))
        h = fq.amax_history.cpu().numpy()
        s = fq.scale.cpu().numpy()
        assert same_f32(h, DATA[f"c{ci}_h{k}"]), (m["name"], k, "history")
        assert same_f32(s, DATA[f"c{ci}_s{k}"]), (m["name"], k, "scale")


@pytest.mark.parametrize("shape,axis,dtype", [
    ([11008, 4096], 0, "f32"),     # per-output-channel weight: long runs
    ([4096, 11008], 1, "bf16"),    # channel-last: column view
    ([7, 300, 5], 1, "f32"),       # short odd runs
    ([2, 3, 70001], 2, "bf16"),    # channel-last, wide
    ([3, 131, 4097], 0, "f32"),    # unaligned runs
])
def test_per_channel_sizes(shape, axis, dtype):
    from voyager_b200.observer import update_amax_scale

    rng = np.random.default_rng(sum(shape) + axis)
    x = rng.standard_normal(shape).astype(np.float32)
    x *= np.exp2(rng.integers(-8, 8, size=[shape[axis] if i == axis else 1 for i in range(len(shape))]))
    x = x.astype(np.float32)
    xd = f32_to_bf16_bits(x) if dtype == "bf16" else x
    xf = bf16_bits_to_f32(xd) if dtype == "bf16" else x
    C = shape[axis]
    hist = torch.zeros(2, C, device="cuda")
    scale = torch.ones(C, device="cuda")
    h0, s0 = None, None
    for _ in range(2):
        update_amax_scale(to_dev(xd, dtype), hist, scale, 448.0, per_channel=True, ch_axis=axis,
                          power_of_two=True)
        h0, s0 = ob.update_amax_scale(xf, h0, s0, 448.0, per_channel=True, ch_axis=axis,
                                      history_len=2, power_of_two=True)
    assert same_f32(hist.cpu().numpy(), h0.reshape(2, C))
    assert same_f32(scale.cpu().numpy(), s0.reshape(C))


def test_per_tensor_large():
    from voyager_b200.observer import update_amax_scale

    rng = np.random.default_rng(7)
    x = (rng.standard_normal([11008, 4096]) * 0.02).astype(np.float32)
    x[1234, 567] = -3.5
    hist = torch.zeros(1, device="cuda")
    scale = torch.ones((), device="cuda")
    update_amax_scale(to_dev(x, "f32"), hist, scale, 127.0, per_channel=False)
    update_amax_scale(to_dev(x, "f32"), hist, scale, 127.0, per_channel=False)
    assert hist.item() == 3.5
    assert scale.item() == np.float32(np.float32(3.5) / np.float32(127.0))


def test_forward_fake_quant():
    """forward = observe, then quantize / dequantize against the new scale."""
    from voyager_b200.observer import FusedAmaxObsFakeQuantize

    rng = np.random.default_rng(3)
    x = (rng.standard_normal([64, 128]) * 0.5).astype(np.float32)
    fq = FusedAmaxObsFakeQuantize("int8", "per_channel_symmetric", 127.0, 1, ch_axis=0,
                                  device="cuda")
    xt = to_dev(x, "f32")
    fq(xt)  # first call: the scale stays one
    y = fq(xt).cpu().numpy()
    h, s = ob.update_amax_scale(x, None, None, 127.0, per_channel=True, ch_axis=0,
                                history_len=1, power_of_two=False)
    assert s.reshape(-1).tolist() == [1.0] * 64
    _, s = ob.update_amax_scale(x, h, s, 127.0, per_channel=True, ch_axis=0, history_len=1,
                                power_of_two=False)
    qmap = quantization_map("int8")
    want = oops.dequantize(oops.quantize(x, s, qmap=qmap), s)
    assert same_f32(y, want)


def test_errors():
    from voyager_b200.observer import update_amax_scale

    hist = torch.zeros(2, 1, device="cuda")
    scale = torch.ones(1, device="cuda")
    with pytest.raises(RuntimeError, match="empty"):
        update_amax_scale(torch.empty(0, 4, device="cuda"), hist, scale, 1.0, per_channel=False)
    with pytest.raises(ZeroDivisionError):
        update_amax_scale(torch.ones((), device="cuda"), hist, scale, 1.0, per_channel=True,
                          ch_axis=0)
