"""The amax observer (``_update_amax_scale``, fake_quantize.py:494-527): the
oracle restatement against the reference's own outputs, and the host side
of the device module (construction, flags, lazy sizing, errors) on CPU."""

import json
import os

import numpy as np
import pytest

from oracle import observer as ob
from oracle.numerics import bf16_bits_to_f32

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


def load_cases():
    with open(os.path.join(GOLD, "observer.json")) as f:
        meta = json.load(f)
    data = np.load(os.path.join(GOLD, "observer.npz"))
    return meta, data


def as_f32(x, dtype):
    return bf16_bits_to_f32(x) if dtype == "bf16" else x.astype(np.float32)


def same_f32(a, b):
    """Equal bit patterns, or both NaN."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb) and np.array_equal(a.view(np.uint32)[~na], b.view(np.uint32)[~nb]))


META, DATA = load_cases()


@pytest.mark.parametrize("ci", range(len(META)), ids=[m["name"] for m in META])
def test_oracle_matches_reference(ci):
    m = META[ci]
    hist, scale = None, None
    for k in range(m["calls"]):
        x = as_f32(DATA[f"c{ci}_x{k}"], m["dtype"])
        hist, scale = ob.update_amax_scale(
            x, hist, scale, m["quant_max"], per_channel=m["per_channel"], ch_axis=m["ch_axis"],
            history_len=m["history_len"], power_of_two=m["pow2"])
        assert same_f32(hist, DATA[f"c{ci}_h{k}"]), (m["name"], k, "history")
        assert same_f32(scale, DATA[f"c{ci}_s{k}"]), (m["name"], k, "scale")


def test_pow2_edges_cover_rounded_log2():
    """The edge set holds inputs whose float32 log2 rounds onto an integer
    (so the ceiling is that integer, not the next one)."""
    ci = [m["name"] for m in META].index("pow2_edges")
    x = DATA[f"c{ci}_x0"].reshape(-1)
    s = DATA[f"c{ci}_s1"].reshape(-1)
    exact_next = np.ldexp(np.float64(1.0), np.floor(np.log2(x.astype(np.float64))).astype(int) + 1)
    not_pow2 = (x.view(np.uint32) & 0x7FFFFF) != 0
    rounded_down = not_pow2 & (s.astype(np.float64) < exact_next) & (x >= np.float32(2.0 ** -126))
    assert rounded_down.sum() > 100


def test_roll_drops_row_one():
    """history = roll(history, -1, 0) then row 0 = amax_cur: with 3 rows the
    old row 1 is the one that leaves."""
    h = np.array([[1.0], [2.0], [3.0]], dtype=np.float32)
    x = np.array([[9.0]], dtype=np.float32)
    h2, s = ob.update_amax_scale(x, h, np.ones((1, 1), np.float32), 1.0, per_channel=True,
                                 ch_axis=0, history_len=3, power_of_two=False)
    assert h2.reshape(-1).tolist() == [9.0, 3.0, 1.0]
    assert s.reshape(-1).tolist() == [3.0]  # from the history before the fold


def test_module_host_side():
    torch = pytest.importorskip("torch")
    from voyager_b200.observer import FusedAmaxObsFakeQuantize

    fq = FusedAmaxObsFakeQuantize("int8", "per_channel_symmetric", 127.0, 4, ch_axis=1)
    assert fq.is_per_channel and fq.scale.tolist() == [1.0] and fq.amax_history.numel() == 0
    with pytest.raises(ValueError):
        FusedAmaxObsFakeQuantize("int8", "microscaling", 127.0, 4)
    fq.disable_observer()
    assert not fq.observer_on() and fq.fake_quant_on()
    fq.freeze_flags()
    fq.enable_observer()
    assert not fq.observer_on()  # frozen
    with pytest.raises(NotImplementedError):  # no CPU path
        FusedAmaxObsFakeQuantize("int8", "per_tensor_symmetric", 127.0, 2)._update_amax_scale(
            torch.ones(4, 4))
