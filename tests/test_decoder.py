"""Decoder stack host logic on CPU, with the oracle as the quantized ops:
shapes and sharding rules, and the tensor-parallel split (gloo, 2 ranks)
against the single-device forward.

Tolerance of the split: the row-parallel o_proj / down products are rounded
to bf16 per rank and summed by the reduce-scatter, where one device rounds
the full float32 sum once; that moves values by about one bf16 ulp, and a
moved value can land on the other side of an E4M3 rounding boundary
downstream.  Measured rel-L2 of the 2-layer output is ~1e-3; the bound is
1e-2."""

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from voyager_b200.decoder import Decoder, DecoderConfig, init_weights

SMALL = DecoderConfig(layers=2, hidden=256, heads=2, ffn=512)
BATCH, SEQ = 2, 64


def _inputs(cfg, seed=3):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((BATCH, SEQ, cfg.hidden), generator=g).bfloat16()


def _single():
    from _oracle_ops import OracleOps

    ops = OracleOps()
    w = init_weights(SMALL, 11, "cpu")
    return Decoder(SMALL, w, table=ops.table(), ops=ops)(_inputs(SMALL))


def test_flops_c5():
    # 4 layers of hidden 4096 / ffn 11008 at B=8, S=2048: 28.72 TFLOP
    c = DecoderConfig()
    assert abs(c.flops(8, 2048) / 1e12 - 28.72) < 0.01


def test_oracle_forward_shape_and_finite():
    y = _single()
    assert y.shape == (BATCH, SEQ, SMALL.hidden) and y.dtype == torch.bfloat16
    assert torch.isfinite(y.float()).all()


def test_rejects_unaligned_shards():
    from _oracle_ops import OracleOps

    ops = OracleOps()
    cfg = DecoderConfig(layers=1, hidden=256, heads=2, ffn=520)  # 520 % 32 != 0
    w = init_weights(cfg, 1, "cpu")

    class FakeTP:
        pass

    from voyager_b200 import decoder as D

    tp = D.TensorParallel()
    tp.world, tp.rank = 2, 0
    with pytest.raises(ValueError):
        D.DecoderLayer(cfg, w[0], ops.table(), ops, tp)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "voyager-compiler_b200"), here):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from _oracle_ops import OracleOps

        ops = OracleOps()
        w = init_weights(SMALL, 11, "cpu")
        dec = Decoder(SMALL, w, table=ops.table(), ops=ops)
        y = dec(_inputs(SMALL))
        q.put((rank, y.view(torch.int16).numpy().copy()))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_2_ranks_matches_single():
    from _oracle_ops import rel_l2

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(out[r], str), out[r]
    y0 = torch.from_numpy(out[0]).view(torch.bfloat16)
    y1 = torch.from_numpy(out[1]).view(torch.bfloat16)
    assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))  # gathered output
    want = _single()
    assert rel_l2(y0, want) < 1e-2, rel_l2(y0, want)


def test_pad_k_chunks_layout():
    """The column-parallel down projection's K layout: per-rank chunks of the
    ffn padded to 128 with zeros, products unchanged."""
    from voyager_b200.tp import pad_k_chunks

    w = torch.arange(3 * 1376 * 2, dtype=torch.float32).reshape(3, 2 * 1376)
    p = pad_k_chunks(w, 2)
    assert p.shape == (3, 2 * 1408)
    assert torch.equal(p[:, :1376], w[:, :1376]) and torch.equal(p[:, 1408:2784], w[:, 1376:])
    assert not p[:, 1376:1408].any() and not p[:, 2784:].any()
    a = torch.randn(5, 2 * 1376)
    ap = pad_k_chunks(a, 2)
    assert torch.allclose(a @ w.T, ap @ p.T)
