"""Tensor parallel on 2 GPUs (NCCL over NVLink) against the single-GPU
result: the N-sharded linear_mx (bit-identical) and the decoder stack
(Megatron split with sequence-parallel norms; rel-L2 <= 1e-2, since the
row-parallel products are rounded to bf16 per rank before the
reduce-scatter sums them); skipped with fewer than two GPUs."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import datetime
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "voyager-compiler_b200"), here):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import torch.distributed as dist

    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import voyager_b200  # noqa: F401
        from voyager_b200 import parallel
        from voyager_b200.tables import get_quantization_map

        g = torch.Generator(device="cpu").manual_seed(3)
        a = torch.randn(256, 1024, generator=g).bfloat16().to(dev)
        w = (torch.randn(2048, 1024, generator=g) * 0.02).bfloat16().to(dev)
        Q = torch.ops.quantized_ops
        e4m3 = get_quantization_map("fp8_e4m3", dev)
        sa, ca = Q.quantize_mx(a, e4m3, [-1], 32, 448.0, True)
        sw, cw = Q.quantize_mx(w, e4m3, [-1], 32, 448.0, True)
        full = Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
        lin = parallel.NShardedLinear(cw, sw)
        y = lin(ca, sa)
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(y, full)), tuple(y.shape)))
    finally:
        dist.destroy_process_group()


def test_nsharded_linear_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same, shape in res:
        assert shape == (256, 2048)
        assert same, f"rank {rank}: TP result differs from the single-GPU product"


def _decoder_worker(rank, world, port, q):
    import datetime
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "voyager-compiler_b200"), here):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import torch.distributed as dist

    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import voyager_b200  # noqa: F401
        from voyager_b200.decoder import Decoder, DecoderConfig, init_weights

        cfg = DecoderConfig(layers=2, hidden=512, heads=4, ffn=1024)
        w = init_weights(cfg, 21, dev)
        g = torch.Generator(device=dev).manual_seed(5)
        x = torch.randn((2, 256, cfg.hidden), generator=g, device=dev).bfloat16()
        y = Decoder(cfg, w)(x)
        y1 = Decoder(cfg, w, parallel=False)(x)
        torch.cuda.synchronize()
        rel = float((y.float() - y1.float()).norm() / y1.float().norm())
        ys = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(ys, y)
        same = all(torch.equal(ys[0], t) for t in ys)
        q.put((rank, rel, same, tuple(y.shape)))
    finally:
        dist.destroy_process_group()


def test_decoder_tensor_parallel_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decoder_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, rel, same, shape in res:
        assert shape == (2, 256, 512)
        assert same, "ranks disagree on the gathered output"
        assert rel < 1e-2, f"rank {rank}: rel-L2 {rel} against the single-GPU stack"
