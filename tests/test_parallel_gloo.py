"""Multi-rank logic on CPU ranks (gloo, world size 2): the tensor-parallel
linear's shard / all-gather against the full oracle product, row-sharded
quantize_mx against the unsharded oracle, and the global amax all-reduce.
The local compute is the CPU oracle (the CUDA kernels need a GPU)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (root, os.path.join(root, "voyager-compiler_b200"), here):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import oracle
        from oracle.numerics import quantization_map
        from voyager_b200 import parallel
        from voyager_b200.synth import f32_to_bf16_bits

        rng = np.random.default_rng(7)
        M, K, N = 48, 128, 64
        a = f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
        w = f32_to_bf16_bits((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        qm = quantization_map("fp8_e4m3")
        sa, ca = oracle.quantize_mx(a, qm, [-1], 32, 448.0, True)
        sw, cw = oracle.quantize_mx(w, qm, [-1], 32, 448.0, True)

        def t(x):  # numpy bf16 bits -> torch (as float32 values for transport)
            return torch.from_numpy(oracle.numerics.bf16_bits_to_f32(x).copy())

        def local(x, wsh, b, s):
            # oracle on this rank's weight rows (float32 result)
            wb = f32_to_bf16_bits(wsh.numpy())
            wsb = f32_to_bf16_bits(lin.ws.numpy())
            y = oracle.linear_mx(f32_to_bf16_bits(x.numpy()), wb, None,
                                 input_scale=f32_to_bf16_bits(s.numpy()),
                                 weight_scale=wsb, block_size=32, out_fp32=True)
            return torch.from_numpy(y)

        lin = parallel.NShardedLinear(t(cw), t(sw), local=local)
        y = lin(t(ca), t(sa)).numpy()
        full = oracle.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32,
                                out_fp32=True)
        ok_tp = np.array_equal(y, full)

        # row-sharded quantize_mx: the union of the shards is the full result
        x = f32_to_bf16_bits(rng.standard_normal((37, 64)).astype(np.float32))
        lo, hi = parallel.shard_bounds(37, rank, world)
        s_sh, c_sh = oracle.quantize_mx(x[lo:hi], quantization_map("fp4_e2m1"), [-1], 16, 6.0,
                                        False, quantization_map("fp8_e4m3"))
        s_full, c_full = oracle.quantize_mx(x, quantization_map("fp4_e2m1"), [-1], 16, 6.0,
                                            False, quantization_map("fp8_e4m3"))
        ok_rows = np.array_equal(s_sh, s_full[lo:hi]) and np.array_equal(c_sh, c_full[lo:hi])

        # global amax over shards
        xs = torch.from_numpy(rng.standard_normal(10).astype(np.float32) * (rank + 1))
        g = parallel.global_amax(xs)
        allx = [torch.zeros(10) for _ in range(world)]
        dist.all_gather(allx, xs)
        ok_amax = float(g) == float(torch.cat(allx).abs().max())
        q.put((rank, ok_tp, ok_rows, ok_amax))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_and_row_sharding_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_tp, ok_rows, ok_amax in res:
        assert ok_tp, f"rank {rank}: all-gathered N shards differ from the full product"
        assert ok_rows, f"rank {rank}: row shard differs"
        assert ok_amax, f"rank {rank}: global amax"


def test_shard_bounds():
    from voyager_b200.parallel import shard_bounds

    for n in (0, 1, 7, 11008):
        for w in (1, 2, 3, 8):
            b = [shard_bounds(n, r, w) for r in range(w)]
            assert b[0][0] == 0 and b[-1][1] == n
            assert all(b[i][1] == b[i + 1][0] for i in range(w - 1))


def test_shard_n_rejects_uneven():
    from voyager_b200.parallel import shard_n

    with pytest.raises(ValueError):
        shard_n(torch.zeros(100, 8), None, 0, 8)
    w, s = shard_n(torch.arange(64 * 2).reshape(64, 2).float(), torch.zeros(64, 1), 1, 4)
    assert w.shape == (16, 2) and float(w[0, 0]) == 32.0
