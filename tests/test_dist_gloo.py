"""Multi-rank host logic on CPU (gloo, world size 2): the weight-shard split
and the global-amax reduction that makes a sharded per-tensor cast equal the
single-GPU cast. The per-rank encode here is the CPU oracle standing in for
the CUDA kernels; the GPU path runs the same reduction in bench.py --gpus N."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from breccia_b200.dist import shard_rows, allreduce_amax_word


def test_shard_rows_cover_and_align():
    for n, world in ((8192, 8), (28672, 8), (4096, 3), (100, 4), (0, 2)):
        spans = [shard_rows(n, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        for (a, b), (c, d) in zip(spans, spans[1:]):
            assert b == c
        for lo, hi in spans:
            assert hi == lo or lo % 128 == 0  # non-empty shards start 128-aligned


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, x_full, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import codec
        n = x_full.shape[0]
        lo, hi = shard_rows(n, world, rank)
        shard = x_full[lo:hi]
        local = float(np.max(np.abs(shard))) if shard.size else 0.0
        word = torch.tensor([int(np.array(np.float32(local)).view(np.int32))], dtype=torch.int32)
        allreduce_amax_word(word)
        amax = float(np.array(word.numpy()[0], dtype=np.int32).view(np.float32))
        scale = np.float32(max(amax, 1e-10) / 448.0)
        codes = codec.encode_e4m3(shard / scale)
        out_q.put((rank, lo, hi, codes, scale))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("with_nan", [False, True])
def test_sharded_per_tensor_cast_equals_full_cast(with_nan):
    from oracle import cast as ocast
    from breccia_b200.types import Float8CurrentScaling
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((300, 64)) * np.exp2(rng.integers(-4, 4, (300, 1)))).astype(np.float32)
    x[217, 5] = 900.0  # the global amax sits in the second shard
    if with_nan:
        x[10, 3] = np.nan
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, x, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = ocast.cast(x, Float8CurrentScaling())
    got = np.concatenate([r[3] for r in results], axis=0)
    np.testing.assert_array_equal(got, full.data)
    for r in results:
        assert np.array_equal(np.float32(r[4]).view(np.uint32), full.scale.view(np.uint32)) or \
            (np.isnan(r[4]) and np.isnan(full.scale))
