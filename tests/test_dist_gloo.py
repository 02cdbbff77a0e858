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


def _layer_worker(rank, world, port, A, Wt, rname, out_q):
    """One rank of the weight-split layer (``dist.cast_weight_split``), with
    the CPU oracle standing in for the CUDA kernels: 1/world of the
    activation's rows and the rank's W^T shard reduce into two amax words,
    one all-reduce(MAX) of both, then the rank's C[:, n0:n1]."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import cast as ocast
        from breccia_b200.types import Float8CurrentScaling, MXFP8BlockScaling
        r = {"current": Float8CurrentScaling(), "mxfp8": MXFP8BlockScaling()}[rname]
        n0, n1 = shard_rows(Wt.shape[0], world, rank)
        w = Wt[n0:n1]
        if rname == "current":
            lo, hi = shard_rows(A.shape[0], world, rank)

            def word(x):
                v = float(np.max(np.abs(x))) if x.size else 0.0
                return int(np.array(np.float32(v)).view(np.int32))
            words = torch.tensor([word(A[lo:hi]), word(w)], dtype=torch.int32)
            allreduce_amax_word(words)  # one collective for both words
            amax_a, amax_w = [float(np.array(v, dtype=np.int32).view(np.float32))
                              for v in words.numpy()]
            qa = ocast.cast_per_tensor_fp8(A, r, amax=max(amax_a, 1e-10))
            qw = ocast.cast_per_tensor_fp8(w, r, amax=max(amax_w, 1e-10))
        else:
            qa, qw = ocast.cast(A, r), ocast.cast(w, r)  # rank-local: blocks run along K
        c = ocast.matmul(qa, ocast.dequantize(qw).T)
        out_q.put((rank, n0, n1, c, qw.data, np.asarray(qw.scale)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rname", ["current", "mxfp8"])
def test_weight_split_shards_concatenate_to_full_result(rname):
    """The shards' C[:, n0:n1] concatenated along N equal the unsharded
    oracle matmul bit for bit, and every shard's codes and scales equal the
    rows [n0, n1) of the full weight cast (per-tensor: the same global
    scale on every rank)."""
    from oracle import cast as ocast
    from breccia_b200.types import Float8CurrentScaling, MXFP8BlockScaling
    r = {"current": Float8CurrentScaling(), "mxfp8": MXFP8BlockScaling()}[rname]
    rng = np.random.default_rng(3)
    A = rng.standard_normal((96, 256)).astype(np.float32)
    A[70, 9] = 40.0  # the activation's amax sits in the second rank's rows
    Wt = (rng.standard_normal((384, 256)) * 0.02).astype(np.float32)
    Wt[300, 1] = 0.9  # and the weight's in the second rank's shard
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_layer_worker, args=(k, world, port, A, Wt, rname, q))
             for k in range(world)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=120) for _ in range(world)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0][1] == 0 and results[-1][2] == Wt.shape[0]
    qa, qw = ocast.cast(A, r), ocast.cast(Wt, r)
    full = ocast.matmul(qa, ocast.dequantize(qw).T)
    np.testing.assert_array_equal(np.concatenate([t[3] for t in results], axis=1), full)
    for _, n0, n1, _, codes, scale in results:
        np.testing.assert_array_equal(codes, qw.data[n0:n1])
        want = qw.scale if rname == "current" else qw.scale[n0:n1]
        np.testing.assert_array_equal(np.atleast_1d(scale).view(np.uint8),
                                      np.atleast_1d(np.asarray(want)).view(np.uint8))
