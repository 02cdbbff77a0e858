"""Weight-split layer on 2 GPUs (one process per GPU, NCCL), against one GPU.

Each rank holds the whole activation and rows [n0, n1) of W^T, casts both
through ``dist.cast_weight_split`` (per-tensor recipes: one all-reduce(MAX)
of two amax words) and computes its C[:, n0:n1]. Codes and scales must equal
the single-GPU casts bit for bit; the concatenated C must equal the
single-GPU GEMM up to float32 summation order (the shard may take a
different GEMM kernel shape). ``cast_matmul_weight_split`` (the activation's
cast fused into the GEMM) must equal ``cast_weight_split`` + ``linear`` on
each rank bit for bit. Skipped where fewer than 2 GPUs are visible.
"""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RECIPES = ("current", "mxfp8", "nvfp4")


def _recipe(name):
    import breccia_b200 as bb
    return {"current": bb.Float8CurrentScaling(), "mxfp8": bb.MXFP8BlockScaling(),
            "nvfp4": bb.NVFP4BlockScaling()}[name]


def _inputs():
    g = torch.Generator().manual_seed(17)
    A = torch.randn(2048, 1024, generator=g)
    A[1500, 7] = 60.0  # the activation amax sits in the second rank's share of rows
    Wt = torch.randn(4096, 1024, generator=g) * 0.02
    Wt[3000, 3] = 1.5  # the weight amax in the second rank's shard
    return A.to(torch.bfloat16), Wt.to(torch.bfloat16)


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        import breccia_b200 as bb
        from breccia_b200.dist import shard_rows, cast_weight_split, cast_matmul_weight_split
        A, Wt = _inputs()
        n0, n1 = shard_rows(Wt.shape[0], world, rank)
        for name in RECIPES:
            sa, sw = cast_weight_split(A.to(dev), Wt[n0:n1].to(dev), _recipe(name))
            c = bb.linear(sa, sw, out_dtype=torch.float32)
            # the same step with the activation's cast fused into the GEMM
            cf, saf, swf = cast_matmul_weight_split(A.to(dev), Wt[n0:n1].to(dev), _recipe(name),
                                                    out_dtype=torch.float32, fused=True)
            torch.cuda.synchronize()
            fused_same = bool(torch.equal(cf.view(torch.int32), c.view(torch.int32)) and
                              torch.equal(saf.data.view(torch.uint8), sa.data.view(torch.uint8)) and
                              torch.equal(swf.data.view(torch.uint8), sw.data.view(torch.uint8)))
            q.put((name, rank, n0, n1, c.cpu().numpy(),
                   sw.data.view(torch.uint8).cpu().numpy(), sw.scale.cpu().numpy(),
                   sa.scale.cpu().numpy(), fused_same))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


def test_weight_split_two_gpus_equals_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import breccia_b200 as bb
    world = 2
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world * len(RECIPES))]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    A, Wt = _inputs()
    for name in RECIPES:
        r = _recipe(name)
        sa, sw = bb.cast(A.cuda(), r), bb.cast(Wt.cuda(), r)
        full = bb.linear(sa, sw, out_dtype=torch.float32).cpu().numpy()
        codes = sw.data.view(torch.uint8).cpu().numpy()
        scale = sw.scale.cpu().numpy()
        parts = sorted((t for t in got if t[0] == name), key=lambda t: t[1])
        c = np.concatenate([t[4] for t in parts], axis=1)
        assert np.abs(c - full).max() <= 1e-6 * np.abs(full).max(), name
        for _, _, n0, n1, _, sh_codes, sh_scale, a_scale, fused_same in parts:
            assert fused_same, name
            assert np.array_equal(sh_codes, codes[n0:n1]), name
            want = scale if name == "current" else scale[n0:n1]
            assert np.array_equal(np.atleast_1d(sh_scale).view(np.uint8),
                                  np.atleast_1d(want).view(np.uint8)), name
            assert np.array_equal(np.atleast_1d(a_scale).view(np.uint8),
                                  np.atleast_1d(sa.scale.cpu().numpy()).view(np.uint8)), name
