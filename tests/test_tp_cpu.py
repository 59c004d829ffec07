"""Host-side tensor-parallel logic on CPU with world_size-2 gloo process groups:
the column / row sharding of quantized tensors (no re-quantization) reproduces
the unsharded quantized matmul once the row-parallel partials are summed, and
the handle exchange used to bootstrap the P2P group returns every rank's blob
in rank order."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from vmlx_b200_loader import load_package
        import oracle
        vm = load_package()
        rng = np.random.default_rng(0)  # same weights on every rank
        H, K, gs = 256, 512, 64
        W = oracle.f32_to_bf16(rng.normal(0, 0.02, (H, K)).astype(np.float32))
        wq, s, b = oracle.quantize(W, gs, 4)
        x = oracle.f32_to_bf16(rng.normal(0, 1, (3, K)).astype(np.float32))
        full = oracle.qmm_f64(x, wq, s, b, gs, 4)
        # row-parallel: slice K at whole groups, partial matmul, all-sum
        t = lambda a: torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a.view(np.int16))  # noqa: E731
        wq_r = vm.llama.shard_k(t(wq), rank, world).numpy().view(np.uint32)
        s_r = vm.llama.shard_k(t(s), rank, world).numpy().view(np.uint16)
        b_r = vm.llama.shard_k(t(b), rank, world).numpy().view(np.uint16)
        kb = K // world
        part = oracle.qmm_f64(np.ascontiguousarray(x[:, rank * kb:(rank + 1) * kb]), np.ascontiguousarray(wq_r),
                              np.ascontiguousarray(s_r), np.ascontiguousarray(b_r), gs, 4)
        pt = torch.from_numpy(part)
        dist.all_reduce(pt)
        row_ok = np.allclose(pt.numpy(), full, rtol=1e-9, atol=1e-9)
        # column-parallel with segments (q | k | v style): concat of the ranks' rows == full rows
        segs = [128, 64, 64]
        wq_c = vm.llama.shard_rows(t(wq), rank, world, segs)
        gathered = [torch.empty_like(wq_c) for _ in range(world)]
        dist.all_gather(gathered, wq_c)
        rows, off = [], 0  # rebuild each segment from the ranks' blocks
        for seg in segs:
            blk = seg // world
            rows += [gathered[r][off:off + blk] for r in range(world)]
            off += blk
        col_ok = torch.equal(torch.cat(rows), t(wq))
        # handle exchange in rank order
        blobs = vm.distributed.Group._torch_exchange(bytes([rank]) * 64)
        ex_ok = [bb[0] for bb in blobs] == list(range(world))
        q.put((rank, row_ok, col_ok, ex_ok))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None, None))


def test_tp_sharding_and_exchange_gloo_world2():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, row_ok, col_ok, ex_ok in res:
        assert row_ok is True, (rank, row_ok)
        assert col_ok and ex_ok, (rank, col_ok, ex_ok)
