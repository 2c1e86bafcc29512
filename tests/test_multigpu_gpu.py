"""The fused all-gather of C over NVLink (sp24_gemm_allgather) on two GPUs.

Each rank computes its column shard of C = A B into its own full-width C and,
with peer stores, into the other rank's; after a barrier both full copies
must equal, bit for bit, the same shards computed on one GPU and placed side
by side (each shard runs the same kernel on either path; whether a shard
also equals the full-width GEMM depends on the kernel and is tested in
test_gemm_gpu.py).
Skipped on a box with fewer than two GPUs.  The ranks are spawned processes
(NCCL for the barrier, CUDA IPC for the peer buffers); no kernel waits on
another rank.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shapes, results):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "sparse-gemm-with-hopper-sptc_b200"))
    import torch.distributed as dist
    import sp24

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    out = []
    try:
        for (m, n, k, outs, align) in shapes:
            g = torch.Generator(device=dev).manual_seed(11)
            a = sp24.prune_2of4(torch.randn((m, k), device=dev, generator=g).to(torch.bfloat16))
            b = torch.randn((k, n), device=dev, generator=g).to(torch.bfloat16)
            ac, meta = sp24.compress(a)
            img = sp24.repack_meta(meta, m, k, torch.bfloat16)
            n0, n1 = sp24.shard_columns(n, world, rank, align)
            full32 = torch.full((m, n), float("nan"), device=dev) if "f32" in outs else None
            full16 = (torch.full((m, n), float("nan"), device=dev, dtype=torch.bfloat16)
                      if "bf16" in outs else None)
            mine = [sp24.ipc_handle(t) if t is not None else None for t in (full32, full16)]
            allh = [None] * world
            dist.all_gather_object(allh, mine)
            opened, peer32, peer16 = {}, [], []   # one mapping per peer allocation
            for r in range(world):
                if r == rank:
                    continue
                for slot, esz, dst in ((0, 4, peer32), (1, 2, peer16)):
                    if allh[r][slot] is not None:
                        handle, off = allh[r][slot]
                        if handle not in opened:
                            opened[handle] = sp24.ipc_open(handle)
                        dst.append(opened[handle] + off + n0 * esz)
            desc = sp24.make_desc(ac, img, b[:, n0:n1], m, n1 - n0, k, meta_format=sp24.META_TC,
                                  c_f32=None if full32 is None else full32[:, n0:n1],
                                  c_bf16=None if full16 is None else full16[:, n0:n1])
            if n1 > n0:
                sp24.gemm_allgather(desc, peer_f32=peer32, peer_bf16=peer16)
            torch.cuda.synchronize()
            dist.barrier()
            ref32 = torch.empty((m, n), device=dev)
            ref16 = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
            for r in range(world):   # every rank's shard, computed here
                s0, s1 = sp24.shard_columns(n, world, r, align)
                if s1 > s0:
                    sp24.gemm(ac, img, b[:, s0:s1].contiguous(), m, s1 - s0, k,
                              meta_format=sp24.META_TC, c_f32=ref32[:, s0:s1],
                              c_bf16=ref16[:, s0:s1])
            torch.cuda.synchronize()
            ok = sp24.last_kernel_status() == 0
            if full32 is not None:
                ok &= torch.equal(full32, ref32)
            if full16 is not None:
                ok &= torch.equal(full16, ref16)
            dist.barrier()
            for base in opened.values():
                sp24.ipc_close(base)
            out.append(bool(ok))
        results[rank] = out
    finally:
        dist.destroy_process_group()


def test_fused_allgather_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    world = 2
    shapes = [(512, 1024, 512, ("f32",), 256), (256, 768, 1024, ("f32", "bf16"), 256),
              (1024, 512, 256, ("bf16",), 256), (384, 4096, 2048, ("f32",), 256),
              (128, 512, 2048, ("f32", "bf16"), 256),   # narrow: split-K, cluster reduce
              # 128 columns per rank: the 128-wide CTA-pair tile (56 row tiles) and
              # its K-split form (16 row tiles), each with peer stores
              (14336, 256, 512, ("f32", "bf16"), 128), (4096, 256, 2048, ("f32", "bf16"), 128)]
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        assert results[r] == [True] * len(shapes), (r, results[r])
