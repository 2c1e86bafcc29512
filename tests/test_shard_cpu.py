"""N-sharding host logic over two gloo ranks on the CPU: each rank owns the
column block sp24_shard_columns gives it, computes its C shard (here with
the CPU oracle standing in for the GPU), the shards are all-gathered, and
the column-block -> row-major permutation (the same index math as the
library's unshard kernel) rebuilds the full C."""
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
    port = s.getsockname()[1]
    s.close()
    return port


def unshard_reference(flat, m, n, world, spans):
    """Host restatement of unshard_columns_kernel: shard r's block starts at
    element m * n0(r) and is m x (n1 - n0) row-major."""
    out = np.empty((m, n), np.float32)
    for (n0, n1) in spans:
        w = n1 - n0
        out[:, n0:n1] = flat[m * n0: m * n0 + m * w].reshape(m, w)
    return out


def _worker(rank, world, port, m, n, k, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "sparse-gemm-with-hopper-sptc_b200"),
                    os.path.join(root, "oracle")]
    import oracle
    import sp24
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = oracle.Gen(1234)
        a, b, _, _, _ = oracle.host_case(gen, oracle.BF16, m, n, k, False)
        spans = [sp24.shard_columns(n, world, r, 16) for r in range(world)]
        n0, n1 = spans[rank]
        c_shard = oracle.gemm(oracle.BF16, a, np.ascontiguousarray(b[:, n0:n1]))
        # Collectives move equal-sized buffers: every shard is padded to the
        # widest one and trimmed after the gather.
        sizes = [m * (s1 - s0) for s0, s1 in spans]
        mine = torch.zeros(max(sizes))
        mine[:sizes[rank]] = torch.from_numpy(c_shard.reshape(-1))
        gathered = [torch.empty(max(sizes)) for _ in sizes]
        dist.all_gather(gathered, mine)
        if rank == 0:
            flat = torch.cat([g[:sz] for g, sz in zip(gathered, sizes)]).numpy()
            full = unshard_reference(flat, m, n, world, spans)
            q.put(bool(np.array_equal(full, oracle.gemm(oracle.BF16, a, b))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_nshard_allgather_unshard_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 64, 200, 128, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert q.get(timeout=5) is True
