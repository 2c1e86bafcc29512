"""sp24_gemm_multi: the N-sharded GEMM over the GPUs of one process, from one
host thread, through the C ABI.

A_c and the metadata image are replicated with sp24_replicate; B and C are
per device, as whole matrices (SP24_MULTI_FULL) or as each device's column
block (SP24_MULTI_SHARD).  Every device's columns must equal, bit for bit,
the same column block computed by sp24_gemm on one GPU (same shard width, so
the same kernel), and C must meet the row-norm bound against the CPU oracle
on sampled rows.  With the fused all-gather every device's full C holds all
columns once the call's streams are synchronised.  The one-GPU cases run on
any box; the two-GPU cases skip on a box with fewer GPUs.
"""
import numpy as np
import pytest
import torch

import oracle
import sp24

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _case(ndev, m, n, k, outs, b_layout, c_layout, allgather):
    devs = [torch.device("cuda", i) for i in range(ndev)]
    g = torch.Generator(device=devs[0]).manual_seed(m + 3 * n + 7 * k)
    a = sp24.prune_2of4(torch.randn((m, k), device=devs[0], generator=g).to(torch.bfloat16))
    b = torch.randn((k, n), device=devs[0], generator=g).to(torch.bfloat16)
    ac0, meta0 = sp24.compress(a)
    img0 = sp24.repack_meta(meta0, m, k, torch.bfloat16)
    acs = [ac0] + [torch.empty_like(ac0, device=d) for d in devs[1:]]
    imgs = [img0] + [torch.empty_like(img0, device=d) for d in devs[1:]]
    torch.cuda.synchronize(devs[0])
    sp24.replicate(ac0, acs)
    sp24.replicate(img0, imgs)
    shards = [sp24.shard_columns(n, ndev, r, 256) for r in range(ndev)]
    if b_layout == sp24.MULTI_FULL:
        bs = [b.to(d) for d in devs]
    else:
        bs = [b[:, n0:n1].contiguous().to(d) for (n0, n1), d in zip(shards, devs)]

    def out(dt):
        if c_layout == sp24.MULTI_FULL:
            return [torch.full((m, n), float("nan"), device=d, dtype=dt) for d in devs]
        return [torch.full((m, n1 - n0), float("nan"), device=d, dtype=dt)
                for (n0, n1), d in zip(shards, devs)]

    c32 = out(torch.float32) if "f32" in outs else None
    c16 = out(torch.bfloat16) if "bf16" in outs else None
    for d in devs:
        torch.cuda.synchronize(d)
    md = sp24.make_multi_desc(m, n, k, torch.bfloat16, acs, imgs, bs, c_f32=c32, c_bf16=c16,
                              b_layout=b_layout, c_layout=c_layout)
    keep = sp24.gemm_multi(md, allgather)
    for d in devs:
        torch.cuda.synchronize(d)
    del keep
    assert sp24.last_kernel_status() == 0

    # Each column block against sp24_gemm of the same block on device 0.
    with torch.cuda.device(devs[0]):
        blocks32, blocks16 = [], []
        for (n0, n1) in shards:
            if n1 == n0:          # more devices than 256-column blocks: this one idles
                blocks32.append(None)
                blocks16.append(None)
                continue
            r32, r16 = sp24.gemm(ac0, img0, b[:, n0:n1], m, n1 - n0, k, meta_format=sp24.META_TC,
                                 out_f32="f32" in outs, out_bf16="bf16" in outs)
            blocks32.append(r32)
            blocks16.append(r16)
        torch.cuda.synchronize()
    for gi in range(ndev):
        owned = [gi] if not allgather else range(ndev)
        for r in owned:
            n0, n1 = shards[r]
            if n1 == n0:
                continue
            for got, want in ((c32, blocks32), (c16, blocks16)):
                if got is None:
                    continue
                view = got[gi][:, n0:n1] if c_layout == sp24.MULTI_FULL else got[gi]
                assert torch.equal(view.to(devs[0]), want[r]), (gi, r)
    # Oracle on 16 seeded rows of the assembled C.
    full = torch.cat([x for x in blocks32 if x is not None], dim=1) if c32 is not None else \
        torch.cat([x.float() for x in blocks16 if x is not None], dim=1)
    rows = np.sort(np.random.default_rng(m).choice(m, min(m, 16), replace=False))
    a_bits, b_bits = _bits(a)[rows], _bits(b)
    ref = oracle.gemm(1, a_bits, b_bits, threads=8)
    err = oracle.row_norm_rel_error(full[rows].cpu().numpy(), ref, oracle.to_float(1, a_bits),
                                    oracle.to_float(1, b_bits))
    assert err <= (1e-2 if c32 is not None else 2e-2), err


@pytest.mark.parametrize("outs,b_layout,c_layout,allgather", [
    (("f32",), sp24.MULTI_FULL, sp24.MULTI_FULL, False),
    (("f32", "bf16"), sp24.MULTI_SHARD, sp24.MULTI_SHARD, False),
    (("bf16",), sp24.MULTI_FULL, sp24.MULTI_FULL, True),
])
def test_gemm_multi_one_gpu(outs, b_layout, c_layout, allgather):
    _case(1, 512, 768, 512, outs, b_layout, c_layout, allgather)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("m,n,k,outs,b_layout,c_layout,allgather", [
    (512, 1024, 512, ("f32",), sp24.MULTI_FULL, sp24.MULTI_FULL, False),
    (1000, 700, 256, ("f32", "bf16"), sp24.MULTI_SHARD, sp24.MULTI_SHARD, False),
    (512, 1024, 512, ("f32",), sp24.MULTI_FULL, sp24.MULTI_FULL, True),
    (768, 1280, 1024, ("f32", "bf16"), sp24.MULTI_SHARD, sp24.MULTI_FULL, True),
    (256, 96, 2048, ("bf16",), sp24.MULTI_FULL, sp24.MULTI_FULL, True),
])
def test_gemm_multi_two_gpus(m, n, k, outs, b_layout, c_layout, allgather):
    _case(2, m, n, k, outs, b_layout, c_layout, allgather)
