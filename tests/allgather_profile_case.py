"""The fused all-gather on two GPUs of one process, as a small case to profile:
sp24_gemm_multi with allgather_c over 2 devices, bf16 4096 x (2 x 512) x 1024
(each device's GEMM is 4096 x 512 x 1024 and sends its 8 MiB fp32 block to the
other device over NVLink).  Runs `reps` calls and checks both gathered copies
against the same blocks computed by sp24_gemm on device 0 (bit for bit).
Used by the profile recipe in profiles/sp24_gemm_allgather_nvlink.md:

    python tests/allgather_profile_case.py
    ncu --metrics gpu__time_duration.sum,nvltx__bytes.sum,nvlrx__bytes.sum,\\
        dram__bytes_read.sum,dram__bytes_write.sum --clock-control none \\
        -k regex:sp24_gemm2sm -s 2 -c 1 python tests/allgather_profile_case.py
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "sparse-gemm-with-hopper-sptc_b200"))

import torch  # noqa: E402

import sp24  # noqa: E402


def main(reps: int = 4) -> None:
    if torch.cuda.device_count() < 2:
        raise SystemExit("needs two GPUs")
    m, n, k = 4096, 1024, 1024
    devs = [torch.device("cuda", 0), torch.device("cuda", 1)]
    g = torch.Generator(device=devs[0]).manual_seed(21)
    a = sp24.prune_2of4(torch.randn((m, k), device=devs[0], generator=g).to(torch.bfloat16))
    b = torch.randn((k, n), device=devs[0], generator=g).to(torch.bfloat16)
    ac0, meta0 = sp24.compress(a)
    img0 = sp24.repack_meta(meta0, m, k, torch.bfloat16)
    acs = [ac0, torch.empty_like(ac0, device=devs[1])]
    imgs = [img0, torch.empty_like(img0, device=devs[1])]
    torch.cuda.synchronize(devs[0])
    sp24.replicate(ac0, acs)
    sp24.replicate(img0, imgs)
    bs = [b, b.to(devs[1])]
    cs = [torch.full((m, n), float("nan"), device=d) for d in devs]
    for d in devs:
        torch.cuda.synchronize(d)
    md = sp24.make_multi_desc(m, n, k, torch.bfloat16, acs, imgs, bs, c_f32=cs)
    for _ in range(reps):
        sp24.gemm_multi(md, allgather_c=True)
    for d in devs:
        torch.cuda.synchronize(d)
    with torch.cuda.device(devs[0]):
        for n0, n1 in (sp24.shard_columns(n, 2, r, 256) for r in range(2)):
            want, _ = sp24.gemm(ac0, img0, b[:, n0:n1], m, n1 - n0, k, meta_format=sp24.META_TC)
            torch.cuda.synchronize()
            for c in cs:
                assert torch.equal(c[:, n0:n1].to(devs[0]), want)
    print("allgather profile case ok")


if __name__ == "__main__":
    main()
