"""The C ABI from several host threads at once.

A fresh process (so no kernel has been launched yet and every per-device
first-call set-up is still to run) starts four threads behind a barrier;
each makes its first sp24_gemm calls on the same device with a different
kernel family (CTA pair, single CTA, split K, narrow CTA pair), each on its
own stream, then the results are compared bit for bit with the same calls
made one after another in the main thread.
"""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = textwrap.dedent(r"""
    import sys, threading
    sys.path.insert(0, sys.argv[1])
    import torch, sp24
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    # (m, n, k, tile_n): CTA pair; single CTA (BlockN 64 forced); split K; narrow pair
    shapes = [(512, 512, 1024, 0), (256, 512, 512, 64), (256, 16, 4096, 0), (4096, 96, 512, 0)]
    inputs = []
    g = torch.Generator(device=dev).manual_seed(5)
    for (m, n, k, t) in shapes:
        a = sp24.prune_2of4(torch.randn((m, k), device=dev, generator=g).to(torch.bfloat16))
        b = torch.randn((k, n), device=dev, generator=g).to(torch.bfloat16)
        ac, meta = sp24.compress(a)
        img = sp24.repack_meta(meta, m, k, torch.bfloat16)
        inputs.append((ac, img, b, m, n, k, t))
    torch.cuda.synchronize()
    barrier = threading.Barrier(len(inputs))
    results = [None] * len(inputs)
    errors = []

    def work(i):
        try:
            ac, img, b, m, n, k, t = inputs[i]
            s = torch.cuda.Stream(device=dev)
            barrier.wait()
            outs = []
            for _ in range(3):
                c, _ = sp24.gemm(ac, img, b, m, n, k, meta_format=sp24.META_TC, tile_n=t, stream=s)
                outs.append(c)
            s.synchronize()
            results[i] = outs
        except Exception as e:   # reported below
            errors.append(repr(e))

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(inputs))]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    for i, (ac, img, b, m, n, k, t) in enumerate(inputs):
        c, _ = sp24.gemm(ac, img, b, m, n, k, meta_format=sp24.META_TC, tile_n=t)
        torch.cuda.synchronize()
        for got in results[i]:
            assert torch.equal(got, c), i
    assert sp24.last_kernel_status() == 0
    print("THREADS OK")
""")


def test_first_calls_from_four_threads():
    pkg = os.path.join(ROOT, "sparse-gemm-with-hopper-sptc_b200")
    out = subprocess.run([sys.executable, "-c", SCRIPT, pkg], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert "THREADS OK" in out.stdout
