"""The allocation-free GEMV entry point (GPU).

Some hosts cannot let this library call cudaMalloc: their device memory belongs to another
allocator (a framework that reserves most of HBM at start-up and hands out slices of it) or to a
fixed budget (an embedded runtime), and a library allocation could fail, escape their accounting or
synchronize the device in the middle of their pipeline. ls_qgemv_rows_noalloc serves them: it reads
the stored rows, the activations and the result from buffers the caller owns, and keeps its K-split
partial sums in a fixed 4 MiB per-GPU array inside the library.

Checked here, on two calls in a row (the second call finds the first one's partials in the shared
array): the output against the CPU oracle's kernels::matmul (src/kernels.rs:196-203) at the tight
bound of the f32 CUDA-core path, 1e-4 * (1 + |y|), and against the device GEMV entry point at the
tensor-core tolerance; a matrix whose columns are one group (three of the four K slices are empty
and must contribute zeros); the first call on a fresh device in a new process; and the size limit.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def stored_rows(bits, group, rows, cols, seed):
    """Random stored rows (.lsq row format) with bf16 scales near 1e-2."""
    rb = cols * bits // 8 + cols // group * 2
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(rows, rb), dtype=np.uint8)
    sc = raw[:, cols * bits // 8:].view(np.uint16)
    sc[:] = (0x3C23 + rng.integers(-64, 64, size=sc.shape)).astype(np.uint16)  # bf16 ~ 1e-2
    return np.ascontiguousarray(raw.reshape(-1))


def tc_tolerance(want):
    return 2e-3 * np.sqrt(np.mean(want**2)) + 2e-3 * np.abs(want)


@pytest.mark.parametrize("bits,group,rows,cols,M", [(4, 32, 1152, 896, 9), (8, 64, 896, 4864, 5), (4, 16, 9728, 896, 16),
                                                    (4, 16, 16, 16, 1), (8, 16, 40, 16, 3)])
def test_allocation_free_gemv_matches_the_cpu_path_on_two_calls(bits, group, rows, cols, M):
    import torch

    import layerstream_b200 as ls
    from oracle import oracle as O

    torch.cuda.set_device(0)
    raw = stored_rows(bits, group, rows, cols, seed=rows + M)
    w = ls.QWeights(bits, group, raw, rows, cols) if cols % 64 == 0 else None  # the device GEMV takes 64-column blocks
    raw_dev = torch.from_numpy(raw).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = torch.randn(M, cols, device="cuda", generator=torch.Generator("cuda").manual_seed(call))
        dev_gemv = torch.empty(M, rows, device="cuda")
        got = torch.full((M, rows), float("nan"), device="cuda")
        if w is not None:
            w.gemv(x.data_ptr(), M, dev_gemv.data_ptr(), stream)
        ls.qgemv_rows_noalloc(bits, group, raw_dev.data_ptr(), rows, cols, x.data_ptr(), M, got.data_ptr(), stream)
        torch.cuda.synchronize()
        got_h, dev_h = got.cpu().numpy(), dev_gemv.cpu().numpy()
        want = O.matmul(bits, group, raw, rows, cols, x.cpu().numpy())
        assert np.all(np.isfinite(got_h)), call
        assert np.all(np.abs(got_h - want) <= 1e-4 * (1 + np.abs(want))), (call, float(np.max(np.abs(got_h - want))))
        if w is not None:
            assert np.all(np.abs(got_h - dev_h) <= tc_tolerance(dev_h)), call


FRESH = r"""
import sys
sys.path[:0] = [sys.argv[1]]
import numpy as np, torch
import layerstream_b200 as ls
from oracle import oracle as O
torch.cuda.set_device(0)
rows, cols, M = 300, 512, 4
rng = np.random.default_rng(3)
raw = rng.integers(0, 256, size=(rows, cols // 2 + cols // 32 * 2), dtype=np.uint8)
raw[:, cols // 2:].view(np.uint16)[:] = (0x3C23 + rng.integers(-64, 64, size=(rows, cols // 32))).astype(np.uint16)
raw = np.ascontiguousarray(raw.reshape(-1))
raw_dev = torch.from_numpy(raw).cuda()
for call in range(2):  # the first call on this device looks up the array's address
    x = torch.randn(M, cols, device="cuda", generator=torch.Generator("cuda").manual_seed(call))
    y = torch.full((M, rows), float("nan"), device="cuda")
    ls.qgemv_rows_noalloc(4, 32, raw_dev.data_ptr(), rows, cols, x.data_ptr(), M, y.data_ptr())
    torch.cuda.synchronize()
    want = O.matmul(4, 32, raw, rows, cols, x.cpu().numpy())
    assert np.all(np.abs(y.cpu().numpy() - want) <= 1e-4 * (1 + np.abs(want))), call
print("fresh ok")
"""


def test_the_first_call_on_a_fresh_device_sets_up_the_array():
    r = subprocess.run([sys.executable, "-c", FRESH, ROOT], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "fresh ok" in r.stdout, r.stdout + r.stderr


def test_allocation_free_gemv_rejects_requests_beyond_its_scratch():
    import torch

    import layerstream_b200 as ls

    torch.cuda.set_device(0)
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(16, 896, device="cuda")
    y = torch.zeros(16, 64, device="cuda")
    # 16 x 151936 partial rows exceed the fixed array: rejected before any kernel runs
    with pytest.raises(ls.LayerstreamError, match="static scratch"):
        ls.qgemv_rows_noalloc(4, 32, buf.data_ptr(), 151936, 896, x.data_ptr(), 16, y.data_ptr())
    with pytest.raises(ls.LayerstreamError, match="1..16 token rows"):
        ls.qgemv_rows_noalloc(4, 32, buf.data_ptr(), 64, 896, x.data_ptr(), 17, y.data_ptr())
