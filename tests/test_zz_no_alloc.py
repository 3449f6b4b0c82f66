"""The allocation-free GEMV entry point against the device GEMV entry point (GPU).

ls_qgemv_rows_noalloc reads the stored rows straight from a device buffer the caller owns and keeps
its K-split partial sums in a fixed per-GPU array; ls_qgemv_device runs the verify-path GEMV on
planes uploaded by ls_qweights_upload. Both compute y = W x for the same stored rows, so their
outputs agree within the tolerance the GEMV parity tests use for the tensor-core path.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def stored_rows(bits, group, rows, cols, seed):
    """Random stored rows (.lsq row format) with bf16 scales near 1e-2."""
    rb = cols * bits // 8 + cols // group * 2
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(rows, rb), dtype=np.uint8)
    sc = raw[:, cols * bits // 8:].view(np.uint16)
    sc[:] = (0x3C23 + rng.integers(-64, 64, size=sc.shape)).astype(np.uint16)  # bf16 ~ 1e-2
    return np.ascontiguousarray(raw.reshape(-1))


def tolerance(want):
    return 2e-3 * np.sqrt(np.mean(want**2)) + 2e-3 * np.abs(want)


@pytest.mark.parametrize("bits,group,rows,cols,M", [(4, 32, 1152, 896, 9), (8, 64, 896, 4864, 5), (4, 16, 9728, 896, 16)])
def test_allocation_free_gemv_matches_the_device_gemv_on_two_calls(bits, group, rows, cols, M):
    import torch

    import layerstream_b200 as ls

    torch.cuda.set_device(0)
    raw = stored_rows(bits, group, rows, cols, seed=rows + M)
    w = ls.QWeights(bits, group, raw, rows, cols)
    raw_dev = torch.from_numpy(raw).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = torch.randn(M, cols, device="cuda", generator=torch.Generator("cuda").manual_seed(call))
        want = torch.empty(M, rows, device="cuda")
        got = torch.full((M, rows), float("nan"), device="cuda")
        w.gemv(x.data_ptr(), M, want.data_ptr(), stream)
        ls.qgemv_rows_noalloc(bits, group, raw_dev.data_ptr(), rows, cols, x.data_ptr(), M, got.data_ptr(), stream)
        torch.cuda.synchronize()
        want_h, got_h = want.cpu().numpy(), got.cpu().numpy()
        assert np.all(np.isfinite(got_h)), call
        assert np.all(np.abs(got_h - want_h) <= tolerance(want_h)), (call, float(np.max(np.abs(got_h - want_h))))


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
