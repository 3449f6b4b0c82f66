"""Failure paths on one GPU, made on the host (needs a B200; nothing faults on the GPU).

* Every wait inside the persistent pass kernel is bounded. A test hook makes one grid barrier wait
  for an arrival that never comes (with a short poll limit): the wait runs out, the kernel releases
  its tensor memory and returns, the call fails with LS_ERR_DEVICE, the cache is unchanged, and the
  model keeps working (its next results equal those of a model that never failed). This is the
  error-as-a-value rule of the reference (src/model.rs:142-158, src/spec.rs:65-80).
* A damaged model file is an I/O error at open in both residency modes (the stream mode reads the
  whole file into pinned host memory at open, so no layer read can fail in the middle of a pass;
  the reference's mid-pass Source errors, tests/pipeline.rs:170-198, have no counterpart there).
"""

import os

import numpy as np
import pytest

import fixtures as F
import layerstream_b200 as ls
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():
    d = F.TempDir("gpu-fail").path
    F.write_tiny_model(d, 17)
    p = os.path.join(d, "q8g32.lsq")
    O.quantize_model(d, p, (8, 32), (8, 32), clip=True)
    yield p


def test_a_grid_barrier_wait_that_runs_out_fails_the_call_and_the_model_recovers(tiny):
    g, ref = ls.Model(tiny, max_ctx=128), ls.Model(tiny, max_ctx=128)
    assert g.info.persistent_pass == 1
    g.forward(F.PROMPT)
    ref.forward(F.PROMPT)
    L = g.info.layers
    # after the embedding, inside the first and the last layer, after the LM head
    for barrier in (1, 3, 1 + 5 * (L - 1) + 4, 1 + 5 * L + 1):
        g.inject_stall(barrier)
        with pytest.raises(ls.LayerstreamError) as e:
            g.verify([5, 6, 7])
        assert e.value.code == -4, e.value
        assert "grid barrier" in str(e.value)
        assert g.pos == len(F.PROMPT)
    a, b = g.forward([9]), ref.forward([9])
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert g.verify([int(np.argmax(a)), 1, 2]) == ref.verify([int(np.argmax(b)), 1, 2])
    with pytest.raises(ls.LayerstreamError):
        g.inject_stall(1 + 5 * L + 2)  # no such barrier
    g.close()
    ref.close()


def test_a_damaged_model_file_is_an_io_error_in_both_modes(tiny):
    data = open(tiny, "rb").read()
    cut = tiny + ".cut"
    with open(cut, "wb") as f:
        f.write(data[: len(data) - 4096])
    for mode in ("resident", "stream"):
        with pytest.raises(ls.LayerstreamError) as e:
            ls.Model(cut, mode=mode, slots=2)
        assert e.value.code == -2, (mode, e.value)
    os.remove(cut)
