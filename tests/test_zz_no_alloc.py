"""hf_cuda_argmax_noalloc: the argmax for callers that must not allocate device
memory (a host application that owns all device memory and hands the library
ready buffers, or a latency-budgeted thread such as an audio callback, where
cudaMalloc/cudaFree may synchronise the device). Its candidate scratch is a
fixed file-scope device array instead of a per-call allocation.

Checked through the C-ABI against the allocating entry point, hf_cuda_argmax,
on two calls in a row with different shapes (so the second call runs over the
first call's leftovers in the shared scratch), exactly: an argmax is an index.
Collected last, so a failure here comes after every other test has run.
"""
import numpy as np
import pytest

import oracle_bindings as ob
from huggingfaceeacp_b200 import native

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _rows(rows, length, seed):
    logits = ob.spread_values(rows * length, seed, 4.0).reshape(rows, length)
    logits[:, length // 3] = 50.0           # a tie the lowest index must win...
    logits[:, 2 * length // 3] = 50.0
    logits[rows // 2, length - 1] = 80.0    # ...and one row with the winner at the end
    mask = np.zeros(length, dtype=np.float32)
    mask[7] = 1.0
    mask[length // 3] = 1.0 if seed % 2 else 0.0
    return np.ascontiguousarray(logits, dtype=np.float32), mask


def test_no_alloc_argmax_matches_the_allocating_entry_point_on_two_calls():
    lib = native.cuda()
    with native.Context(native.SMALL_INT8) as ctx:
        for rows, length, seed in ((3, 256000, 1), (17, 50000, 2)):
            logits, mask = _rows(rows, length, seed)
            expected = ctx.argmax(logits, mask)
            d_logits = torch.from_numpy(logits).cuda()
            d_mask = torch.from_numpy(mask).cuda()
            d_out = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
            rc = lib.hf_cuda_argmax_noalloc(d_logits.data_ptr(), d_mask.data_ptr(), rows, length, d_out.data_ptr(),
                                            None)
            torch.cuda.synchronize()
            assert rc == native.HF_OK
            np.testing.assert_array_equal(d_out.cpu().numpy().view(np.uint32), expected)


def test_no_alloc_argmax_refuses_more_candidates_than_its_scratch_holds():
    lib = native.cuda()
    rows, length = 129, 256000  # 129 rows x 64 candidates > 8192
    d_logits = torch.zeros(rows * length, device="cuda")
    d_out = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    rc = lib.hf_cuda_argmax_noalloc(d_logits.data_ptr(), None, rows, length, d_out.data_ptr(), None)
    torch.cuda.synchronize()
    assert rc == native.HF_E_CAPACITY
    assert torch.all(d_out == -1)
