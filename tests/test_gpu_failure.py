"""Failure detection on the GPU without a GPU fault.

* Bounded waits: a one-thread kernel waits on an mbarrier that nothing arrives
  on, with a 1 ms limit.  The wait must give up, record
  (WAIT_TIMEOUT << 16) | site in the device status word and return; the host
  maps the word to ScreeError, and the context stays usable (a normal
  attention call right after it is correct).
* Offsets: the device-side check that the attention schedule kernel runs
  before any attention work (offsets[0] == 0, non-decreasing, offsets[B] == T)
  flags malformed offsets in the status word.  Only the check runs on them:
  no attention, softmax or gather kernel is given bad offsets here.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_reports_and_returns(cuda):
    from scree_b200 import _lib

    lib = _lib.load()
    assert _lib.device_status(reset=True) == 0
    res = torch.full((1,), 7, dtype=torch.int32, device=cuda)
    rc = lib.scree_selftest_wait_timeout(1_000_000, res.data_ptr(), _lib.stream_ptr(cuda))
    _lib.check(rc, "scree_selftest_wait_timeout")
    torch.cuda.synchronize()
    assert int(res.item()) == 0  # the wait gave up instead of completing
    st = _lib.device_status(reset=False)
    assert st == (_lib.DEVERR_WAIT_TIMEOUT << 16) | 99, hex(st)
    with pytest.raises(_lib.ScreeError, match="bounded wait timed out at site 99"):
        _lib.raise_device_status(reset=True)
    assert _lib.device_status(reset=False) == 0
    # The context is still usable: an attention forward right after is correct.
    from scree_b200.kernels.native import varlen_attention_triton

    q = torch.randn((5, 1, 64), device=cuda).to(torch.float16)
    cu = torch.tensor([0, 5], dtype=torch.int32, device=cuda)
    out = varlen_attention_triton(q, q, q, cu, causal=True)
    torch.cuda.synchronize()
    assert torch.equal(out[0], q[0])
    assert _lib.device_status() == 0


def test_selftest_rejects_bad_limits(cuda):
    from scree_b200 import _lib

    lib = _lib.load()
    res = torch.zeros((1,), dtype=torch.int32, device=cuda)
    assert lib.scree_selftest_wait_timeout(0, res.data_ptr(), None) == _lib.SCREE_ERR_INVALID
    assert lib.scree_selftest_wait_timeout(2_000_000_000, res.data_ptr(), None) == _lib.SCREE_ERR_INVALID


@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_offsets_validation_on_device(cuda, dtype):
    from scree_b200 import _lib

    assert _lib.device_status(reset=True) == 0
    good = [0, 3, 3, 10, 17]
    _lib.validate_offsets(torch.tensor(good, dtype=dtype, device=cuda), 17)
    assert _lib.device_status() == 0
    bad_cases = [
        ([1, 3, 10, 17], 17),        # offsets[0] != 0
        ([0, 3, 10, 16], 17),        # offsets[-1] != T
        ([0, 9, 4, 17], 17),         # decreasing
        ([0, 3, 10, 17], 12),        # ends past T
    ]
    big = np.concatenate([[0], np.cumsum(np.ones(5000, dtype=np.int64))])
    big[3001] = big[3000] - 1       # one decreasing step deep in a long array
    bad_cases.append((big.tolist(), int(big[-1])))
    for offs, T in bad_cases:
        _lib.validate_offsets(torch.tensor(offs, dtype=dtype, device=cuda), T)
        st = _lib.device_status(reset=True)
        assert st == (_lib.DEVERR_BAD_INPUT << 16) | 40, (offs[:6], T, hex(st))
