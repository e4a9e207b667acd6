"""Device-side failure detection without a GPU fault: a peer wait on a flag that nothing ever
sets must give up after its clock64 bound, record the peer-timeout code in the device error
word, return, and leave the context usable."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from flextensor_b200.ops import api as ops  # noqa: E402
from flextensor_b200.ops import native  # noqa: E402

DEV = torch.device("cuda", 0)
K_ERR_PEER_TIMEOUT = 3


def test_unset_peer_flag_times_out_and_context_survives():
    assert native.device_error(reset=True) == 0
    flags = [torch.zeros(2, dtype=torch.int64, device=DEV) for _ in range(2)]
    acks = [torch.zeros(2, dtype=torch.int64, device=DEV) for _ in range(2)]
    t0 = time.time()
    # rank 0 waits for rank 1's acknowledgement of epoch 5: no one will ever write it
    native.lib().p2p_wait_acks_raw([f.data_ptr() for f in flags], [a.data_ptr() for a in acks], 0, 1, 0, 5)
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert native.device_error(reset=True) == K_ERR_PEER_TIMEOUT
    assert waited < 15.0, f"bounded wait took {waited:.1f}s"
    # the context is intact: a kernel launched afterwards runs and is correct
    a = torch.randn(256, 128, device=DEV).bfloat16()
    w = torch.randn(64, 128, device=DEV).bfloat16()
    y = ops.linear(a, w, None, epi="none")
    torch.cuda.synchronize()
    assert native.device_error(reset=True) == 0
    assert float((y.float() - a.float() @ w.float().t()).abs().max()) < 0.5
