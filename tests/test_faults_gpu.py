"""Failure detection on the device without faulting the GPU: a bounded wait
for a flag that no peer ever writes must give up (about 2 s), record a status
code the host turns into an exception, and leave the CUDA context usable."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_missing_peer_times_out_cleanly(cuda):
    from mod_b200.ops import check_status, load_extension, native
    from mod_b200.parallel.ep import ExchangeBuffer

    C = load_extension()
    check_status()                             # start clean
    N, cap, H, El = 1, 16, 256, 4
    buf = ExchangeBuffer(C.ep_buffer_bytes(N, cap, H))
    state = torch.zeros(8 + N, dtype=torch.int32, device=cuda)   # epoch 0 -> waits for flag >= 1
    row_pos = torch.empty(N * cap, dtype=torch.int32, device=cuda)
    offs = torch.empty(El + 1, dtype=torch.int32, device=cuda)
    abort = torch.zeros(1, dtype=torch.int32, device=cuda)
    t0 = time.time()
    C.ep_recv_only(buf.peers, state, 0, cap, El, H, row_pos, offs, abort)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert 1.0 < dt < 30.0
    assert int(abort.item()) == 1
    with pytest.raises(RuntimeError, match="peer flag wait timed out"):
        check_status()
    # the context still works
    x = torch.randn(8, 256, device=cuda).bfloat16()
    w = torch.randn(128, 256, device=cuda).bfloat16()
    torch.testing.assert_close(native.linear(x, w).float(), x.float() @ w.float().t(), rtol=3e-2, atol=3e-1)
    check_status()
    buf.close()
