"""A cross-GPU wait that runs out: the tensor-parallel reduce kernel waits on a flag that no
peer ever sets. It must give up after its bounded wait, record SQ_ERR_TIMEOUT_PEER in the
status word, finish, and leave the context usable (no trap, no hang)."""
import time

import pytest
import torch

from squish_b200._ext import native

pytestmark = pytest.mark.gpu

SQ_ERR_TIMEOUT_PEER = 5


def test_peer_wait_times_out_and_reports(cuda):
    tp, T, N, tiles = 2, 16, 256, 4
    recv = torch.zeros(2 * tp * T * N, dtype=torch.bfloat16, device=cuda)
    flags = torch.zeros(2 * tp * tiles, dtype=torch.int32, device=cuda)  # nobody ever sets these
    out = torch.zeros(T, N, dtype=torch.bfloat16, device=cuda)
    seq = torch.zeros(1, dtype=torch.int32, device=cuda)
    done = torch.zeros(1, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    t0 = time.time()
    native().tp_reduce(recv, tp * T * N, T * N, N, flags, tp * tiles, tiles, 1, out, True, T, N, 16, 128, 2, 1, tp,
                       seq, done, status)
    torch.cuda.synchronize()
    assert int(status.item()) == SQ_ERR_TIMEOUT_PEER
    assert time.time() - t0 < 60
    # the context still works
    x = torch.ones(4, device=cuda)
    assert float((x * 2).sum().item()) == 8.0
