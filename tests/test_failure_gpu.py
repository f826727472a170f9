"""Bounded device waits: a peer flag that nothing sets makes the kernel give up after its time limit (~2 s) and
leave an error code in the status word; the CUDA context stays usable.  Both "ranks" live on one GPU in one
kernel (no kernel waits for another launch)."""
import time

import pytest
import torch

from inference_optimizations_b200.parallel import health as HL

pytestmark = pytest.mark.gpu


def _peers(cuda, nbytes):
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda) for _ in range(2)]
    return bufs, torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=cuda)


def test_ep_barrier_gives_up_on_a_silent_peer(cuda):
    from inference_optimizations_b200._ext import ext
    bufs, peers = _peers(cuda, 256)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    t0 = time.time()
    ext().ep_barrier(peers, 0, 0, 2, epoch, status)       # rank 0 of 2; rank 1 never signals
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(status.item()) == 4 and dt < 15, (int(status.item()), dt)
    with pytest.raises(HL.DeviceWaitTimeout):
        HL.check_status([status])
    x = torch.randn(4096, device=cuda)
    assert torch.isfinite((x * 2).sum()).item()          # context still usable


def test_dcp_merge_gives_up_on_a_silent_peer(cuda):
    from inference_optimizations_b200._ext import ext
    T_max, H = 2, 128
    half = T_max * H * (1024 + 4)
    bufs, peers = _peers(cuda, 2 * half + 256)
    epoch = torch.tensor([1, 0], dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.zeros(1, H // 2, 512, dtype=torch.bfloat16, device=cuda)
    t0 = time.time()
    ext().dcp_merge(peers, 0, 2 * half, 1, T_max, H, 0, 2, 0, epoch, out, None, status)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(status.item()) == 4 and dt < 15, (int(status.item()), dt)
    y = torch.ones(16, device=cuda).cumsum(0)
    assert float(y[-1]) == 16.0
