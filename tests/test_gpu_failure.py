"""Failure detection on the GPU without a fault: the bounded mbarrier wait used by the
TMA-staged kernels, and the decode step's wait for another CTA's bytes, give up after
their poll budget, record MOC_STATUS_WAIT_TIMEOUT in the device status word, and return;
the CUDA context stays usable."""
from __future__ import annotations

import pytest
import torch

from moc import _lib

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_not_hung():
    lib = _lib.load()
    _lib.device_status(clear=True)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.moc_wait_timeout_probe(2000, stream), "moc_wait_timeout_probe")
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) & 1
    assert _lib.device_status() == 0
    t = torch.arange(8, device="cuda", dtype=torch.float32)
    assert t.sum().item() == 28.0  # context still healthy


def test_cluster_wait_timeout_is_reported_not_hung():
    lib = _lib.load()
    _lib.device_status(clear=True)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.moc_cluster_wait_timeout_probe(2000, stream), "moc_cluster_wait_timeout_probe")
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) & 1
    assert _lib.device_status() == 0
    t = torch.arange(8, device="cuda", dtype=torch.float32)
    assert t.sum().item() == 28.0  # context still healthy


def test_normal_kernels_record_no_timeouts():
    from moc import MoC

    _lib.device_status(clear=True)
    m = MoC(256, 256, 4, 16).cuda().bfloat16()
    x = torch.randn(2, 512, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    z = torch.randn(2, 512, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y, _ = m(x, z)
    y.float().sum().backward()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0


def test_allreduce_wait_timeout_is_reported_not_hung():
    """The NVLink all-reduce kernel as rank 0 of two ranks whose rank 1 never calls: every
    wait for rank 1's flag gives up after the given poll limit and records the timeout."""
    lib = _lib.load()
    _lib.device_status(clear=True)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.moc_comm_wait_timeout_probe(4000, stream), "moc_comm_wait_timeout_probe")
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) & 1
    assert _lib.device_status() == 0
    t = torch.arange(8, device="cuda", dtype=torch.float32)
    assert t.sum().item() == 28.0  # context still healthy
