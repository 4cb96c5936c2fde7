"""The driver's entry point smoke() (one small invocation of each hot-path op on cuda:0, checked against the CPU
oracle) runs clean on the GPU, so the suite catches a regression in it before the round-end run does."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available(), reason="no CUDA device")
def test_smoke_entry_point():
    import __graft_entry__
    __graft_entry__.smoke()
