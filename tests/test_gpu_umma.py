"""The tcgen05 building block of the prefill kernel against a float32 host matmul."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("N,K", [(64, 64), (128, 64), (64, 128), (128, 128)])
def test_umma_selftest(mode, N, K):
    from nifre_b200 import _lib
    g = torch.Generator().manual_seed(N + K + mode)
    A = torch.randn(128, K, generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, generator=g).to(torch.bfloat16) if mode == 0 else \
        torch.randn(K, N, generator=g).to(torch.bfloat16)
    ref = A.float() @ (B.float().t() if mode == 0 else B.float())
    Ad, Bd = A.cuda(), B.cuda()
    C = torch.full((128, N), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(_lib.load().nf_selftest_umma(Ad.data_ptr(), Bd.data_ptr(), C.data_ptr(), N, K, mode,
                                            status.data_ptr(), _lib.stream_handle(torch.device("cuda"))),
               "nf_selftest_umma")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    torch.testing.assert_close(C.cpu(), ref, rtol=1e-4, atol=1e-3)
