"""Device-side bounded waits: a wait on a flag that nothing sets returns an
error status instead of hanging, and the context stays usable."""
import pytest
import torch

from abacus_b200.ops._ext import check_status, ext
from abacus_b200.utils.fault import check_device

pytestmark = pytest.mark.gpu


def test_wait_on_unset_flag_times_out_with_status():
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    result = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    ext().wait_flag(flag, 1, 200.0, result)
    torch.cuda.synchronize()
    assert result.item() == 0
    assert ext().read_status(torch.cuda.current_device()) == 5
    with pytest.raises(RuntimeError, match="status 5"):
        check_device()
    # Status was cleared by the check; the context still runs kernels.
    check_status()
    ext().set_flag(flag, 1)
    ext().wait_flag(flag, 1, 200.0, result)
    torch.cuda.synchronize()
    assert result.item() == 1
    check_status()
    x = torch.randn(256, 256, device="cuda")
    from abacus_b200.ops import gemm

    torch.testing.assert_close(gemm.matmul(x, x), x @ x, rtol=1e-4, atol=1e-3)
