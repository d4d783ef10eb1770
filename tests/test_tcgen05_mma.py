"""One-tile tcgen05 GEMMs: every operand arrangement the attention kernels use
(A in smem or TMEM, B K-major or MN-major, bf16 via kind::f16, fp32 via
kind::tf32) against a PyTorch fp32 matmul of the same operands.

tf32 operands are only used K-major: an MN-major tf32 operand needs the
128-byte swizzle with 32-byte atoms, so the fp32 path stores V transposed
instead."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _tf32(x):
    # round-to-nearest tf32 so the tensor core sees exactly these values
    b = x.contiguous().view(torch.int32)
    b = (b + 0x1000) & ~0x1FFF
    return b.view(torch.float32)


CASES = [
    # dtype, N, K, a_in_tmem, b_mn_major
    (torch.bfloat16, 128, 64, False, False),
    (torch.bfloat16, 128, 128, False, False),
    (torch.bfloat16, 64, 64, False, False),
    (torch.float32, 128, 32, False, False),
    (torch.float32, 64, 64, False, False),
    (torch.bfloat16, 128, 64, True, False),
    (torch.bfloat16, 128, 64, True, True),
    (torch.bfloat16, 128, 128, True, True),
    (torch.float32, 128, 64, True, False),
    (torch.bfloat16, 128, 64, False, True),
]


@pytest.mark.parametrize("dtype,N,K,a_tmem,b_mn", CASES)
def test_umma_tile(ext, cuda_device, dtype, N, K, a_tmem, b_mn):
    g = torch.Generator(device="cpu").manual_seed(1234 + N + K)
    A = torch.randn(128, K, generator=g)
    Bt = torch.randn(N, K, generator=g)  # logical B^T: [N, K]
    if dtype == torch.float32:
        A, Bt = _tf32(A), _tf32(Bt)
    else:
        A, Bt = A.to(dtype), Bt.to(dtype)
    ref = A.float() @ Bt.float().T
    Bdev = (Bt.T.contiguous() if b_mn else Bt.contiguous()).to(cuda_device)
    D = torch.full((128, N), float("nan"), device=cuda_device)
    status = torch.zeros(8, dtype=torch.int32, device=cuda_device)
    ext.umma_selftest(A.contiguous().to(cuda_device), Bdev, D, a_tmem, b_mn, status)
    torch.cuda.synchronize()
    assert int(status[0]) == 0, f"device status {status.tolist()}"
    err = (D.cpu() - ref).abs().max().item()
    assert err < 1e-3 * max(1.0, ref.abs().max().item()), f"max err {err}"
