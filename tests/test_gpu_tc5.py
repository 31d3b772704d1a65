"""The 5th-generation tensor-core building blocks against a CPU product.

``gpa_b200_umma_selftest`` runs D = A B on one CTA with tcgen05.mma: bf16 operands in the
shared-memory layouts the scan kernels use (K-major or MN-major, no swizzle), an fp32
accumulator in tensor memory read back with tcgen05.ld, and optionally the A operand brought
in by one bulk (TMA) copy of its pre-tiled image.  Products of bf16 values accumulate exactly
in fp32 up to rounding of the sums, so D must match the fp64 product to ~1e-6.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from gpa_b200 import _lib

pytestmark = pytest.mark.gpu


def _off(r, k, Kd, mn):
    """Byte offset of element (row r, reduction column k) in the shared-memory operand image."""
    inner = (k % 8) * 16 + (r % 8) * 2 if mn else (r % 8) * 16 + (k % 8) * 2
    return (r // 8) * 16 * Kd + (k // 8) * 128 + inner


def _tiled(A, Kd, mn):
    img = torch.zeros(128 * Kd, dtype=torch.bfloat16)
    for r in range(A.shape[0]):
        for k in range(Kd):
            img[_off(r, k, Kd, mn) // 2] = A[r, k]
    return img


BULK_A, LD16 = 1, 2  # GPA_B200_UMMA_BULK_A, GPA_B200_UMMA_LD16

CASES = [  # (M, mma_m, N, Kd, a_mn, b_mn, flags)
    *[(128, 128, 128, 128, a, b, 0) for a in (0, 1) for b in (0, 1)],
    (128, 128, 64, 64, 0, 1, 0), (128, 128, 64, 64, 1, 0, 0),
    (64, 64, 64, 128, 0, 0, 0), (64, 64, 64, 128, 0, 1, 0), (64, 64, 128, 64, 1, 1, 0),
    (64, 128, 256, 64, 0, 1, 0), (48, 128, 16, 16, 1, 1, 0),
    (100, 128, 64, 128, 0, 1, 1), (128, 128, 128, 64, 1, 0, 1),
    # B read through the MN-major view of its own K-major tile (the WY kernel's K tile)
    (64, 64, 128, 64, 0, 2, 0), (64, 64, 64, 64, 0, 2, 0), (128, 128, 128, 64, 1, 2, 0),
    # M = 64 accumulators read back through the 16-lane tcgen05.ld shape
    (64, 64, 64, 128, 0, 0, LD16), (64, 64, 128, 64, 1, 1, LD16), (48, 64, 32, 64, 0, 2, LD16),
]


@pytest.mark.parametrize("M,mma_m,N,Kd,a_mn,b_mn,flags", CASES)
def test_umma_matches_cpu_product(M, mma_m, N, Kd, a_mn, b_mn, flags):
    lib = _lib.load()
    a_bulk = flags & BULK_A
    g = torch.Generator().manual_seed(M * 7 + N * 3 + Kd + 11 * a_mn + 5 * b_mn + flags)
    A = torch.randn(M, Kd, generator=g).bfloat16()
    B = torch.randn(Kd, N, generator=g).bfloat16()
    ref = A.double() @ B.double()
    dA, dB = A.cuda(), B.cuda()
    dT = _tiled(A, Kd, a_mn).cuda() if a_bulk else dA
    D = torch.full((M, N), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.gpa_b200_umma_selftest(M, mma_m, N, Kd, a_mn, b_mn, flags, dA.data_ptr(),
                                    dB.data_ptr(), dT.data_ptr(), D.data_ptr(),
                                    status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "gpa_b200_umma_selftest")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    Dc = D.double().cpu()
    err = float((Dc - ref).norm() / ref.norm())
    # on a mismatch, name which product entry a few outputs hold (a read-layout error shows
    # as a permutation)
    where = [((r, c), divmod(int((ref - Dc[r, c]).abs().argmin()), N))
             for r, c in ((0, 0), (0, 1), (0, 2), (1, 0), (4, 0), (8, 0), (0, 8))
             if err > 1e-6 and r < M and c < N]
    assert err <= 1e-6, (err, where)


def test_no_tensor_core_kernel_timed_out():
    """Every bounded wait of the tensor-core kernels run so far in this process completed."""
    assert _lib.device_status() == 0
