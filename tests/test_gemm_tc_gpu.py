"""The tcgen05 tensor-core GEMM (vkllm_b200_gemm_f16, the kernel behind VKLLM_OP_MATMUL for fp16
M > 1) against a plain PyTorch fp32 reference of the same op: C = act(scale * A . B^T), fp16 out.

Shapes: the BASELINE prefill GEMMs (M 512 x (N, K) in {(4096, 4096), (11008, 4096), (4096, 11008)}),
the batched-decode M = 64, odd tails in M, N and K (TMA zero fill), SiLU and a scale. Tolerance, per
element: two fp16 ulps of |ref| (the output rounding) plus 2 K 2^-24 sum_k |a_ik| |b_jk| |scale| (the
standard bound on fp32 accumulation error in any summation order, for ours and the reference's;
x1.1 under SiLU, whose slope is below 1.1). The kernel's sticky error word must stay 0 (no bounded wait expired)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def run_gemm(vk, torch, M, N, K, scale=1.0, act=0, lda=None, ldb=None, ldc=None, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    lda, ldb, ldc = lda or K, ldb or K, ldc or N
    A = (torch.rand((M, lda), generator=g, device="cuda") * 2 - 1).half()
    B = (torch.rand((N, ldb), generator=g, device="cuda") * 2 - 1).half()
    Cm = torch.full((M, ldc), float("nan"), device="cuda", dtype=torch.float16)
    s = torch.cuda.current_stream().cuda_stream
    err = vk.lib().vkllm_b200_gemm_f16(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), M, N, K, lda, ldb, ldc, scale, act, s)
    assert err == vk.OK
    torch.cuda.synchronize()
    assert vk.lib().vkllm_b200_gemm_f16_error() == 0
    ref = (A[:, :K].float() @ B[:, :K].float().T) * scale
    if act:
        ref = ref / (1.0 + torch.exp(-ref))
    mag = (A[:, :K].float().abs() @ B[:, :K].float().abs().T) * abs(scale)
    acc_tol = 2 * K * 2.0 ** -24 * mag * (1.1 if act else 1.0)  # ours plus the fp32 reference's own
    return Cm[:, :N].float(), ref, Cm, acc_tol


def check(got, ref, acc_tol):
    import torch

    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(2.0 ** -14))) - 10)
    tol = 2 * ulp + acc_tol
    bad = (got - ref).abs() > tol
    assert not bool(bad.any()), (f"{int(bad.sum())} of {bad.numel()} off; max diff {(got - ref).abs().max().item()}, "
                                 f"max diff / tol {((got - ref).abs() / tol).max().item()}")


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (128, 128, 128), (512, 4096, 4096), (512, 11008, 4096),
                                   (512, 4096, 11008), (64, 4096, 4096), (33, 65, 264), (300, 1000, 1032),
                                   (1, 512, 512), (700, 384, 96)])
def test_gemm_matches_torch_fp32(vk, torch_cuda, M, N, K):
    got, ref, _, tol = run_gemm(vk, torch_cuda, M, N, K, seed=M + N + K)
    check(got, ref, tol)


def test_gemm_scale_and_silu(vk, torch_cuda):
    got, ref, _, tol = run_gemm(vk, torch_cuda, 200, 520, 320, scale=0.125, act=1, seed=5)
    check(got, ref, tol)


def test_gemm_strided_operands_leave_padding_untouched(vk, torch_cuda):
    got, ref, Cm, tol = run_gemm(vk, torch_cuda, 96, 200, 128, lda=136, ldb=144, ldc=208, seed=9)
    check(got, ref, tol)
    assert bool(torch_cuda.isnan(Cm[:, 200:]).all())  # columns past N are not written


def test_gemm_rejects_unaligned_k(vk, torch_cuda):
    lib = vk.lib()
    buf = torch_cuda.zeros(4096, device="cuda", dtype=torch_cuda.float16)
    p = buf.data_ptr()
    assert lib.vkllm_b200_gemm_f16(p, p, p, 4, 4, 12, 12, 12, 4, 1.0, 0, None) == vk.ARGS  # K % 8 != 0


@pytest.mark.parametrize("tile,splits,M,N,K", [("256x192", "1", 512, 12288, 4096), ("256x192", "2", 300, 1000, 1032),
                                               ("256x160", "1", 512, 2200, 512), ("256x160", "3", 700, 384, 960),
                                               ("256x224", "1", 512, 3200, 512), ("256x224", "2", 260, 500, 264)])
def test_gemm_wave_fitting_tiles(vk, torch_cuda, monkeypatch, tile, splits, M, N, K):
    """The 256-row tiles of 192, 160 and 224 columns (two accumulators of 128 rows, tensor memory
    rounded up to 512 columns), forced, with and without split K and with ragged M, N, K."""
    monkeypatch.setenv("VKLLM_B200_GEMM_TILE", tile)
    monkeypatch.setenv("VKLLM_B200_GEMM_SPLITS", splits)
    got, ref, _, tol = run_gemm(vk, torch_cuda, M, N, K, seed=M + N + K + 1)
    check(got, ref, tol)


@pytest.mark.parametrize("tile,splits,M,N,K", [("128x256a64", "1", 64, 4096, 4096), ("128x256a64", "3", 64, 12288, 4096),
                                               ("128x128a64", "2", 33, 1000, 1032), ("128x128a64", "1", 1, 512, 512),
                                               ("128x256a64", "4", 48, 700, 11008)])
def test_gemm_tiles_loading_64_rows_of_a(vk, torch_cuda, monkeypatch, tile, splits, M, N, K):
    """128-row tiles that load only 64 rows of A per stage (M <= 64: batched decode), forced, with and
    without split K; the MMA's upper 64 rows read other staged data and are never stored."""
    monkeypatch.setenv("VKLLM_B200_GEMM_TILE", tile)
    monkeypatch.setenv("VKLLM_B200_GEMM_SPLITS", splits)
    got, ref, _, tol = run_gemm(vk, torch_cuda, M, N, K, seed=M + N + K + 2)
    check(got, ref, tol)
