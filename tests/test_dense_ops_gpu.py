"""Fused decoder-step kernels (csrc/dense_ops.cu) against the eager ops they replace.

``add_rms_norm`` is the residual add followed by dense.rms_norm, and
``silu_mul`` is SwiGLU's product (F.silu(gate) * up), each with the same FP16
rounding points.  The residual add must match bit for bit.  The norm sums
its squares in another order than torch's reduction; a last-bit difference
in the FP32 scale can move the normalised value by one FP16 ulp, which the
weight multiply (rounded again) can turn into two, on rare elements.  The
SiLU product uses expf and IEEE division in FP32 as torch's kernel does, and
is checked to one ulp.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from pagedcore_b200 import kernels
from pagedcore_b200.dense import rms_norm
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu


def ulp_close(actual: torch.Tensor, expected: torch.Tensor, ulps: int = 1) -> None:
    a = actual.view(torch.int16).int()
    b = expected.view(torch.int16).int()
    assert int((a - b).abs().max()) <= ulps
    assert float((a == b).float().mean()) > 0.99


@pytest.mark.parametrize("rows", [1, 7, 256])
def test_add_rms_norm_matches_the_eager_residual_add_and_norm(rows) -> None:
    device = cuda_device()
    generator = torch.Generator(device=device).manual_seed(rows)
    hidden = torch.randn(rows, 2048, dtype=torch.float16, device=device, generator=generator)
    delta = torch.randn(rows, 2048, dtype=torch.float16, device=device, generator=generator)
    weight = (1 + 0.1 * torch.randn(2048, device=device, generator=generator)).half()
    expected_hidden = hidden + delta
    expected = rms_norm(expected_hidden, weight)
    out = torch.empty_like(hidden)
    kernels.add_rms_norm(hidden, delta, weight, out)
    assert torch.equal(hidden, expected_hidden)  # the residual add, in place
    ulp_close(out, expected, ulps=2)
    # Without delta: the norm alone, hidden untouched.
    before = hidden.clone()
    kernels.add_rms_norm(hidden, None, weight, out)
    assert torch.equal(hidden, before)
    ulp_close(out, rms_norm(before, weight), ulps=2)


@pytest.mark.parametrize("rows, inter", [(64, 32), (64, 5632), (1, 5632), (2047, 5632), (3, 37)])
def test_silu_mul_matches_the_eager_swiglu_product(rows, inter) -> None:
    # 16-byte chunks when inter is a multiple of 8, one value a thread otherwise (37).
    device = cuda_device()
    generator = torch.Generator(device=device).manual_seed(inter + rows)
    gate_up = 3 * torch.randn(rows, 2 * inter, dtype=torch.float16, device=device, generator=generator)
    gate, up = gate_up.chunk(2, -1)
    ulp_close(kernels.silu_mul(gate_up), F.silu(gate) * up)


def test_silu_mul_pairs_equal_the_one_value_path_bit_for_bit() -> None:
    """The 16-byte path multiplies two values at once in FP16 (the FP32 product
    of two FP16 values is exact, so its FP16 rounding is the FP16 multiply);
    the one-value path, taken for operands off 16-byte alignment, rounds the
    FP32 product.  Both must give the same bits."""
    device = cuda_device()
    generator = torch.Generator(device=device).manual_seed(5)
    rows, inter = 300, 5632
    buffer = torch.empty(rows * 2 * inter + 1, dtype=torch.float16, device=device)
    buffer[1:] = 3 * torch.randn(rows * 2 * inter, dtype=torch.float16, device=device, generator=generator)
    unaligned = buffer[1:].view(rows, 2 * inter)
    assert unaligned.data_ptr() % 16
    aligned = unaligned.clone()
    assert aligned.data_ptr() % 16 == 0
    assert torch.equal(kernels.silu_mul(aligned), kernels.silu_mul(unaligned))


def test_fused_ops_reject_bad_shapes() -> None:
    device = cuda_device()
    hidden = torch.zeros(2, 2048, dtype=torch.float16, device=device)
    with pytest.raises(ValueError, match="weight"):
        kernels.add_rms_norm(hidden, None, torch.zeros(1024, dtype=torch.float16, device=device), hidden.clone())
    with pytest.raises(ValueError, match="gate_up"):
        kernels.silu_mul(torch.zeros(2, 7, dtype=torch.float16, device=device))


def gemv(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor) -> None:
    """pkv_gemv through the C ABI, whatever kernels.linear would dispatch."""
    from pagedcore_b200._lib import check, lib

    check(lib.pkv_gemv(x.data_ptr(), x.stride(0), weight.data_ptr(), x.shape[0], weight.shape[0], x.shape[1],
                       out.data_ptr(), out.stride(0), torch.cuda.current_stream().cuda_stream))


def sums_close(actual: torch.Tensor, expected: torch.Tensor) -> None:
    """Same FP32 products summed in another order, each rounded once to FP16:
    within 4 FP16 ulps (or 1e-5 near zero, where the sign may flip), and equal
    for nearly all elements."""
    torch.testing.assert_close(actual.float(), expected.float(), atol=1e-5, rtol=4 * 2.0**-10)
    assert float((actual == expected).float().mean()) > 0.99


@pytest.mark.parametrize("rows", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("n, k", [(2560, 2048), (2048, 5632), (31, 2048), (32000, 2048)])
def test_gemv_matches_the_fp32_product_rounded_once(rows, n, k) -> None:
    device = cuda_device()
    generator = torch.Generator(device=device).manual_seed(rows * 7 + n)
    x = torch.randn(rows, k, dtype=torch.float16, device=device, generator=generator)
    weight = (0.02 * torch.randn(n, k, device=device, generator=generator)).half()
    expected = (x.float() @ weight.float().T).half()
    actual = torch.empty(rows, n, dtype=torch.float16, device=device)
    gemv(x, weight, actual)  # the kernel itself, for every row count it takes
    sums_close(actual, expected)
    torch.testing.assert_close(actual, torch.nn.functional.linear(x, weight), atol=2e-3, rtol=2e-3)


def test_gemv_takes_strided_rows_and_leaves_other_shapes_to_the_library() -> None:
    device = cuda_device()
    generator = torch.Generator(device=device).manual_seed(3)
    wide = torch.randn(4, 2560, dtype=torch.float16, device=device, generator=generator)
    x = wide[:, 512:]  # rows 2560 elements apart
    weight = (0.02 * torch.randn(96, 2048, device=device, generator=generator)).half()
    actual = torch.empty(4, 96, dtype=torch.float16, device=device)
    gemv(x, weight, actual)
    sums_close(actual, (x.float() @ weight.float().T).half())
    one = x[:1]
    sums_close(kernels.linear(one, weight), (one.float() @ weight.float().T).half())  # one row: the kernel
    many = torch.randn(9, 2048, dtype=torch.float16, device=device, generator=generator)  # the library GEMM
    assert torch.equal(kernels.linear(many, weight), torch.nn.functional.linear(many, weight))
    with pytest.raises(ValueError, match="1 to 8 rows"):
        gemv(many, weight, torch.empty(9, 96, dtype=torch.float16, device=device))


@pytest.mark.parametrize("rows", [512, 2047])
def test_add_rms_norm_of_a_prompt_equals_the_small_batch_kernel_bit_for_bit(rows) -> None:
    """From 512 rows the norm runs one warp per row; it sums the squares in the
    order of the kernel used below 512 rows, so the same rows normalised in
    batches of 256 give the same bits (the residual add in place, and out)."""
    device = cuda_device()
    generator = torch.Generator(device=device).manual_seed(rows + 1)
    hidden = torch.randn(rows, 2048, dtype=torch.float16, device=device, generator=generator)
    delta = torch.randn(rows, 2048, dtype=torch.float16, device=device, generator=generator)
    weight = (1 + 0.1 * torch.randn(2048, device=device, generator=generator)).half()
    for with_delta in (True, False):
        whole, parts = hidden.clone(), hidden.clone()
        out_whole, out_parts = torch.empty_like(hidden), torch.empty_like(hidden)
        kernels.add_rms_norm(whole, delta if with_delta else None, weight, out_whole)
        for begin in range(0, rows, 256):
            end = min(begin + 256, rows)
            kernels.add_rms_norm(parts[begin:end], delta[begin:end] if with_delta else None, weight,
                                 out_parts[begin:end])
        assert torch.equal(whole, parts) and torch.equal(out_whole, out_parts)
        if with_delta:
            assert torch.equal(whole, hidden + delta)
        ulp_close(out_whole, rms_norm(whole, weight), ulps=2)
