"""The tcgen05 linear layer of the batched decode step (pkv_linear) and its split-sum consumers.

Numerics against a plain PyTorch FP32 reference of the same op
(x.float() @ w.float().T, rounded once to FP16 at the end by the kernel):
every output within one FP16 rounding step plus the FP32 sum-order noise,
atol 1e-3 / rtol 2e-3 on N(0, 1) x N(0, 0.02) operands.  The consumers of
split sums (residual add + RMSNorm, SwiGLU product, the plain sum) must give
bit for bit what the FP16-input kernels give on the summed product, since
they add the splits in the same order and round at the same point.
"""

from __future__ import annotations

import pytest
import torch

from pagedcore_b200 import _lib, kernels
from tests.conftest import cuda_device

pytestmark = pytest.mark.gpu

# The decoder's projections: fused Q/K/V, output, fused gate/up, down, LM head.
SHAPES = [(2560, 2048), (2048, 2048), (11264, 2048), (2048, 5632), (32000, 2048)]


def operands(rows: int, n: int, k: int, seed: int):
    device = cuda_device()
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(rows, k, dtype=torch.float16, device=device, generator=g)
    w = (torch.randn(n, k, dtype=torch.float32, device=device, generator=g) * 0.02).half()
    return x, w


@pytest.fixture(autouse=True)
def _every_row_count_on_the_tcgen05_kernel(monkeypatch):
    # The kernel takes 2-256 rows; kernels.linear sends it only the row counts
    # where it is the faster path.  These tests exercise all of them.
    monkeypatch.setattr(kernels, "TC_MAX_ROWS", 256)


@pytest.mark.parametrize("rows", [2, 17, 64, 256])
@pytest.mark.parametrize("n,k", SHAPES)
def test_linear_matches_an_fp32_reference(rows: int, n: int, k: int) -> None:
    x, w = operands(rows, n, k, seed=rows * 7 + n)
    reference = x.float() @ w.float().T
    got = kernels.linear(x, w)
    assert isinstance(got, torch.Tensor) and got.shape == (rows, n) and got.dtype == torch.float16
    torch.testing.assert_close(got.float(), reference, atol=1e-3, rtol=2e-3)
    # The same layer through its split sums, added by pkv_split_sum.
    sums = kernels.linear(x, w, split_sums=True)
    if isinstance(sums, kernels.SplitSums):
        assert sums.splits == kernels.linear_splits(rows, n, k) > 1
        assert torch.equal(sums.to_half(), got)
    assert int(kernels.linear_error_flag(x.device).item()) == 0


def test_linear_takes_strided_rows_and_rejects_bad_shapes() -> None:
    device = cuda_device()
    x, w = operands(48, 2560, 2048, seed=3)
    wide = torch.zeros(48, 2048 + 64, dtype=torch.float16, device=device)
    wide[:, :2048] = x
    view = wide[:, :2048]  # rows 2112 elements apart
    torch.testing.assert_close(kernels.linear(view, w), kernels.linear(x, w), atol=0, rtol=0)
    flag = kernels.linear_error_flag(device).data_ptr()
    for rows, n, k in ((300, 2560, 2048), (48, 2500, 2048), (48, 2560, 2000)):  # > 256 rows, n % 128, k % 64
        status = _lib.lib.pkv_linear(x.data_ptr(), 2048, w.data_ptr(), rows, n, k, 1, x.data_ptr(), 2560, None, flag,
                                     None)
        assert status == _lib.PKV_VALUE_ERROR


@pytest.mark.parametrize("rows", [3, 200])
def test_split_sum_consumers_equal_the_fp16_path_bit_for_bit(rows: int) -> None:
    device = cuda_device()
    x, w = operands(rows, 2048, 2048, seed=11)
    sums = kernels.linear(x, w, split_sums=True)
    assert isinstance(sums, kernels.SplitSums) and sums.splits > 1
    delta = sums.to_half()
    g = torch.Generator(device=device).manual_seed(12)
    hidden = torch.randn(rows, 2048, dtype=torch.float16, device=device, generator=g)
    weight = (1 + 0.1 * torch.randn(2048, device=device, generator=g)).half()
    hidden_a, hidden_b = hidden.clone(), hidden.clone()
    out_a, out_b = torch.empty_like(hidden), torch.empty_like(hidden)
    kernels.add_rms_norm(hidden_a, sums, weight, out_a)
    kernels.add_rms_norm(hidden_b, delta, weight, out_b)
    assert torch.equal(hidden_a, hidden_b) and torch.equal(out_a, out_b)
    # SwiGLU product from the gate/up layer's split sums.
    xg, wg = operands(rows, 11264, 2048, seed=13)
    gate_up = kernels.linear(xg, wg, split_sums=True)
    assert isinstance(gate_up, kernels.SplitSums)
    assert torch.equal(kernels.silu_mul(gate_up), kernels.silu_mul(gate_up.to_half()))
