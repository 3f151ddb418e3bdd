"""Kernel building blocks against plain PyTorch fp32 references (B200 only)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

from foldforge_b200 import _lib, kernels  # noqa: E402


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert _lib.device_error() == 0


@pytest.mark.parametrize("rows,c,dtype", [(128 * 128, 128, torch.bfloat16), (13, 128, torch.bfloat16),
                                          (1, 128, torch.bfloat16), (500, 384, torch.bfloat16),
                                          (777, 128, torch.float32), (64, 384, torch.float32)])
def test_layernorm(rows, c, dtype):
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(rows, c, device="cuda", generator=g) * 2 + 0.5).to(dtype)
    w = torch.randn(c, device="cuda", generator=g)
    b = torch.randn(c, device="cuda", generator=g)
    y = kernels.layer_norm(x, w, b)
    want = torch.nn.functional.layer_norm(x.float(), (c,), w, b, 1e-5)
    assert rel(y.float(), want) < (4e-3 if dtype == torch.bfloat16 else 1e-6)


@pytest.mark.parametrize("batch,m,n,k", [(1, 128, 256, 64), (1, 300, 384, 384), (4, 512, 512, 512),
                                         (2, 24, 24, 24), (1, 1000, 128, 128), (3, 130, 200, 136)])
def test_gemm_store_f32(batch, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(1)
    a = torch.randn(batch, m, k, device="cuda", generator=g).bfloat16()
    b = torch.randn(batch, n, k, device="cuda", generator=g).bfloat16()
    d = kernels.gemm_nt(a, b, out_dtype=torch.float32)
    want = a.float() @ b.float().transpose(-1, -2)
    assert rel(d, want) < 1e-5


def test_gemm_bias_bf16_out():
    g = torch.Generator(device="cuda").manual_seed(2)
    a = torch.randn(200, 384, device="cuda", generator=g).bfloat16()
    w = torch.randn(1536, 384, device="cuda", generator=g).bfloat16()
    bias = torch.randn(1536, device="cuda", generator=g)
    d = kernels.gemm_nt(a, w, bias=bias)
    want = a.float() @ w.float().T + bias
    assert rel(d.float(), want) < 4e-3


def test_gemm_residual_row_mask():
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(77, 384, device="cuda", generator=g).bfloat16()
    w = torch.randn(384, 384, device="cuda", generator=g).bfloat16()
    r = torch.randn(77, 384, device="cuda", generator=g)
    mask = torch.rand(77, device="cuda", generator=g) > 0.3
    d = kernels.gemm_nt(a, w, epilogue=kernels.EPI_RESIDUAL, residual=r, row_mask=mask, out_dtype=torch.float32)
    want = r + (a.float() @ w.float().T) * mask[:, None].float()
    assert rel(d, want) < 1e-5
    assert torch.equal(d[~mask], r[~mask])


def test_gemm_swiglu():
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.randn(150, 384, device="cuda", generator=g).bfloat16()
    wa = torch.randn(1536, 384, device="cuda", generator=g).bfloat16()
    wb = torch.randn(1536, 384, device="cuda", generator=g).bfloat16()
    packed = torch.stack([wa.view(96, 16, 384), wb.view(96, 16, 384)], 1).reshape(3072, 384)
    d = kernels.gemm_nt(a, packed, epilogue=kernels.EPI_SWIGLU)
    want = torch.nn.functional.silu(a.float() @ wa.float().T) * (a.float() @ wb.float().T)
    assert rel(d.float(), want) < 4e-3


def test_cpu_tensor_is_refused():
    with pytest.raises(_lib.UnsupportedCall):
        kernels.layer_norm(torch.randn(4, 128).bfloat16(), None, None)
