"""PyTorch tiled-GEMM bridge (xvram_b200.torch_bridge): mm / linear on CUDA tensors (device
entry point, every stride pattern) and on host tensors (out of core through an SDK
session with a small device budget), against torch in FP64."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from xvram_b200 import torch_bridge as tb  # noqa: E402

TOL = 1e-6  # max|err| / (K max|a| max|b|)


def err(got, a, b, ref):
    k = a.shape[1]
    return float((got.double().cpu() - ref).abs().max()) / (k * float(a.abs().max()) *
                                                           float(b.abs().max()))


def views(x):
    """The same logical matrix as a row-major tensor and as a column-major (transposed) view."""
    return [x.contiguous(), x.t().contiguous().t()]


@pytest.mark.parametrize("shape", [(257, 130, 99), (64, 64, 64), (1000, 8, 513), (3, 500, 7)])
@pytest.mark.parametrize("tensor_cores", [False, True])
def test_mm_cuda_all_layouts(shape, tensor_cores):
    m, k, n = shape
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.rand((m, k), generator=g, device="cuda") * 2 - 1
    B = torch.rand((k, n), generator=g, device="cuda") * 2 - 1
    ref = A.double().cpu() @ B.double().cpu()
    for a in views(A):
        for b in views(B):
            got = tb.mm(a, b, tensor_cores=tensor_cores)
            assert got.shape == (m, n) and got.is_contiguous()
            assert err(got, A, B, ref) <= TOL


def test_mm_cuda_strict_equals_itself_across_layouts():
    """Strict FP32: each output is one FFMA chain in k order whatever the operand layout."""
    g = torch.Generator(device="cuda").manual_seed(4)
    A = torch.rand((300, 200), generator=g, device="cuda")
    B = torch.rand((200, 100), generator=g, device="cuda")
    outs = [tb.mm(a, b) for a in views(A) for b in views(B)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_linear_cuda_bias_relu():
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.rand((96, 384), generator=g, device="cuda") * 2 - 1
    w = (torch.randn((512, 384), generator=g, device="cuda") / 20)
    b = torch.rand((512,), generator=g, device="cuda") - 0.5
    ref = torch.relu(x.double() @ w.double().t() + b.double()).cpu()
    got = tb.linear(x, w, b, relu=True)
    assert float((got.double().cpu() - ref).abs().max()) <= 1e-5
    got2 = tb.linear(x, w)  # bias-free, no activation: plain mm
    ref2 = (x.double() @ w.double().t()).cpu()
    assert float((got2.double().cpu() - ref2).abs().max()) <= 1e-5


def test_host_tensors_run_out_of_core():
    """Host operands stream through a 24 MiB device budget (several panels)."""
    tb.set_host_budget(24 << 20)
    try:
        g = torch.Generator().manual_seed(6)
        A = torch.rand((1500, 1300), generator=g) * 2 - 1
        B = torch.rand((1300, 1100), generator=g) * 2 - 1
        got = tb.mm(A, B)
        assert got.device.type == "cpu"
        ref = A.double() @ B.double()
        assert err(got, A, B, ref) <= TOL
        w = torch.randn((700, 1300), generator=g) / 40
        bias = torch.rand((700,), generator=g) - 0.5
        y = tb.linear(A, w, bias, relu=True)
        ref = torch.relu(A.double() @ w.double().t() + bias.double())
        assert float((y.double() - ref).abs().max()) <= 1e-5
        tel = tb._host_session().s.telemetry()
        assert tel.handle_reuses > 0
    finally:
        tb.set_host_budget(0)


HALF_ROUND = {torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(257, 130, 99), (64, 64, 64), (3, 500, 7)])
def test_mm_cuda_half_types(dtype, shape):
    """FP16 / BF16 matrices: strict FP32 arithmetic on the exactly widened values, the
    result rounded to the type once -- bit-identical to the FP32 kernel on the widened
    operands followed by one rounding, in every layout."""
    m, k, n = shape
    g = torch.Generator(device="cuda").manual_seed(7)
    A = (torch.rand((m, k), generator=g, device="cuda") * 2 - 1).to(dtype)
    B = (torch.rand((k, n), generator=g, device="cuda") * 2 - 1).to(dtype)
    want = tb.mm(A.float(), B.float()).to(dtype)
    ref = A.double().cpu() @ B.double().cpu()
    bound = TOL * k * float(A.abs().max()) * float(B.abs().max())
    for a in views(A):
        for b in views(B):
            got = tb.mm(a, b)
            assert got.dtype == dtype and got.shape == (m, n) and got.is_contiguous()
            assert torch.equal(got, want)
            d = (got.double().cpu() - ref).abs()
            assert bool((d <= bound + HALF_ROUND[dtype] * ref.abs()).all())


@pytest.mark.parametrize("shape", [(257, 130, 99), (200, 64, 300), (3, 500, 7)])
def test_mm_cuda_float64(shape):
    m, k, n = shape
    g = torch.Generator(device="cuda").manual_seed(8)
    A = torch.rand((m, k), generator=g, device="cuda", dtype=torch.float64) * 2 - 1
    B = torch.rand((k, n), generator=g, device="cuda", dtype=torch.float64) * 2 - 1
    ref = (A.cpu() @ B.cpu())
    for a in views(A):
        for b in views(B):
            got = tb.mm(a, b)
            assert got.dtype == torch.float64
            assert err(got, A, B, ref) <= 1e-13


def test_typed_options_refused():
    x = torch.ones((8, 8), device="cuda", dtype=torch.float16)
    with pytest.raises(TypeError):
        tb.mm(x, x, tensor_cores=True)
    with pytest.raises(TypeError):
        tb.linear(x, x, torch.ones(8, device="cuda", dtype=torch.float16))
    with pytest.raises(TypeError):
        tb.mm(x, x.float())


@pytest.mark.parametrize("dtype", [torch.float16, torch.float64])
def test_host_tensors_out_of_core_typed(dtype):
    """FP16 and FP64 host operands stream through a 16 MiB budget (several panels)."""
    tb.set_host_budget(16 << 20)
    try:
        g = torch.Generator().manual_seed(9)
        A = (torch.rand((1500, 1300), generator=g, dtype=torch.float64) * 2 - 1).to(dtype)
        B = (torch.rand((1300, 1100), generator=g, dtype=torch.float64) * 2 - 1).to(dtype)
        got = tb.mm(A, B)
        assert got.device.type == "cpu" and got.dtype == dtype
        ref = A.double() @ B.double()
        k = A.shape[1]
        if dtype == torch.float64:
            assert err(got, A, B, ref) <= 1e-13
        else:  # panels of K accumulate in an FP32 slot; one rounding to FP16 at the end
            bound = TOL * k * float(A.abs().max()) * float(B.abs().max())
            assert bool(((got.double() - ref).abs() <= bound + 2.0 ** -11 * ref.abs()).all())
        w = (torch.randn((700, 1300), generator=g, dtype=torch.float64) / 40).to(dtype)
        y = tb.linear(A, w)
        assert y.dtype == dtype
        ref = A.double() @ w.double().t()
        bound = TOL * k * float(A.abs().max()) * float(w.abs().max())
        if dtype == torch.float64:
            assert float((y.double() - ref).abs().max()) <= 1e-7 * bound
        else:
            assert bool(((y.double() - ref).abs() <= bound + 2.0 ** -11 * ref.abs()).all())
    finally:
        tb.set_host_budget(0)
