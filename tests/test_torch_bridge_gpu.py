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
