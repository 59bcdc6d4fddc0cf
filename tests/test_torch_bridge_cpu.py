"""PyTorch bridge argument checks that need no GPU: element types outside the reference
route's four (python/xvram/torch_native.py:95-100), mixed types, and options that apply
to float32 only are refused before any device work; without a CUDA device a host call
raises instead of computing on the CPU."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from xvram_b200 import torch_bridge as tb  # noqa: E402


def test_unsupported_and_mixed_types_are_refused():
    a = torch.ones((4, 4), dtype=torch.int32)
    with pytest.raises(TypeError):
        tb.mm(a, a)
    with pytest.raises(TypeError):
        tb.mm(torch.ones((4, 4), dtype=torch.float16), torch.ones((4, 4)))


def test_float32_only_options():
    h = torch.ones((4, 4), dtype=torch.bfloat16)
    with pytest.raises(TypeError):
        tb.mm(h, h, tensor_cores=True)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.float64])
def test_no_cpu_path(dtype):
    a = torch.ones((4, 4), dtype=dtype)
    with pytest.raises(RuntimeError, match="needs a CUDA device"):
        tb.mm(a, a)


def test_bias_on_half_types_refused_before_any_work():
    x = torch.ones((4, 4), dtype=torch.float16)
    with pytest.raises(TypeError):
        tb.linear(x, x, torch.ones(4, dtype=torch.float16))
    with pytest.raises(TypeError):
        tb.linear(x, x, relu=True)
