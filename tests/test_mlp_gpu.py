"""Linear + bias + ReLU layers through the SDK with weights streamed through a small device
budget (xvram_b200.mlp.StreamedMLP, the C5 path at test size), against an FP64 forward."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from xvram_b200 import sdk  # noqa: E402
from xvram_b200.mlp import StreamedMLP  # noqa: E402

MiB = 1 << 20


@pytest.mark.parametrize("budget_mib", [16, 256])
def test_streamed_mlp_matches_fp64(budget_mib):
    F, batch, layers = 1024, 64, 5
    rng = np.random.default_rng(11)
    W = [(rng.standard_normal((F, F)) / np.sqrt(F)).astype(np.float32) for _ in range(layers)]
    bias = rng.uniform(-1 / 32, 1 / 32, (layers, F)).astype(np.float32)
    x = rng.uniform(-1, 1, (batch, F)).astype(np.float32)
    cfg = sdk.session_config(chunk_size_bytes=2 * MiB, cache_target_bytes=budget_mib * MiB)
    with sdk.Sdk(cfg) as s:
        net = StreamedMLP(s, F, batch, layers)
        for i, w in enumerate(W):
            # column-major out x in: element (o, i) at o + i * F, i.e. the C-order bytes of w.T
            net.load_weight(i, np.ascontiguousarray(w.T))
        net.load_biases(np.ascontiguousarray(bias))
        out = np.empty((batch, F), dtype=np.float32)
        for _ in range(2):  # the second pass streams the weights back in from the host
            net.forward(x, out)
        tel = s.telemetry()
        net.close()
    ref = x.astype(np.float64)
    for i in range(layers):
        ref = np.maximum(ref @ W[i].astype(np.float64).T + bias[i], 0.0)
    err = float(np.max(np.abs(out - ref)))
    assert err <= 1e-5 * np.sqrt(F) * layers, err
    assert net.statuses and all(st == 0 for st in net.statuses)
    # per pass and layer: the GEMM and the bias/ReLU transaction each complete one
    # residency transaction (the reference counts every executed tile the same way)
    assert tel.transactions_completed == 2 * 2 * layers
    if budget_mib == 16:  # 5 x 4 MiB of weights through 16 MiB: evictions and frame reuse
        assert tel.clean_evictions + tel.dirty_evictions > 0 and tel.handle_reuses > 0
