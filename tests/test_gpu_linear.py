"""nsa_linear (ops.linear with the epilogue of the reference's tiled GEMM) against the CPU oracle:
the reference's lin (tools/reference.py:208-210, pinned by tests/golden/linear.npz) and the GEMM
epilogue (app/gpu/gemm.js:155-165).  Operands are bf16 and the oracle runs in float64 on the same
bf16 values, so the only difference is the fp32 accumulation order."""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O
from tests._helpers import bf16_round

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module", autouse=True)
def _lib_loaded():
    torch.cuda.set_device(DEV)
    from nanosaur2_web_b200 import _lib
    _lib.lib()
    yield
    torch.cuda.synchronize()


def t(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=DEV, dtype=dtype)


def check_device():
    from nanosaur2_web_b200.ops import check_device as chk
    chk(DEV)


def operands(seed, M, N, K):
    rng = np.random.default_rng(seed)
    a = bf16_round(rng.standard_normal((M, K), dtype=np.float32))
    w = bf16_round(rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K))
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    return rng, a, w, b


def test_dit_output_projection_gated_residual():
    """x += gate[2C + n] * (a @ W_proj^T + b) over 3952 rows, C = 1536 (app/models/nanosaur2.js:210)."""
    from nanosaur2_web_b200.ops import linear
    M, C = 3952, 1536
    rng, a, w, b = operands(3, M, C, C)
    x = rng.standard_normal((M, C), dtype=np.float32)
    mod = rng.standard_normal(6 * C).astype(np.float32)
    out = t(x)
    linear(t(a, torch.bfloat16), t(w, torch.bfloat16), bias=t(b), out=out, resid=True, gate=t(mod), gOff=2 * C)
    check_device()
    want = O.linear_epilogue(O.linear(a, w, b, acc=np.float64), x, mod[2 * C:3 * C], resid=True, acc=np.float64)
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-3, atol=2e-3)


def test_linear_ragged_silu_column_window():
    """M, N, K off the tiles (300 x 200, K = 200: partial row / column tiles and a partial K slice),
    alpha 0.5, silu, written into columns [8, 208) of a wider output that keeps its other columns."""
    from nanosaur2_web_b200.ops import linear
    M, N, K = 300, 200, 200
    _, a, w, b = operands(4, M, N, K)
    out = torch.full((M, 216), 7.0, device=DEV)
    linear(t(a, torch.bfloat16), t(w, torch.bfloat16), bias=t(b), out=out, act="silu", cOff=8, alpha=0.5)
    check_device()
    y = 0.5 * O.linear(a, w, acc=np.float64) + b
    want = O.linear_epilogue(y, act="silu", acc=np.float64)
    got = out.cpu().numpy()
    np.testing.assert_allclose(got[:, 8:208], want, rtol=1e-3, atol=2e-3)
    assert (got[:, :8] == 7.0).all() and (got[:, 208:] == 7.0).all()


def test_linear_plain_residual_without_bias():
    from nanosaur2_web_b200.ops import linear
    M, N, K = 129, 512, 64
    rng, a, w, _ = operands(5, M, N, K)
    x = rng.standard_normal((M, N), dtype=np.float32)
    out = t(x)
    linear(t(a, torch.bfloat16), t(w, torch.bfloat16), out=out, resid=True)
    check_device()
    want = O.linear_epilogue(O.linear(a, w, acc=np.float64), x, resid=True, acc=np.float64)
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-3, atol=2e-3)
