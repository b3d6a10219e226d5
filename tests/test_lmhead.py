"""The LM-head GEMV oracle (oracle/aux_oracle.c) pinned to the reference's
own noel_gemv_quantized (src/dequant.c:412-470, compiled into oracle/_ref):
F32, F16 and BF16 rows, widths a multiple of 8, bit for bit."""
import numpy as np
import pytest

from oracle.oracle import RefAux


def head_inputs(rows=777, cols=4096, B=3, seed=0):
    g = np.random.Generator(np.random.PCG64(seed))
    w32 = (g.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    x = g.standard_normal((B, cols)).astype(np.float32)
    return {
        0: w32,
        30: (w32.view(np.uint32) >> 16).astype(np.uint16),   # bf16: the top half
        1: w32.astype(np.float16).view(np.uint16),
    }, x


@pytest.mark.parametrize("cols", [4096, 1000, 64])
@pytest.mark.parametrize("wtype", [0, 1, 30])
def test_gemv_oracle_matches_reference(oracle, wtype, cols):
    if not RefAux.available():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    ws, x = head_inputs(cols=cols, seed=cols + wtype)
    a = oracle.gemv(ws[wtype], wtype, x)
    b = RefAux().gemv(ws[wtype], wtype, x)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
