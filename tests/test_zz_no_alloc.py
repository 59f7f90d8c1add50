"""rb_weight_matmul_noalloc: the GEMV entry point that allocates nothing.

Checked against rb_weight_matmul (the allocating entry point) on device
buffers, through the C ABI, on two calls in a row with different inputs (the
second call reuses the shared scratch the first left behind). Tolerance as the
GEMV parity tests: relative to sum_k |W[n,k] x[k]|, 3e-5 for Q4_K and 1e-5 for
Q6_K / Q8_0. Collected last so it also runs after every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rel_err(got, ref, w, x):
    scale = np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T + 1e-30
    return (np.abs(got.astype(np.float64) - ref.astype(np.float64)) / scale).max()


@pytest.mark.parametrize("fmt,n,k,m", [
    ("q4k", 22016, 4096, 8),   # Llama-2-7B gate|up
    ("q4k", 4096, 11008, 1),   # down projection, one row
    ("q6k", 1024, 4096, 5),
    ("q80", 300, 512, 3),      # ragged last row group
])
def test_noalloc_matches_weight_matmul(ctx, oracle, fmt, n, k, m):
    import torch
    import realm_b200 as rb
    O = oracle
    dt = {"q4k": O.Q4K, "q6k": O.Q6K, "q80": O.Q80}[fmt]
    tol = 3e-5 if dt == O.Q4K else 1e-5
    rng = np.random.default_rng(n + k + m)
    wf = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    blocks = O.quantize(dt, wf)
    wdq = O.dequant(dt, blocks).reshape(n, k)
    w = rb.Weight(ctx, dt, n, k, blocks)
    dev = torch.device("cuda", 0)
    try:
        for call in range(2):
            x = torch.from_numpy(rng.normal(0, 1, size=(m, k)).astype(np.float32)).to(dev)
            ref = torch.empty(m, n, device=dev)
            got = torch.full((m, n), float("nan"), device=dev)
            w.matmul(x, m, out=ref)
            w.matmul_noalloc(x, got, m)
            ctx.sync()
            g, r = got.cpu().numpy(), ref.cpu().numpy()
            assert np.all(np.isfinite(g)), call
            err = _rel_err(g, r, wdq, x.cpu().numpy())
            assert err < tol, (call, err)
    finally:
        w.free()


def test_noalloc_rejects_beyond_limits(ctx, oracle):
    import torch
    import realm_b200 as rb
    O = oracle
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(9)
    n, k = 256, 512
    w = rb.Weight(ctx, O.Q4K, n, k, O.quantize(O.Q4K, rng.normal(0, 0.02, size=(n, k)).astype(np.float32)))
    try:
        x = torch.zeros(9, k, device=dev)
        y = torch.zeros(9, n, device=dev)
        with pytest.raises(rb.RealmError) as e:
            w.matmul_noalloc(x, y, 9)          # batch above the maximum of 8
        assert e.value.code == -3 and "maximum" in str(e.value)
        with pytest.raises(ValueError):
            w.matmul_noalloc(np.zeros((1, k), np.float32), np.zeros((1, n), np.float32), 1)  # host buffers
    finally:
        w.free()
    big = rb.Weight(ctx, O.Q80, 16, 16640, O.quantize(O.Q80, np.zeros((16, 16640), np.float32)))
    try:
        with pytest.raises(rb.RealmError) as e:
            big.matmul_noalloc(torch.zeros(1, 16640, device=dev), torch.zeros(1, 16, device=dev), 1)  # K > 16384
        assert e.value.code == -3 and "16384" in str(e.value)
    finally:
        big.free()
