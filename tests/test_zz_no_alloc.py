"""rb_weight_matmul_noalloc: the GEMV entry point that allocates nothing.

Some callers cannot allocate device memory when they run a matmul (a host that
hands the library a fixed memory budget, an allocator owned by another
runtime, or a serving loop where cudaMalloc/cudaFree and their device-wide
synchronisation are not allowed). This entry point keeps its working memory in
one fixed device array inside the library.

Checked through the C ABI on device buffers, on two calls in a row with
different inputs (the second call reuses the shared scratch the first left
behind):
- against the oracle's dequant + GEMM accumulated in double, at the GEMV parity
  tests' tolerance (1e-5 relative to sum_k |W[n,k] x[k]|);
- against rb_weight_matmul (the allocating entry point), within the same bound;
- free device memory is unchanged across a warm call (no allocation).
Collected last so that it also runs after every other test.
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
def test_noalloc_matches_oracle(ctx, oracle, fmt, n, k, m):
    import torch
    import realm_b200 as rb
    O = oracle
    dt = {"q4k": O.Q4K, "q6k": O.Q6K, "q80": O.Q80}[fmt]
    tol = 1e-5
    rng = np.random.default_rng(n + k + m)
    wf = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    blocks = O.quantize(dt, wf)
    wdq = O.dequant(dt, blocks).reshape(n, k)
    w = rb.Weight(ctx, dt, n, k, blocks)
    dev = torch.device("cuda", 0)
    try:
        for call in range(2):
            xh = rng.normal(0, 1, size=(m, k)).astype(np.float32)
            x = torch.from_numpy(xh).to(dev)
            got = torch.full((m, n), float("nan"), device=dev)
            via_alloc = torch.empty(m, n, device=dev)
            w.matmul_noalloc(x, got, m)
            w.matmul(x, m, out=via_alloc)
            ctx.sync()
            g = got.cpu().numpy()
            assert np.all(np.isfinite(g)), call
            ref = O.dequant_matmul(dt, blocks, xh, m, n, k, f64=True)
            err = _rel_err(g, ref, wdq, xh)
            assert err < tol, ("vs oracle", call, err)
            err2 = _rel_err(g, via_alloc.cpu().numpy(), wdq, xh)
            assert err2 < tol, ("vs rb_weight_matmul", call, err2)
    finally:
        w.free()


def test_noalloc_allocates_no_device_memory(ctx, oracle):
    import torch
    import realm_b200 as rb
    O = oracle
    rng = np.random.default_rng(17)
    n, k, m = 11008, 4096, 8
    blocks = O.quantize(O.Q4K, rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    w = rb.Weight(ctx, O.Q4K, n, k, blocks)
    dev = torch.device("cuda", 0)
    try:
        x = torch.randn(m, k, device=dev)
        y = torch.empty(m, n, device=dev)
        w.matmul_noalloc(x, y, m)  # first call: looks up the scratch array's address
        ctx.sync()
        torch.cuda.synchronize(dev)
        free0, _ = torch.cuda.mem_get_info(dev)
        for _ in range(3):
            w.matmul_noalloc(x, y, m)
        ctx.sync()
        free1, _ = torch.cuda.mem_get_info(dev)
        assert free1 == free0, (free0, free1)
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
    # Q8_0 rows whose K is not a multiple of 256 are zero-padded at upload:
    # refused here (the allocating entry point takes them)
    pad = rb.Weight(ctx, O.Q80, 40, 96, O.quantize(O.Q80, rng.normal(0, 0.02, size=(40, 96)).astype(np.float32)))
    try:
        with pytest.raises(rb.RealmError) as e:
            pad.matmul_noalloc(torch.zeros(1, 96, device=dev), torch.zeros(1, 40, device=dev), 1)
        assert e.value.code == -23 and "256" in str(e.value)
    finally:
        pad.free()
