"""pi05_linear_static: the few-token linear layer for callers that cannot allocate device memory
(a host process whose device memory belongs to another allocator, a real-time loop that must not
allocate after start-up).  Its split-K scratch is a fixed device array inside the library.

Checked through the C ABI against the engine's pi05_op_linear (the same layer with engine-owned
scratch) where that accepts the shape, and against fp32 x . w^T + b, on two calls in a row so that
the second call runs on the array the first one left behind.  Tolerance (the engine's linear-layer
tests): max-abs <= 2e-2 * max|ref| + 1e-2.  pi05_linear_static_status reports no device-side wait
that gave up.  This file sorts last so that a run stopping at the first failure has already run
every other test.
"""
import pytest

pytestmark = pytest.mark.gpu

# (T, F, K, bias): split along K with tickets and partial tiles in the array; one token; a full
# 64-token tile; K = 192 (three K blocks: unsplit); K = 72 (a partial last K block read past the
# end); F = 100 and 200 (ragged last 128-row tile); F = 20000 (more tiles than SMs: unsplit); no bias
SHAPES = [(50, 4096, 1024, True), (37, 2560, 2048, True), (1, 1024, 4096, True), (64, 2048, 1024, True),
          (16, 768, 192, True), (1, 200, 72, False), (5, 100, 1024, True), (64, 20000, 64, True),
          (50, 1024, 4096, False)]


@pytest.mark.parametrize("T,F,K,with_bias", SHAPES)
def test_static_scratch_linear_matches_engine_linear(pn, T, F, K, with_bias):
    import torch

    eng = pn.Engine(pn.Config.make(siglip_layers=0, gemma_layers=1, num_steps=1), max_batch=1)
    g = torch.Generator(device="cuda").manual_seed(1234 + T + F + K)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(F, K, device="cuda", generator=g) * 0.02).bfloat16()
    b = (torch.randn(F, device="cuda", generator=g) * 0.02).bfloat16() if with_bias else None
    fp32 = x.float() @ w.float().t() + (b.float() if with_bias else 0.0)
    tol = 2e-2 * fp32.abs().max().item() + 1e-2
    ref = None
    if F % 8 == 0:  # the engine's operator takes 16-byte aligned rows only
        ref = torch.empty(T, F, device="cuda", dtype=torch.bfloat16)
        torch.cuda.synchronize()  # x, w, b come from torch's stream; the engine runs on its own
        eng.op_linear(x, w, ref, "store", bias=b)
        eng.sync()
    for _ in range(2):
        out = torch.full((T, F), float("nan"), device="cuda", dtype=torch.bfloat16)
        pn.linear_static(x, w, out, bias=b)
        pn.linear_static_status()  # waits for the default stream; raises if a device-side wait gave up
        assert torch.isfinite(out.float()).all()
        if ref is not None:
            assert (out.float() - ref.float()).abs().max().item() <= tol
        assert (out.float() - fp32).abs().max().item() <= tol
    eng.close()


def test_static_scratch_linear_rejects_sizes_and_pointers_beyond_its_limits(pn):
    import torch

    x = torch.zeros(65, 1024, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(128, 1024, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(65, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(pn.Pi05Error, match="T <= 64"):
        pn.linear_static(x, w, out)
    buf = torch.zeros(4 * 128 + 1, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(pn.Pi05Error, match="16-byte aligned"):
        pn.linear_static(x[:4], w, buf[1:].view(4, 128))
    pn.linear_static_status()
