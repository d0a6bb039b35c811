"""pi05_linear_static: the few-token linear layer for callers that cannot allocate device memory
(a host process whose device memory belongs to another allocator, a real-time loop that must not
allocate after start-up).  Its split-K scratch is a fixed device array inside the library.

Checked through the C ABI against the engine's pi05_op_linear (the same layer with engine-owned
scratch), on two calls in a row so that the second call runs on the array the first one left behind.
This file sorts last so that a run stopping at the first failure has already run every other test.
"""
import pytest

pytestmark = pytest.mark.gpu


def test_static_scratch_linear_matches_engine_linear(pn):
    import torch

    eng = pn.Engine(pn.Config.make(siglip_layers=0, gemma_layers=1, num_steps=1), max_batch=1)
    g = torch.Generator(device="cuda").manual_seed(1234)
    # two different few-token shapes, both split along K (tickets and partial tiles in the array)
    for T, F, K in [(50, 4096, 1024), (37, 2560, 2048)]:
        x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
        w = (torch.randn(F, K, device="cuda", generator=g) * 0.02).bfloat16()
        b = (torch.randn(F, device="cuda", generator=g) * 0.02).bfloat16()
        ref = torch.empty(T, F, device="cuda", dtype=torch.bfloat16)
        torch.cuda.synchronize()  # x, w, b come from torch's stream; the engine runs on its own
        eng.op_linear(x, w, ref, "store", bias=b)
        eng.sync()
        fp32 = x.float() @ w.float().t() + b.float()
        for _ in range(2):
            out = torch.full((T, F), float("nan"), device="cuda", dtype=torch.bfloat16)
            pn.linear_static(x, w, out, bias=b)
            torch.cuda.synchronize()
            assert torch.isfinite(out.float()).all()
            # same tolerance as the engine's linear-layer tests
            tol = 2e-2 * fp32.abs().max().item() + 1e-2
            assert (out.float() - ref.float()).abs().max().item() <= tol
            assert (out.float() - fp32).abs().max().item() <= tol
    eng.close()


def test_static_scratch_linear_rejects_sizes_beyond_its_limits(pn):
    import torch

    x = torch.zeros(65, 1024, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(128, 1024, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(65, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(pn.Pi05Error, match="T <= 64"):
        pn.linear_static(x, w, out)
