"""gm_router_select_noalloc: the router for callers that cannot allocate
device memory (they hand over inputs and outputs only; the scratch is a fixed
array inside libgmoe.so).  Checked through the C ABI against gm_router_select,
which takes a caller-allocated scratch buffer, on two calls in a row (the
second call finds the first call's leftovers in the shared array).  This file
runs last so that a failure here leaves every other test already run."""
import numpy as np
import pytest
import torch

import gmoe

pytestmark = pytest.mark.gpu

H, E, TOPK = gmoe.HIDDEN, gmoe.NUM_EXPERTS, gmoe.TOP_K
MAX_T = 256


def router_weights(seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    wr = (torch.randn(E, H, generator=g) * 0.5).to(torch.bfloat16).cuda()
    rs = (1.0 + 0.25 * torch.randn(H, generator=g)).to(torch.bfloat16).cuda()
    pes = (1.0 + 0.25 * torch.randn(E, generator=g)).to(torch.bfloat16).cuda()
    return wr, rs, pes


def with_scratch(x, wr, rs, pes, T):
    ws = torch.empty(gmoe.lib().gm_router_workspace_bytes(T) // 4, dtype=torch.float32, device="cuda")
    idx = torch.empty(T, TOPK, dtype=torch.int32, device="cuda")
    w = torch.empty(T, TOPK, dtype=torch.float32, device="cuda")
    gmoe.call("gm_router_select", x, wr, rs, pes, T, ws, idx, w, None)
    torch.cuda.synchronize()
    return idx.cpu().numpy(), w.cpu().numpy()


def without_scratch(x, wr, rs, pes, T):
    idx = torch.full((T, TOPK), -7, dtype=torch.int32, device="cuda")
    w = torch.full((T, TOPK), -7.0, dtype=torch.float32, device="cuda")
    gmoe.call("gm_router_select_noalloc", x, wr, rs, pes, T, idx, w, None)
    torch.cuda.synchronize()
    return idx.cpu().numpy(), w.cpu().numpy()


@pytest.mark.parametrize("T1,T2", [(64, 64), (MAX_T, 3), (1, MAX_T)])
def test_noalloc_matches_router_select_two_calls(T1, T2):
    wr, rs, pes = router_weights(11)
    g = torch.Generator(device="cpu")
    g.manual_seed(T1 * 1000 + T2)
    xs = [torch.randn(T, H, generator=g).to(torch.bfloat16).cuda() for T in (T1, T2)]
    refs = [with_scratch(x, wr, rs, pes, x.shape[0]) for x in xs]
    # two calls in a row of the entry point under test
    outs = [without_scratch(x, wr, rs, pes, x.shape[0]) for x in xs]
    for (idx, w), (ref_idx, ref_w) in zip(outs, refs):
        assert np.array_equal(idx, ref_idx)
        # same kernels on the same inputs: the weights agree far inside the
        # router test tolerance (1e-4)
        assert np.abs(w - ref_w).max() <= 1e-6


def test_noalloc_rejects_sizes_beyond_the_limit():
    wr, rs, pes = router_weights(12)
    x = torch.zeros(MAX_T + 1, H, dtype=torch.bfloat16, device="cuda")
    idx = torch.empty(MAX_T + 1, TOPK, dtype=torch.int32, device="cuda")
    w = torch.empty(MAX_T + 1, TOPK, dtype=torch.float32, device="cuda")
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL.*256"):
        gmoe.call("gm_router_select_noalloc", x, wr, rs, pes, MAX_T + 1, idx, w, None)
