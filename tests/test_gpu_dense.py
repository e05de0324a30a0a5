"""Dense butterquant MLP on the GPU (gm_bq_dense_gate_up, gm_bq_block_linear,
gm_dense_forward, gm_ffn_forward) against the oracle's restatement of the
dense half of dispatch_bq_ffn (modeling/gemma_4_moe_bq.mojo:749-783).

Given identical int8 inputs the stages are bit-identical to the oracle; end
to end, the activation quantisation may differ in its last bit where inv_rms
differs from another f32 summation order, so the dense output is checked
within the bq tolerance and for a large fraction of bit-equal values."""
import numpy as np
import pytest
import torch

import gmoe
import synth
from oracle import oracle as O
import golden_cases as G
from helpers import raw_dense_np, oracle_dense_layer, raw_layer_np, tokens_np, rel_err, golden

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

H, DI = O.H, O.DENSE_I
TOL = 3e-2


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    return torch.from_numpy(a).cuda()


def host(t):
    return synth.to_numpy(t)


@pytest.fixture(scope="module")
def dense():
    raw = raw_dense_np(seed=77)
    d = oracle_dense_layer(raw)
    L = synth.dense_layer({k: dev(v) for k, v in raw.items()}, keep_rowmajor=True)
    # the on-device quantizer reproduces the oracle's weights bit for bit
    for name, key in (("gate", "wg"), ("up", "wu"), ("down", "wd")):
        assert np.array_equal(host(L[name + "_rowmajor"]), d[key])
        assert np.array_equal(host(L[name + "_scale"]), d[key + "s"])
    assert np.array_equal(host(L["pre_ffn_norm"]), d["gamma"])
    return raw, d, L


@pytest.mark.parametrize("T", [1, 5, 16, 17, 64, 300])
def test_dense_stages_bit_exact(dense, T):
    raw, d, L = dense
    x = tokens_np(T, seed=1000 + T)
    xi8, xsa = O.bq_norm_quant(x, d["gamma"])
    _, hb, hq, hs = O.dense_mlp(x, d)
    h_i8 = torch.empty(T, DI, dtype=torch.int8, device="cuda")
    h_sa = torch.empty(T, DI // 64, dtype=torch.float32, device="cuda")
    h_bf = torch.empty(T, DI, dtype=torch.bfloat16, device="cuda")
    gmoe.call("gm_bq_dense_gate_up", dev(xi8), dev(xsa), T, L["gate"], L["gate_scale"], L["up"],
              L["up_scale"], h_i8, h_sa, h_bf, None)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    gmoe.call("gm_bq_block_linear", dev(hq), dev(hs), T, L["down"], L["down_scale"], out, None)
    torch.cuda.synchronize()
    assert np.array_equal(host(h_bf), hb)
    assert np.array_equal(host(h_i8), hq)
    assert np.array_equal(host(h_sa), hs)
    want = O.bq_block_linear(hq, hs, d["wd"], d["wds"], d["wdcs"])
    assert np.array_equal(host(out), want)
    if T == G.DENSE_T:
        # the committed golden vectors of the same inputs
        gd = golden("dense_mlp")
        assert np.array_equal(host(h_bf), gd["bucket"])
        assert np.array_equal(host(h_i8), gd["bucket_q"])
        assert np.array_equal(host(h_sa), gd["bucket_sa"])
        assert np.array_equal(host(out), gd["out"])


@pytest.mark.parametrize("T", [3, 64, 700])
def test_dense_forward_matches_oracle(dense, T):
    raw, d, L = dense
    blk = gmoe.MoeBlock(max(T, 16), 1)
    blk.register_dense(0, L["gate"], L["gate_scale"], L["up"], L["up_scale"], L["down"],
                       L["down_scale"], L["pre_ffn_norm"])
    x = tokens_np(T, seed=2000 + T)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    blk.dense_forward(0, dev(x), out, T)
    torch.cuda.synchronize()
    want, _, _, _ = O.dense_mlp(x, d)
    got = host(out)
    assert rel_err(got, want) < TOL
    assert (got == want).mean() > 0.97
    # repeatable
    out2 = torch.empty_like(out)
    blk.dense_forward(0, dev(x), out2, T)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    blk.close()


@pytest.mark.parametrize("T", [8, 640])
def test_ffn_forward_is_dense_plus_moe_tail(dense, T):
    """gm_ffn_forward (dense MLP on a forked stream, MoE, tail) equals
    gm_dense_forward followed by gm_moe_forward_ffn with that dense_out."""
    raw, d, L = dense
    lay = synth.bq_layer(synth.make_layer(seed=123, device="cuda", router_std=1.0, stress_gains=True))
    g = torch.Generator(device="cpu").manual_seed(3)
    gains = [(1.0 + 0.2 * torch.randn(H, generator=g)).to(torch.bfloat16).cuda() for _ in range(3)]
    blk = gmoe.MoeBlock(T, 1)
    blk.register_bq(0, lay["gate_up"], lay["gate_up_scale"], lay["down"], lay["down_scale"],
                    lay["router_centered"], lay["router_scale"], lay["per_expert_scale"],
                    lay["pre_ffn_norm_2"])
    blk.register_post(0, gains[0], gains[1], gains[2], 0.8125)
    blk.register_dense(0, L["gate"], L["gate_scale"], L["up"], L["up_scale"], L["down"],
                       L["down_scale"], L["pre_ffn_norm"])
    x = synth.make_tokens(T, seed=T, device="cuda")
    dense_out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    blk.dense_forward(0, x, dense_out, T)
    a = x.clone()
    blk.forward_ffn(0, a, dense_out, T)
    b = x.clone()
    blk.profile(True)
    blk.ffn_forward(0, b, T)
    stats, _ = blk.profile_read()
    blk.profile(False)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    tc = ".tc" if T >= 128 else ""   # GM_OPT_DENSE_TC_MIN_TOKENS default
    assert {"dense.bq_norm_quant", "bq_linear.gate_up" + tc, "bq_block_linear" + tc} <= set(stats)
    # re-registering the experts keeps the dense MLP and the post gains
    blk.register_bq(0, lay["gate_up"], lay["gate_up_scale"], lay["down"], lay["down_scale"],
                    lay["router_centered"], lay["router_scale"], lay["per_expert_scale"],
                    lay["pre_ffn_norm_2"])
    c = x.clone()
    blk.ffn_forward(0, c, T)
    torch.cuda.synchronize()
    assert torch.equal(a, c)
    blk.close()


def test_dense_errors(dense):
    raw, d, L = dense
    blk = gmoe.MoeBlock(16, 1)
    x = torch.zeros(4, H, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(gmoe.GmoeError, match="register_dense"):
        blk.dense_forward(0, x, x.clone(), 4)
    blk.register_dense(0, L["gate"], L["gate_scale"], L["up"], L["up_scale"], L["down"],
                       L["down_scale"], L["pre_ffn_norm"])
    with pytest.raises(gmoe.GmoeError, match="T=17"):
        blk.dense_forward(0, x, x.clone(), 17)
    with pytest.raises(gmoe.GmoeError, match="no registered experts"):
        blk.ffn_forward(0, x, 4)
    blk.close()
    part = gmoe.MoeBlock(16, 1, rank=0, degree=2)
    raw_l = synth.make_layer(seed=5, device="cuda")
    lay = synth.bq_layer(raw_l)
    epr = 64
    part.register_bq(0, lay["gate_up"][:epr * 1408], lay["gate_up_scale"][:epr * 1408],
                     lay["down"][:epr * H], lay["down_scale"][:epr * H], lay["router_centered"],
                     lay["router_scale"], lay["per_expert_scale"], lay["pre_ffn_norm_2"])
    part.register_post(0, lay["pre_ffn_norm_2"], lay["pre_ffn_norm_2"], lay["pre_ffn_norm_2"], 1.0)
    part.register_dense(0, L["gate"], L["gate_scale"], L["up"], L["up_scale"], L["down"],
                        L["down_scale"], L["pre_ffn_norm"])
    with pytest.raises(gmoe.GmoeError, match="partials"):
        part.ffn_forward(0, x, 4)
    part.close()


@pytest.mark.parametrize("T", [1, 100, 128, 300, 2048])
def test_dense_tcgen05_path_equals_streaming_path(dense, T):
    """The tcgen05 GEMMs (gemm_tc.cu, dense variant) and the HBM-streaming
    kernels (dense_bq.cu, bit-exact to the oracle above) give identical bits."""
    raw, d, L = dense
    blk = gmoe.MoeBlock(T, 1)
    blk.register_dense(0, L["gate"], L["gate_scale"], L["up"], L["up_scale"], L["down"],
                       L["down_scale"], L["pre_ffn_norm"])
    x = synth.make_tokens(T, seed=40 + T, device="cuda")
    outs = []
    for thr in (1, 1 << 30):
        blk.set_option(gmoe.OPT_DENSE_TC_MIN_TOKENS, thr)
        blk.profile(True)
        o = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        blk.dense_forward(0, x, o, T)
        stats, _ = blk.profile_read()
        blk.profile(False)
        assert ("bq_block_linear.tc" in stats) == (thr == 1)
        outs.append(o)
    torch.cuda.synchronize()
    assert blk.device_status() == 0
    assert torch.equal(outs[0], outs[1])
    blk.close()
