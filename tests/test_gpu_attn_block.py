"""The attention block's products (modeling/gemma_4_moe_bq.mojo:418-627)
against the CPU oracle, through the C ABI: the q/k/v projections
(dispatch_bq_qkv, butterquant_kernels/linear.mojo:273-328), the per-head
block quantisation of the attention output (dispatch_bq_block_quant
[head_dim, apply_fwht=False]) and the output projection (dispatch_bq_block_linear
with head-sized blocks).  All three are integer dots followed by the
reference's float epilogue in its order, so the outputs are compared bit for
bit.  Weights follow the reference's recipes (SplitGainPerRowCs[128,
input_layernorm] for q/k/v, PlainPerRowBlockCs[head_dim] for o_proj,
modeling/gemma_4_moe_bq.mojo:91-121), quantised and VNNI-packed by the
oracle."""
import numpy as np
import pytest
import torch

import gmoe
import synth
from oracle import oracle as O
from helpers import tokens_np

pytestmark = pytest.mark.gpu

H = O.H


def bf(a):
    return O.f32_to_bf16(np.asarray(a, np.float32))


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(a).cuda()


def host(t):
    return synth.to_numpy(t)


def proj_weight(rng, rows, cols, block, gamma=None):
    """(row-major int8, scale, per-row colsum, per-block colsum block-major,
    VNNI-packed) of a seeded N(0, 0.02) bf16 weight."""
    w = bf(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02)
    q, sc = O.quantize_rows(w, block, gamma)
    return {"q": q, "scale": sc, "cs_row": O.colsum(q, cols, True).reshape(-1),
            "cs_blk": O.colsum(q, block, False), "packed": O.vnni_pack(q)}


@pytest.fixture(scope="module")
def activations():
    rng = np.random.default_rng(418)
    gain = bf(1.0 + 0.25 * rng.standard_normal(H))
    return rng, gain


# sliding layers: 16 q heads x 256, 8 kv heads x 256; full layers: 16 x 512,
# K = V with 2 kv heads x 512 (modeling/gemma4_common.mojo)
@pytest.mark.parametrize("kind,T", [("sliding", 1), ("sliding", 37), ("full", 16), ("full", 64)])
def test_qkv_projection_bit_exact(kind, T, activations):
    rng, gain = activations
    qn, kvn = (4096, 2048) if kind == "sliding" else (8192, 1024)
    wq = proj_weight(rng, qn, H, 128, gain)
    wk = proj_weight(rng, kvn, H, 128, gain)
    wv = proj_weight(rng, kvn, H, 128, gain) if kind == "sliding" else None
    x = tokens_np(T, seed=4180 + T)
    xi8, xsa = O.bq_norm_quant(x, O.bake_split_gain(gain))
    qo = torch.empty(T, qn, dtype=torch.bfloat16, device="cuda")
    ko = torch.empty(T, kvn, dtype=torch.bfloat16, device="cuda")
    vo = torch.empty(T, kvn, dtype=torch.bfloat16, device="cuda") if wv else None
    gmoe.call("gm_bq_qkv", dev(xi8), dev(xsa), T, dev(wq["packed"]), dev(wq["scale"]), qn,
              dev(wk["packed"]), dev(wk["scale"]), dev(wv["packed"]) if wv else None,
              dev(wv["scale"]) if wv else None, kvn, qo, ko, vo, None)
    torch.cuda.synchronize()
    assert np.array_equal(host(qo), O.bq_linear(xi8, xsa, wq["q"], wq["scale"], wq["cs_row"]))
    assert np.array_equal(host(ko), O.bq_linear(xi8, xsa, wk["q"], wk["scale"], wk["cs_row"]))
    if wv:
        assert np.array_equal(host(vo), O.bq_linear(xi8, xsa, wv["q"], wv["scale"], wv["cs_row"]))
    # the single-product entry point gives the same bits
    k2 = torch.empty_like(ko)
    gmoe.call("gm_bq_linear", dev(xi8), dev(xsa), T, dev(wk["packed"]), dev(wk["scale"]), kvn, k2, None)
    torch.cuda.synchronize()
    assert torch.equal(k2.view(torch.int16), ko.view(torch.int16))


@pytest.mark.parametrize("kind,T", [("sliding", 1), ("sliding", 50), ("full", 20)])
def test_head_quant_and_output_projection_bit_exact(kind, T, activations):
    rng, _ = activations
    hd, nq = (256, 16) if kind == "sliding" else (512, 16)
    k = hd * nq
    wo = proj_weight(rng, H, k, hd)
    attn = bf(rng.standard_normal((T, k), dtype=np.float32) * 0.3)
    attn[0, :hd] = 0  # an all-zero head: amax 0, int8 0
    q = torch.empty(T, k, dtype=torch.int8, device="cuda")
    sa = torch.empty(T, k // hd, dtype=torch.float32, device="cuda")
    gmoe.call("gm_bq_block_quant_ex", dev(attn), T, k, hd, 0, q, sa, None)
    torch.cuda.synchronize()
    rq, rsa = O.bq_block_quant_ex(attn, hd, False)
    assert np.array_equal(host(q), rq) and np.array_equal(host(sa), rsa)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    gmoe.call("gm_bq_block_linear_ex", dev(rq), dev(rsa), T, k, hd, dev(wo["packed"]), dev(wo["scale"]), H,
              out, None)
    torch.cuda.synchronize()
    ref = O.bq_block_linear_ex(rq, rsa, wo["q"], wo["scale"], wo["cs_blk"], hd)
    assert np.array_equal(host(out), ref)


def test_block_ops_match_the_moe_block_quant_and_dense_down(activations):
    """With block 64 and the FWHT the general entry points are the MoE's
    bucket quantiser and the dense MLP's down product."""
    rng, _ = activations
    T, I = 21, O.I
    b = bf(rng.standard_normal((T, I), dtype=np.float32) * 0.1)
    q = torch.empty(T, I, dtype=torch.int8, device="cuda")
    sa = torch.empty(T, I // 64, dtype=torch.float32, device="cuda")
    gmoe.call("gm_bq_block_quant_ex", dev(b), T, I, 64, 1, q, sa, None)
    torch.cuda.synchronize()
    rq, rsa = O.bq_block_quant(b)
    assert np.array_equal(host(q), rq) and np.array_equal(host(sa), rsa)
    DI = 2112
    wd = proj_weight(rng, H, DI, 64)
    h = bf(rng.standard_normal((T, DI), dtype=np.float32) * 0.2)
    hq, hsa = O.bq_block_quant(h)
    o1 = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    o2 = torch.empty_like(o1)
    gmoe.call("gm_bq_block_linear_ex", dev(hq), dev(hsa), T, DI, 64, dev(wd["packed"]), dev(wd["scale"]), H,
              o1, None)
    gmoe.call("gm_bq_block_linear", dev(hq), dev(hsa), T, dev(wd["packed"]), dev(wd["scale"]), o2, None)
    torch.cuda.synchronize()
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    assert np.array_equal(host(o1), O.bq_block_linear(hq, hsa, wd["q"], wd["scale"], wd["cs_blk"]))


def test_attention_block_argument_checks():
    z = torch.zeros(16, dtype=torch.int8, device="cuda")
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):
        gmoe.call("gm_bq_linear", z, z, 1, z, z, 100, z, None)  # n_rows not a multiple of 32
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):
        gmoe.call("gm_bq_block_quant_ex", z, 1, 256, 96, 0, z, z, None)  # unsupported block
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):
        gmoe.call("gm_bq_block_quant_ex", z, 1, 256, 256, 1, z, z, None)  # FWHT only for 64
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):
        gmoe.call("gm_bq_block_linear_ex", z, z, 1, 1280, 256, z, z, 2816, z, None)  # 5 blocks


@pytest.mark.parametrize("T", [1, 37, 600])
def test_norm_residual_add_bit_exact(T, activations):
    """gm_norm_residual_add, the decoder layer's step after the attention
    block (kernels/rmsnorm.mojo:48-64), against the oracle, into a separate
    output and in place over the residual stream (the two bit-identical).  The
    sum of squares is a warp reduction, not the reference's SIMD-lane order, so
    an inv_rms can differ in its last bit and an output by one bf16 step (the
    same bound as the RMSNorm and post-MoE tail tests)."""
    rng, gain = activations
    src = bf(rng.standard_normal((T, H), dtype=np.float32) * 0.7)
    res = bf(rng.standard_normal((T, H), dtype=np.float32))
    ref = O.norm_residual_add(src, res, gain)
    d_src, d_res, d_w = dev(src), dev(res), dev(gain)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    gmoe.call("gm_norm_residual_add", d_src, d_res, d_w, T, out, None)
    gmoe.call("gm_norm_residual_add", d_src, d_res, d_w, T, d_res, None)   # in place
    torch.cuda.synchronize()
    got = host(out)
    assert np.array_equal(host(d_res), got)
    g, r = O.bf16_to_f32(got), O.bf16_to_f32(ref)
    assert np.abs(g - r).max() <= 2 ** -7 * np.abs(r).max()
    assert (got == ref).mean() > 0.97
