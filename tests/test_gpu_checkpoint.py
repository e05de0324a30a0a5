"""gm_moe_load_layer on the GPU: a layer written to a safetensors file in the
reference's on-disk layout (butterquant: int8 row-major weights with ".scale"
members, raw router scale and split gain; bf16: the original 3-D expert
tensors) and loaded through the C ABI must give, bit for bit, the forward of
the same layer registered through gm_moe_register_layer_bq / _bf16 with the
load-time bakes done by the caller; at degree 2 each rank reads its row
block."""
import numpy as np
import pytest
import torch

import gmoe
import synth
from helpers import write_safetensors

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

H, E, GU, I = gmoe.HIDDEN, gmoe.NUM_EXPERTS, gmoe.GATE_UP, gmoe.INTERMEDIATE
PFX = "model.language_model.layers.%d."


def host(t):
    return synth.to_numpy(t)


def post_gains(seed=11):
    g = torch.Generator(device="cpu").manual_seed(seed)
    gains = [(1.0 + 0.2 * torch.randn(H, generator=g)).to(torch.bfloat16) for _ in range(3)]
    return gains, torch.tensor([0.6875], dtype=torch.bfloat16)


def bq_entries(raw, L, layer, gains, ls):
    p = PFX % layer
    return [
        (p + "experts.gate_up_proj", host(L["gate_up_rowmajor"]), None, None),
        (p + "experts.gate_up_proj.scale", host(L["gate_up_scale"]), None, None),
        (p + "experts.down_proj", host(L["down_rowmajor"]), None, None),
        (p + "experts.down_proj.scale", host(L["down_scale"]), None, None),
        (p + "router.proj.weight", host(L["router_centered"]), None, None),
        (p + "router.scale", host(raw["router_scale"]), None, [H, 1]),
        (p + "router.per_expert_scale", host(raw["per_expert_scale"]), None, [E, 1]),
        (p + "pre_feedforward_layernorm_2.weight", host(raw["pre_ffn_norm_2"]), None, [H, 1]),
        (p + "post_feedforward_layernorm_1.weight", host(gains[0]), None, [H, 1]),
        (p + "post_feedforward_layernorm_2.weight", host(gains[1]), None, [H, 1]),
        (p + "post_feedforward_layernorm.weight", host(gains[2]), None, [H, 1]),
        (p + "layer_scalar", host(ls), None, [1, 1]),
    ]


def forward(blk, x, T, ffn_dense=None):
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    blk.forward(0, x, out, T)
    res = [host(out)]
    if ffn_dense is not None:
        xm = x.clone()
        blk.forward_ffn(0, xm, ffn_dense, T)
        res.append(host(xm))
    torch.cuda.synchronize()
    return res


def test_load_bq_layer_matches_register(tmp_path):
    raw = synth.make_layer(seed=606, device="cuda", router_std=1.0, stress_gains=True)
    L = synth.bq_layer(raw, keep_rowmajor=True)
    gains, ls = post_gains()
    path = write_safetensors(tmp_path / "model.safetensors", bq_entries(raw, L, 7, gains, ls))
    del L["gate_up_rowmajor"], L["down_rowmajor"]
    ck = gmoe.Checkpoint(path)
    Tmax = 640
    ref = gmoe.MoeBlock(Tmax, 1)
    ref.register_bq(0, L["gate_up"], L["gate_up_scale"], L["down"], L["down_scale"],
                    L["router_centered"], L["router_scale"], L["per_expert_scale"], L["pre_ffn_norm_2"])
    ref.register_post(0, gains[0].cuda(), gains[1].cuda(), gains[2].cuda(), float(ls.float()))
    got = gmoe.MoeBlock(Tmax, 1)
    got.load_layer(0, ck, ckpt_layer=7, post=True)
    for T in (16, 600):  # decode kernels and the tcgen05 prefill path
        x = synth.make_tokens(T, seed=T, device="cuda")
        dense = synth.make_tokens(T, seed=T + 1, device="cuda")
        a, b = forward(ref, x, T, dense), forward(got, x, T, dense)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    # degree 2: rank 1 reads experts 64..127 (row block of every expert tensor)
    epr = E // 2
    ref2 = gmoe.MoeBlock(64, 1, rank=1, degree=2)
    ref2.register_bq(0, L["gate_up"][epr * GU:], L["gate_up_scale"][epr * GU:], L["down"][epr * H:],
                     L["down_scale"][epr * H:], L["router_centered"], L["router_scale"],
                     L["per_expert_scale"], L["pre_ffn_norm_2"])
    got2 = gmoe.MoeBlock(64, 1, rank=1, degree=2)
    got2.load_layer(0, ck, ckpt_layer=7)
    x = synth.make_tokens(64, seed=5, device="cuda")
    assert np.array_equal(forward(ref2, x, 64)[0], forward(got2, x, 64)[0])
    # wrong layer index: the missing tensor is named
    with pytest.raises(gmoe.GmoeError, match="layers.3.experts.gate_up_proj"):
        got.load_layer(0, ck, ckpt_layer=3)
    for b in (ref, got, ref2, got2):
        b.close()
    ck.close()


def test_load_bf16_layer_matches_register(tmp_path):
    raw = synth.make_layer(seed=707, device="cuda", router_std=1.0, stress_gains=True)
    p = PFX % 0
    entries = [
        (p + "experts.gate_up_proj", host(raw["gate_up"]), None, None),   # [128][1408][2816]
        (p + "experts.down_proj", host(raw["down"]), None, None),         # [128][2816][704]
        (p + "router.proj.weight", host(raw["router_proj"]), None, None),
        (p + "router.scale", host(raw["router_scale"]), None, None),
        (p + "router.per_expert_scale", host(raw["per_expert_scale"]), None, None),
        (p + "pre_feedforward_layernorm_2.weight", host(raw["pre_ffn_norm_2"]), None, None),
    ]
    d = tmp_path / "hf"
    d.mkdir()
    write_safetensors(d / "model-00001-of-00002.safetensors", entries[:1])
    write_safetensors(d / "model-00002-of-00002.safetensors", entries[1:])
    ck = gmoe.Checkpoint(d)
    Lb = synth.bf16_layer(raw)
    ref = gmoe.MoeBlock(64, 1)
    ref.register_bf16(0, Lb["gate_up"], Lb["down"], Lb["router_proj"], Lb["router_scale"],
                      Lb["per_expert_scale"], Lb["pre_ffn_norm_2"])
    got = gmoe.MoeBlock(64, 1)
    got.load_layer(0, ck)
    x = synth.make_tokens(48, seed=9, device="cuda")
    assert np.array_equal(forward(ref, x, 48)[0], forward(got, x, 48)[0])
    # the post tensors are absent from this checkpoint
    with pytest.raises(gmoe.GmoeError, match="post_feedforward_layernorm_1"):
        got.load_layer(0, ck, post=True)
    ref.close()
    got.close()
    ck.close()


def dense_entries(rawd, Ld, layer, quantized):
    p = PFX % layer
    if quantized:
        return [
            (p + "mlp.gate_proj.weight", host(Ld["gate_rowmajor"]), None, None),
            (p + "mlp.gate_proj.weight.scale", host(Ld["gate_scale"]), None, None),
            (p + "mlp.up_proj.weight", host(Ld["up_rowmajor"]), None, None),
            (p + "mlp.up_proj.weight.scale", host(Ld["up_scale"]), None, None),
            (p + "mlp.down_proj.weight", host(Ld["down_rowmajor"]), None, None),
            (p + "mlp.down_proj.weight.scale", host(Ld["down_scale"]), None, None),
            (p + "pre_feedforward_layernorm.weight", host(rawd["pre_ffn_norm"]), None, [H, 1]),
        ]
    return [
        (p + "mlp.gate_proj.weight", host(rawd["gate"]), None, None),
        (p + "mlp.up_proj.weight", host(rawd["up"]), None, None),
        (p + "mlp.down_proj.weight", host(rawd["down"]), None, None),
        (p + "pre_feedforward_layernorm.weight", host(rawd["pre_ffn_norm"]), None, None),
    ]


def register_all(blk, L, Ld, gains, ls):
    blk.register_bq(0, L["gate_up"], L["gate_up_scale"], L["down"], L["down_scale"],
                    L["router_centered"], L["router_scale"], L["per_expert_scale"], L["pre_ffn_norm_2"])
    blk.register_post(0, gains[0].cuda(), gains[1].cuda(), gains[2].cuda(), float(ls.float()))
    blk.register_dense(0, Ld["gate"], Ld["gate_scale"], Ld["up"], Ld["up_scale"], Ld["down"],
                       Ld["down_scale"], Ld["pre_ffn_norm"])


def ffn(blk, T, seed):
    x = synth.make_tokens(T, seed=seed, device="cuda")
    blk.ffn_forward(0, x, T)
    torch.cuda.synchronize()
    return host(x)


def test_load_bq_ffn_with_dense_matches_register(tmp_path):
    """A butterquant file with the dense MLP: GM_LOAD_POST | GM_LOAD_DENSE
    gives the same whole-FFN output as registering the same tensors."""
    raw = synth.make_layer(seed=808, device="cuda", router_std=1.0, stress_gains=True)
    L = synth.bq_layer(raw, keep_rowmajor=True)
    rawd = synth.make_dense(seed=909, device="cuda")
    Ld = synth.dense_layer(rawd, keep_rowmajor=True)
    gains, ls = post_gains(12)
    path = write_safetensors(tmp_path / "model.safetensors",
                             bq_entries(raw, L, 2, gains, ls) + dense_entries(rawd, Ld, 2, True))
    ck = gmoe.Checkpoint(path)
    ref, got = gmoe.MoeBlock(700, 1), gmoe.MoeBlock(700, 1)
    register_all(ref, L, Ld, gains, ls)
    got.load_layer(0, ck, ckpt_layer=2, post=True, dense=True)
    for T in (12, 700):
        assert np.array_equal(ffn(ref, T, T), ffn(got, T, T))
    with pytest.raises(gmoe.GmoeError, match="BF16 checkpoint"):
        got.load_layer(0, ck, ckpt_layer=2, quantize=True)
    ref.close()
    got.close()
    ck.close()


def test_load_bf16_checkpoint_quantized_on_device(tmp_path):
    """GM_LOAD_QUANTIZE: a BF16 checkpoint (experts, router, norms, dense MLP)
    becomes the butterquant layer on the device, bit-identical to the layer
    the on-device restatement of the reference quantizer produces."""
    raw = synth.make_layer(seed=1001, device="cuda", router_std=1.0, stress_gains=True)
    rawd = synth.make_dense(seed=1002, device="cuda")
    gains, ls = post_gains(13)
    p = PFX % 0
    entries = [
        (p + "experts.gate_up_proj", host(raw["gate_up"]), None, None),
        (p + "experts.down_proj", host(raw["down"]), None, None),
        (p + "router.proj.weight", host(raw["router_proj"]), None, None),
        (p + "router.scale", host(raw["router_scale"]), None, None),
        (p + "router.per_expert_scale", host(raw["per_expert_scale"]), None, None),
        (p + "pre_feedforward_layernorm_2.weight", host(raw["pre_ffn_norm_2"]), None, None),
        (p + "post_feedforward_layernorm_1.weight", host(gains[0]), None, None),
        (p + "post_feedforward_layernorm_2.weight", host(gains[1]), None, None),
        (p + "post_feedforward_layernorm.weight", host(gains[2]), None, None),
        (p + "layer_scalar", host(ls), None, None),
    ] + dense_entries(rawd, None, 0, False)
    path = write_safetensors(tmp_path / "bf16.safetensors", entries)
    ck = gmoe.Checkpoint(path)
    L = synth.bq_layer(raw)
    Ld = synth.dense_layer(rawd)
    ref, got = gmoe.MoeBlock(640, 1), gmoe.MoeBlock(640, 1)
    register_all(ref, L, Ld, gains, ls)
    got.load_layer(0, ck, post=True, dense=True, quantize=True)
    for T in (7, 640):
        assert np.array_equal(ffn(ref, T, 50 + T), ffn(got, T, 50 + T))
    with pytest.raises(gmoe.GmoeError, match="GM_LOAD_QUANTIZE"):
        got.load_layer(0, ck, dense=True)
    ref.close()
    got.close()
    ck.close()
