"""The cases of the golden fixtures in tests/golden/.

The reference is Mojo: it cannot be built or run here, and its own tests hold
no golden vectors for the MoE block (its attention tests compute their
expected values at run time from a float restatement).  These fixtures are
therefore the CPU oracle's outputs on the seeded inputs that the parity tests
use, plus the reference's own attention test scenario
(tests/test_sliding_attention_degree_parity.mojo,
tests/test_full_attention_degree_parity.mojo).  They pin the oracle (any
change to its arithmetic, or to the compiler's treatment of it, shows up as a
mismatch in test_golden.py) and give the GPU parity tests a fixed target.

Each case returns three dicts of numpy arrays:
  inputs  - the seeded inputs, pinned by SHA-256 digest (a change in numpy's
            seeded streams is then told apart from a change in arithmetic);
  arrays  - small outputs, stored in tests/golden/<case>.npz;
  digests - large outputs, pinned by SHA-256 digest in tests/golden/digests.json.
"""
import numpy as np

from oracle import oracle as O
from helpers import (raw_dense_np, oracle_dense_layer, oracle_bf16_layer, stress_layer,
                     tokens_np)

H, E, I, TOPK = O.H, O.E, O.I, O.TOPK

CASES = ["scalar_math", "moe_layer", "moe_stages", "moe_forward", "dense_mlp", "attention"]

# inputs of the GPU parity tests that compare against the fixtures
ROUTER_T, ROUTER_SEED = 16, 116          # test_router_parity (T=16, stress)
NORM_T, NORM_SEED, NORM_STD = 37, 237, 3.0   # test_norm_quant_parity (T=37)
BLOCK_ROWS = 77                          # test_block_quant_bit_exact (rows=77)
SCHED_T, SCHED_BASE, SCHED_EPR = 64, 64, 64  # test_schedule_bit_exact
FWD_T, FWD_SEED = 16, 616                # test_forward_bq (T=16, stress)
DENSE_SEED, DENSE_T, DENSE_X_SEED = 77, 5, 1005  # test_dense_stages_bit_exact (T=5)
ATTN_STEPS = (8, 9)                      # the scenario's last two (decode) steps


def _scalar(fn, xs):
    return np.array([fn(float(x)) for x in xs], np.float32)


def scalar_math():
    """The reference-written scalar approximations on fixed grids:
    fast_exp_softmax_biased (simd_math/exponential.mojo:177-194),
    exp_f32_fast (simd_math/ops.mojo:72-96), gelu_tanh_f32
    (simd_math/ops.mojo:144-156), and bf16 round-to-nearest-even stores
    (butterquant/convert.mojo:7-17) on edge values."""
    L = O.lib()
    sm_x = np.linspace(-90.0, 0.0, 2049, dtype=np.float32)
    fe_x = np.linspace(-20.0, 5.0, 2049, dtype=np.float32)
    ge_x = np.linspace(-10.0, 10.0, 2049, dtype=np.float32)
    edge = np.array([0.0, -0.0, 1.0, 1.00390625, 1.01171875, -1.00390625, 3.14159, -2.5e-3, 65504.0,
                     1e38, 3.3895e38, np.finfo(np.float32).max, np.finfo(np.float32).tiny,
                     np.float32(1e-40), np.inf, -np.inf], np.float32)
    arrays = {
        "softmax_exp_x": sm_x, "softmax_exp": _scalar(L.orc_fast_exp_softmax_biased, sm_x),
        "exp_fast_x": fe_x, "exp_fast": _scalar(L.orc_exp_f32_fast, fe_x),
        "gelu_x": ge_x, "gelu": _scalar(L.orc_gelu_tanh, ge_x),
        "bf16_x": edge, "bf16": O.f32_to_bf16(edge),
        "bf16_scalar": np.array([L.orc_f2bf(float(v)) for v in edge], np.uint16),
    }
    return {}, arrays, {}


def moe_layer():
    """The stress layer's weight format: the quantizer (FWHT, split gain,
    absmax int8), the router centring, the baked gains and the VNNI packing
    of the whole layer (quant/quantizer.mojo:963-1051,
    butterquant/kernels.mojo:28-224, butterquant/vnni.mojo:31-83)."""
    raw, ref = stress_layer()
    inputs = dict(raw)
    arrays = {"gu_scale_head": ref["gu_scale"][:64], "dn_scale_head": ref["dn_scale"][:64],
              "router_centered_head": ref["router_centered"][:2, :64], "gamma2_head": ref["gamma2"][:64],
              "gu_q_row0": ref["gu_q"][0, :128], "dn_q_row0": ref["dn_q"][0, :64]}
    digests = {k: ref[k] for k in ("router_centered", "router_scale", "gamma2", "gu_q", "gu_scale",
                                   "gu_cs", "dn_q", "dn_scale", "dn_cs")}
    digests["gate_up_packed"] = O.vnni_pack(ref["gu_q"])
    digests["down_packed"] = O.vnni_pack(ref["dn_q"])
    return inputs, arrays, digests


def skewed_routes(T, base):
    """The routing of test_schedule_bit_exact: 16 hot experts, seeded by T and
    the expert base."""
    rng = np.random.default_rng(T * 7 + base)
    p = np.r_[np.full(16, 0.04), np.full(112, 0.36 / 112)]
    idx = np.stack([rng.choice(E, TOPK, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, TOPK)).astype(np.float32)
    return idx, w


def block_quant_input(rows):
    """The bucket rows of test_block_quant_bit_exact."""
    rng = np.random.default_rng(rows)
    return O.f32_to_bf16(rng.standard_normal((rows, I)).astype(np.float32) * 0.1)


def moe_stages():
    """Router (logits, top-8, weights), norm + FWHT + int8 activations, the
    down-projection block quantiser and the expert schedule, each on the
    inputs of its GPU parity test."""
    _, ref = stress_layer()
    xr = tokens_np(ROUTER_T, seed=ROUTER_SEED)
    idx, w, lg = O.router(xr, ref["router_centered"], ref["router_scale"], ref["pes"])
    xn = tokens_np(NORM_T, seed=NORM_SEED, std=NORM_STD)
    xq, xsa = O.bq_norm_quant(xn, ref["gamma2"])
    b = block_quant_input(BLOCK_ROWS)
    bq, bsa = O.bq_block_quant(b)
    sidx, sw = skewed_routes(SCHED_T, SCHED_BASE)
    off, routes = O.build_schedules(sidx, sw, SCHED_BASE, SCHED_EPR)
    inputs = {"router_x": xr, "norm_x": xn, "block_in": b, "sched_idx": sidx, "sched_w": sw}
    arrays = {"router_idx": idx, "router_w": w, "router_logits": lg, "norm_sa": xsa,
              "block_sa": bsa, "sched_offset": off, "sched_token": routes["token"].copy(),
              "sched_weight": routes["weight"].copy()}
    return inputs, arrays, {"norm_q": xq, "block_q": bq}


def moe_forward():
    """The whole block on the stress layer: butterquant at degree 1 (the GPU
    target) and degree 2 (per-rank partials rounded to bf16 and summed), and
    the bf16 twin on the same weights."""
    raw, ref = stress_layer()
    x = tokens_np(FWD_T, seed=FWD_SEED)
    out, idx, w, lg = O.bq_forward(x, ref)
    out2, idx2, _, _ = O.bq_forward(x, ref, degree=2)
    ob, ib, wb, _ = O.bf16_forward(x, oracle_bf16_layer(raw))
    arrays = {"out": out, "idx": idx, "w": w, "logits": lg, "bf16_idx": ib, "bf16_w": wb}
    return {"x": x}, arrays, {"out_degree2": out2, "idx_degree2": idx2, "bf16_out": ob}


def dense_mlp():
    """The dense butterquant MLP (modeling/gemma_4_moe_bq.mojo:749-783) of
    test_dense_stages_bit_exact: quantized weights, the GeGLU bucket, its
    block quantisation and the output."""
    raw = raw_dense_np(seed=DENSE_SEED)
    d = oracle_dense_layer(raw)
    x = tokens_np(DENSE_T, seed=DENSE_X_SEED)
    out, hb, hq, hs = O.dense_mlp(x, d)
    inputs = dict(raw)
    inputs["x"] = x
    arrays = {"out": out, "bucket": hb, "bucket_q": hq, "bucket_sa": hs}
    digests = {k: d[k] for k in ("wg", "wgs", "wu", "wus", "wd", "wds", "gamma")}
    return inputs, arrays, digests


def attention():
    """The reference's attention test scenarios (sliding: 16 q heads, 8 KV
    heads of 256, two-page ring; full: 2 KV heads of 512, 3-5 pages) through
    the oracle's prep and flash decode: the outputs and query scales of the
    last two steps, and digests of their int8 queries and of the caches after
    the last step."""
    from test_attention_oracle import run_scenario_oracle
    arrays, digests = {}, {}
    for name, full in (("sliding", False), ("full", True)):
        steps = run_scenario_oracle(full=full)
        for s in ATTN_STEPS:
            _, q_i8, fq, out, _ = steps[s]
            arrays[f"{name}_out_s{s}"] = out
            arrays[f"{name}_fq_s{s}"] = fq
            digests[f"{name}_q_s{s}"] = q_i8
        for k, a in zip(("kc", "ks", "vc", "vs"), steps[-1][4]):
            digests[f"{name}_{k}"] = a
    return {}, arrays, digests
