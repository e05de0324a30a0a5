"""Shared test helpers: seeded raw layers and the oracle-side preparation of
the butterquant / bf16 layer (the checker's own copy of every tensor)."""
import hashlib
import json
import os

import numpy as np

from oracle import oracle as O

H, E, I, GU = O.H, O.E, O.I, O.GU


def raw_layer_np(seed=1234, weight_std=0.02, router_std=0.02, stress=False):
    """Seeded raw bf16 layer as uint16 numpy arrays (host)."""
    rng = np.random.default_rng(seed)

    def normal(shape, std=1.0, mean=0.0):
        a = rng.standard_normal(size=shape, dtype=np.float32)
        a *= np.float32(std)
        a += np.float32(mean)
        return O.f32_to_bf16(a)

    L = {
        "router_proj": normal((E, H), router_std),
        "gate_up": normal((E, GU, H), weight_std),
        "down": normal((E, H, I), weight_std),
    }
    if stress:
        L["router_scale"] = normal((H,), 0.25, 1.0)
        L["per_expert_scale"] = normal((E,), 0.25, 1.0)
        L["pre_ffn_norm_2"] = normal((H,), 0.25, 1.0)
    else:
        one = O.f32_to_bf16(np.ones(1, np.float32))[0]
        L["router_scale"] = np.full(H, one, np.uint16)
        L["per_expert_scale"] = np.full(E, one, np.uint16)
        L["pre_ffn_norm_2"] = np.full(H, one, np.uint16)
    return L


_STRESS = []


def stress_layer():
    """The stress layer of the parity tests (seed 4321, router std 1.0, gains
    ~ N(1, 0.25) with negatives) and its oracle preparation, generated once
    per process (about 40 s of numpy normals); callers must not modify it."""
    if not _STRESS:
        raw = raw_layer_np(seed=4321, router_std=1.0, stress=True)
        _STRESS.append((raw, oracle_bq_layer(raw)))
    return _STRESS[0]


GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def digest(a):
    """SHA-256 of an array's bytes, with its dtype and shape."""
    a = np.ascontiguousarray(a)
    return {"sha256": hashlib.sha256(a.tobytes()).hexdigest(), "dtype": a.dtype.str,
            "shape": list(a.shape)}


def golden(name):
    """Arrays of the golden fixture tests/golden/<name>.npz."""
    with np.load(os.path.join(GOLDEN_DIR, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def golden_digests():
    """The digests of tests/golden/digests.json, keyed "<fixture>/<name>"."""
    with open(os.path.join(GOLDEN_DIR, "digests.json")) as f:
        return json.load(f)


def tokens_np(T, seed=99, std=1.0):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal(size=(T, H), dtype=np.float32) * np.float32(std)
    return O.f32_to_bf16(a)


def oracle_bq_layer(raw):
    """Quantize/pack/bake exactly as the reference quantizer + model_init."""
    gu_q, gu_s = O.quantize_rows(raw["gate_up"].reshape(E * GU, H), 128, raw["pre_ffn_norm_2"])
    dn_q, dn_s = O.quantize_rows(raw["down"].reshape(E * H, I), 64)
    return {
        "router_centered": O.router_center(raw["router_proj"]),
        "router_scale": O.bake_router_scale(raw["router_scale"]),
        "pes": raw["per_expert_scale"],
        "gamma2": O.bake_split_gain(raw["pre_ffn_norm_2"]),
        "gu_q": gu_q, "gu_scale": gu_s, "gu_cs": O.colsum(gu_q, H, True).reshape(-1),
        "dn_q": dn_q, "dn_scale": dn_s, "dn_cs": O.colsum(dn_q, 64, False),
    }


DI = 2112  # dense MLP intermediate


def raw_dense_np(seed=2112, weight_std=0.02, stress=True):
    """Seeded raw bf16 dense MLP (gate/up [2112][2816], down [2816][2112],
    pre_feedforward_layernorm gain) as uint16 numpy arrays."""
    rng = np.random.default_rng(seed)

    def normal(shape, std=1.0, mean=0.0):
        a = rng.standard_normal(size=shape, dtype=np.float32)
        a *= np.float32(std)
        a += np.float32(mean)
        return O.f32_to_bf16(a)

    return {"gate": normal((DI, H), weight_std), "up": normal((DI, H), weight_std),
            "down": normal((H, DI), weight_std),
            "pre_ffn_norm": normal((H,), 0.25 if stress else 0.0, 1.0)}


def oracle_dense_layer(raw):
    """Quantize as the reference's DenseGateUp / DenseDown recipes
    (modeling/gemma_4_moe_bq.mojo:113-116) and bake the split gain."""
    wg, wgs = O.quantize_rows(raw["gate"], 128, raw["pre_ffn_norm"])
    wu, wus = O.quantize_rows(raw["up"], 128, raw["pre_ffn_norm"])
    wd, wds = O.quantize_rows(raw["down"], 64)
    return {"wg": wg, "wgs": wgs, "wgcs": O.colsum(wg, H, True).reshape(-1),
            "wu": wu, "wus": wus, "wucs": O.colsum(wu, H, True).reshape(-1),
            "wd": wd, "wds": wds, "wdcs": O.colsum(wd, 64, False),
            "gamma": O.bake_split_gain(raw["pre_ffn_norm"])}


def oracle_bf16_layer(raw):
    return {
        "router_proj": raw["router_proj"],
        "router_scale": O.bake_router_scale(raw["router_scale"]),
        "pes": raw["per_expert_scale"],
        "gamma2": raw["pre_ffn_norm_2"],
        "w_gu": raw["gate_up"],
        "w_dn": raw["down"],
    }


def topk_margin(logits):
    """Gap between the 8th and 9th largest logit per token."""
    s = -np.sort(-logits, axis=1)
    return s[:, 7] - s[:, 8]


def routes_by_expert(idx, w=None):
    """Top-8 lists put in expert-id order.  The MoE output depends on the
    selected SET and the per-expert weights only (the combine sums a token's
    routes in expert order), so two routers agree when these match; the rank
    order inside the top 8 may differ where two survivors' logits differ in
    their last bit (f32 summation order)."""
    order = np.argsort(idx, axis=1, kind="stable")
    si = np.take_along_axis(idx, order, axis=1)
    if w is None:
        return si
    return si, np.take_along_axis(w, order, axis=1)


def rel_err(out_u16, ref_u16, rows=None):
    o = O.bf16_to_f32(out_u16).astype(np.float64)
    r = O.bf16_to_f32(ref_u16).astype(np.float64)
    if rows is not None:
        o, r = o[rows], r[rows]
    if r.size == 0:
        return 0.0
    return float(np.abs(o - r).max() / max(np.abs(r).max(), 1e-30))


NP_TAG = {np.dtype(np.int8): "I8", np.dtype(np.uint8): "U8", np.dtype(np.float32): "F32",
          np.dtype(np.int32): "I32", np.dtype(np.int64): "I64", np.dtype(np.float64): "F64",
          np.dtype(np.int16): "I16"}


def write_safetensors(path, entries):
    """A safetensors file laid out as the reference's writer makes it
    (safetensors/writer.mojo:39-75, entries in plan order with tightly packed
    data, quant/quantizer.mojo:674-683): 8-byte little-endian header length,
    the JSON header padded with spaces to a multiple of 8, then the data.
    entries: list of (name, array, tag or None, shape or None); uint16 arrays
    are bf16 bit patterns unless a tag says otherwise."""
    head, blobs, off = {}, [], 0
    for name, arr, tag, shape in entries:
        a = np.ascontiguousarray(arr)
        tag = tag or ("BF16" if a.dtype == np.uint16 else NP_TAG[a.dtype])
        shape = list(a.shape if shape is None else shape)
        b = a.tobytes()
        head[name] = {"dtype": tag, "shape": shape, "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    js = json.dumps(head, separators=(",", ":")).encode()
    js += b" " * (-len(js) % 8)
    with open(path, "wb") as f:
        f.write(len(js).to_bytes(8, "little"))
        f.write(js)
        for b in blobs:
            f.write(b)
    return path
