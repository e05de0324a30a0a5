"""ctypes front end of the CPU oracle (moe_oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, always as the checker or the
timed CPU baseline, never as the product.  PARITY UNPINNED: see the header of
moe_oracle.cpp.

Arrays are numpy; bf16 tensors travel as uint16 bit patterns.
"""
import ctypes as C
import os

import numpy as np

from . import build as _build

H, E, TOPK, I, GU, DOWN_BLOCK = 2816, 128, 8, 704, 1408, 64
NB_DOWN = I // DOWN_BLOCK

_LIB = None


def lib(variant=None):
    global _LIB
    if _LIB is None:
        variant = variant or os.environ.get("GMOE_ORACLE_VARIANT", "portable")
        path = _build.lib_path(variant)
        if not os.path.exists(path):
            path = _build.build(variant)
        _LIB = C.CDLL(path)
        _declare(_LIB)
    return _LIB


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


class OrcBqLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "router_centered", "router_scale", "pes", "gamma2", "gu_q", "gu_scale",
        "gu_cs", "dn_q", "dn_scale", "dn_cs")]


class OrcBf16Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "router_proj", "router_scale", "pes", "gamma2", "w_gu", "w_dn")]


def _declare(L):
    vp, i32, i64, f32 = C.c_void_p, C.c_int, C.c_long, C.c_float
    sig = {
        "orc_fast_exp_softmax_biased": (f32, [f32]),
        "orc_gelu_tanh": (f32, [f32]),
        "orc_exp_f32_fast": (f32, [f32]),
        "orc_f2bf": (C.c_uint16, [f32]),
        "orc_fwht_rows": (None, [vp, i64, i32, i32]),
        "orc_bake_split_gain": (None, [vp, vp, i32]),
        "orc_bake_router_scale": (None, [vp, vp, i32]),
        "orc_router_center": (None, [vp, i32, i32, vp]),
        "orc_quantize_rows": (None, [vp, i64, i32, vp, i32, vp, vp]),
        "orc_vnni_pack": (None, [vp, i64, i32, vp]),
        "orc_vnni_unpack": (None, [vp, i64, i32, vp]),
        "orc_colsum": (None, [vp, i64, i32, i32, vp, i32]),
        "orc_router": (None, [vp, i32, vp, vp, vp, vp, vp, vp]),
        "orc_build_schedules": (None, [vp, vp, i32, i32, i32, vp, vp]),
        "orc_rms_norm": (None, [vp, vp, i32, vp]),
        "orc_norm_residual_add": (None, [vp, vp, vp, i32, vp]),
        "orc_post_moe": (None, [vp, vp, vp, vp, vp, vp, C.c_float, i32, vp]),
        "orc_phase1_bf16": (None, [vp, vp, vp, vp, i32, vp]),
        "orc_phase2_bf16": (None, [vp, vp, vp, vp, i32, i32, vp]),
        "orc_bq_norm_quant": (None, [vp, vp, i32, vp, vp]),
        "orc_bq_phase1": (None, [vp, vp, vp, vp, vp, vp, vp, i32, vp]),
        "orc_bq_block_quant": (None, [vp, i64, i32, i32, vp, vp]),
        "orc_bq_phase2": (None, [vp, vp, vp, vp, vp, vp, vp, i64, i32, i32, vp]),
        "orc_bq_linear": (None, [vp, vp, i32, vp, vp, vp, i32, i32, vp]),
        "orc_gelu_gate_up": (None, [vp, vp, i64, vp]),
        "orc_bq_block_linear": (None, [vp, vp, i32, i32, vp, vp, vp, i32, vp]),
        "orc_bq_block_quant_ex": (None, [vp, i64, i32, i32, i32, vp, vp]),
        "orc_bq_block_linear_ex": (None, [vp, vp, i32, i32, i32, vp, vp, vp, i32, vp]),
        "orc_dense_mlp": (None, [vp, i32, vp, i32] + [vp] * 9 + [vp, vp, vp, vp]),
        "orc_prep_head": (f32, [vp, vp, vp, vp, i32, i32, i32, vp, vp]),
        "orc_bq_attn_prep": (None, [vp, vp, vp, vp, vp, i32, vp, vp, i32, i32, i32, i32, i32, vp, vp]
                             + [vp] * 7),
        "orc_bq_flash_decode": (None, [vp] * 7 + [i32, vp, vp, i32, i32, i32, i32, i32, vp]),
        "orc_bq_moe_forward": (i32, [vp, i32, vp, i32, vp, vp, vp, vp]),
        "orc_bf16_moe_forward": (i32, [vp, i32, vp, i32, vp, vp, vp, vp]),
        "orc_num_threads": (i32, []),
        "orc_set_num_threads": (None, [i32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


# ------------------------------------------------------------ bf16 helpers
def f32_to_bf16(a):
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = a.view(np.uint32).astype(np.uint64)
    r = (b + ((b >> 16) & 1) + 0x7FFF) >> 16
    return r.astype(np.uint16)


def bf16_to_f32(b):
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------ prep / quantizer
def bake_split_gain(g):
    out = np.empty_like(g)
    lib().orc_bake_split_gain(_p(g), _p(out), g.size)
    return out


def bake_router_scale(s):
    out = np.empty_like(s)
    lib().orc_bake_router_scale(_p(s), _p(out), s.size)
    return out


def router_center(w):
    w = np.ascontiguousarray(w)
    out = np.empty_like(w)
    lib().orc_router_center(_p(w), w.shape[0], w.shape[1], _p(out))
    return out


def quantize_rows(w, block, gamma=None):
    w = np.ascontiguousarray(w.reshape(-1, w.shape[-1]))
    rows, cols = w.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.float32)
    g = np.ascontiguousarray(gamma) if gamma is not None else None
    lib().orc_quantize_rows(_p(w), rows, cols, _p(g), block, _p(q), _p(s))
    return q, s


def vnni_pack(q):
    q = np.ascontiguousarray(q)
    out = np.empty_like(q)
    lib().orc_vnni_pack(_p(q), q.shape[0], q.shape[1], _p(out))
    return out


def vnni_unpack(p, rows, cols):
    p = np.ascontiguousarray(p)
    out = np.empty((rows, cols), np.int8)
    lib().orc_vnni_unpack(_p(p), rows, cols, _p(out))
    return out


def colsum(q, block_cols, row_major):
    q = np.ascontiguousarray(q)
    rows, cols = q.shape
    nb = cols // block_cols
    out = np.empty((rows, nb) if row_major else (nb, rows), np.float32)
    lib().orc_colsum(_p(q), rows, cols, block_cols, _p(out), int(row_major))
    return out


def fwht_rows(v, block):
    v = np.ascontiguousarray(v, dtype=np.float32).copy()
    lib().orc_fwht_rows(_p(v), v.shape[0], v.shape[1], block)
    return v


# ------------------------------------------------------------ stages
def router(x, wr, rscale, pes):
    T = x.shape[0]
    idx = np.empty((T, TOPK), np.int32)
    w = np.empty((T, TOPK), np.float32)
    lg = np.empty((T, E), np.float32)
    lib().orc_router(_p(x), T, _p(wr), _p(rscale), _p(pes), _p(idx), _p(w), _p(lg))
    return idx, w, lg


ROUTE_DTYPE = np.dtype([("token", np.int32), ("weight", np.float32)])


def build_schedules(idx, w, expert_base, epr):
    T = idx.shape[0]
    off = np.empty(epr + 1, np.int32)
    routes = np.zeros(T * TOPK, ROUTE_DTYPE)
    lib().orc_build_schedules(_p(idx), _p(w), T, expert_base, epr, _p(off), _p(routes))
    return off, routes[:off[-1]]


def rms_norm(x, gamma):
    out = np.empty_like(x)
    lib().orc_rms_norm(_p(x), _p(gamma), x.shape[0], _p(out))
    return out


def norm_residual_add(src, residual, w):
    """bf16(residual + src * inv_rms(src) * w) per token (kernels/rmsnorm.mojo:48-64)."""
    out = np.empty_like(residual)
    lib().orc_norm_residual_add(_p(src), _p(residual), _p(w), src.shape[0], _p(out))
    return out


def post_moe(moe, dense, x_main, w1, w2, w, layer_scalar):
    """The post-MoE tail of dispatch_bq_ffn (post norms, residual, layer scalar)."""
    T = moe.shape[0]
    out = np.empty((T, H), np.uint16)
    a = [np.ascontiguousarray(v) for v in (moe, dense, x_main, w1, w2, w)]
    lib().orc_post_moe(*[_p(v) for v in a], float(layer_scalar), T, _p(out))
    return out


def bq_norm_quant(x, gamma):
    T = x.shape[0]
    q = np.empty((T, H), np.int8)
    sa = np.empty(T, np.float32)
    lib().orc_bq_norm_quant(_p(x), _p(gamma), T, _p(q), _p(sa))
    return q, sa


def bq_phase1(xi8, xsa, off, routes, gu_q, gu_scale, gu_cs, epr):
    R = int(off[-1])
    bucket = np.empty((max(R, 1), I), np.uint16)
    routes = np.ascontiguousarray(routes, ROUTE_DTYPE)
    lib().orc_bq_phase1(_p(xi8), _p(xsa), _p(off), _p(routes), _p(gu_q), _p(gu_scale),
                        _p(gu_cs), epr, _p(bucket))
    return bucket[:R]


def bq_block_quant(bucket, block=DOWN_BLOCK):
    bucket = np.ascontiguousarray(bucket)
    R, cols = bucket.shape
    q = np.empty((R, cols), np.int8)
    sa = np.empty((R, cols // block), np.float32)
    lib().orc_bq_block_quant(_p(bucket), R, cols, block, _p(q), _p(sa))
    return q, sa


def bq_phase2(bi8, bsa, off, routes, dn_q, dn_scale, dn_cs, cs_stride, epr, T):
    out = np.empty((T, H), np.uint16)
    routes = np.ascontiguousarray(routes, ROUTE_DTYPE)
    lib().orc_bq_phase2(_p(bi8), _p(bsa), _p(off), _p(routes), _p(dn_q), _p(dn_scale),
                        _p(dn_cs), cs_stride, epr, T, _p(out))
    return out


# ------------------------------------------------------------ dense MLP
DENSE_I = 2112


def bq_linear(xi8, xsa, w, ws, cs):
    """dispatch_bq_linear: bf16 [T][n_rows] from x_i8/x_sa and a row-major int8 weight."""
    T, k = xi8.shape
    n = w.shape[0]
    out = np.empty((T, n), np.uint16)
    lib().orc_bq_linear(_p(np.ascontiguousarray(xi8)), _p(np.ascontiguousarray(xsa)), T,
                        _p(np.ascontiguousarray(w)), _p(ws), _p(cs), n, k, _p(out))
    return out


def gelu_gate_up(g, u):
    out = np.empty_like(g)
    lib().orc_gelu_gate_up(_p(np.ascontiguousarray(g)), _p(np.ascontiguousarray(u)), g.size, _p(out))
    return out


def bq_block_linear(hi8, hsa, w, ws, cs_block_major):
    """dispatch_bq_block_linear: bf16 [T][n_rows]; cs block-major [k/64][n_rows]."""
    T, k = hi8.shape
    n = w.shape[0]
    out = np.empty((T, n), np.uint16)
    lib().orc_bq_block_linear(_p(np.ascontiguousarray(hi8)), _p(np.ascontiguousarray(hsa)), T, k,
                              _p(np.ascontiguousarray(w)), _p(ws), _p(cs_block_major), n, _p(out))
    return out


def bq_block_quant_ex(x, block, apply_fwht):
    """prepare_block_activation[block, apply_fwht] on bf16 rows: (int8, amax [rows][cols/block])."""
    x = np.ascontiguousarray(x)
    R, cols = x.shape
    q = np.empty((R, cols), np.int8)
    sa = np.empty((R, cols // block), np.float32)
    lib().orc_bq_block_quant_ex(_p(x), R, cols, block, 1 if apply_fwht else 0, _p(q), _p(sa))
    return q, sa


def bq_block_linear_ex(hi8, hsa, w, ws, cs_block_major, block):
    """gemm_i8_per_block for any block: bf16 [T][n_rows]; cs [k/block][n_rows]."""
    T, k = hi8.shape
    n = w.shape[0]
    out = np.empty((T, n), np.uint16)
    lib().orc_bq_block_linear_ex(_p(np.ascontiguousarray(hi8)), _p(np.ascontiguousarray(hsa)), T, k, block,
                                 _p(np.ascontiguousarray(w)), _p(ws), _p(cs_block_major), n, _p(out))
    return out


def dense_mlp(x, d):
    """The dense MLP of dispatch_bq_ffn on layer dict d (row-major int8 weights
    wg/wu [2112][2816], wd [2816][2112], scales, colsums, gamma baked).
    Returns (dense_out, h_bf16, h_i8, h_sa)."""
    T = x.shape[0]
    inter = d["wg"].shape[0]
    out = np.empty((T, H), np.uint16)
    hb = np.empty((T, inter), np.uint16)
    hq = np.empty((T, inter), np.int8)
    hs = np.empty((T, inter // DOWN_BLOCK), np.float32)
    a = [np.ascontiguousarray(d[k]) for k in ("wg", "wgs", "wgcs", "wu", "wus", "wucs", "wd", "wds",
                                              "wdcs")]
    lib().orc_dense_mlp(_p(np.ascontiguousarray(x)), T, _p(np.ascontiguousarray(d["gamma"])), inter,
                        *[_p(v) for v in a], _p(out), _p(hb), _p(hq), _p(hs))
    return out, hb, hq, hs


def phase1_bf16(xn, off, routes, w_gu, epr):
    R = int(off[-1])
    bucket = np.empty((max(R, 1), I), np.uint16)
    routes = np.ascontiguousarray(routes, ROUTE_DTYPE)
    lib().orc_phase1_bf16(_p(xn), _p(off), _p(routes), _p(w_gu), epr, _p(bucket))
    return bucket[:R]


def phase2_bf16(off, routes, bucket, w_dn, epr, T):
    out = np.empty((T, H), np.uint16)
    routes = np.ascontiguousarray(routes, ROUTE_DTYPE)
    bucket = np.ascontiguousarray(bucket)
    lib().orc_phase2_bf16(_p(off), _p(routes), _p(bucket), _p(w_dn), epr, T, _p(out))
    return out


# ------------------------------------------------------------ whole block
def bq_forward(x, layer, degree=1):
    """layer: dict with router_centered, router_scale, pes, gamma2, gu_q,
    gu_scale, gu_cs, dn_q, dn_scale, dn_cs (numpy, see OrcBqLayer)."""
    T = x.shape[0]
    keep = {k: np.ascontiguousarray(layer[k]) for k in (
        "router_centered", "router_scale", "pes", "gamma2", "gu_q", "gu_scale",
        "gu_cs", "dn_q", "dn_scale", "dn_cs")}
    L = OrcBqLayer(**{k: v.ctypes.data for k, v in keep.items()})
    out = np.empty((T, H), np.uint16)
    idx = np.empty((T, TOPK), np.int32)
    w = np.empty((T, TOPK), np.float32)
    lg = np.empty((T, E), np.float32)
    rc = lib().orc_bq_moe_forward(_p(np.ascontiguousarray(x)), T, C.byref(L), degree,
                                  _p(out), _p(idx), _p(w), _p(lg))
    assert rc == 0
    return out, idx, w, lg


def bf16_forward(x, layer, degree=1):
    T = x.shape[0]
    keep = {k: np.ascontiguousarray(layer[k]) for k in (
        "router_proj", "router_scale", "pes", "gamma2", "w_gu", "w_dn")}
    L = OrcBf16Layer(**{k: v.ctypes.data for k, v in keep.items()})
    out = np.empty((T, H), np.uint16)
    idx = np.empty((T, TOPK), np.int32)
    w = np.empty((T, TOPK), np.float32)
    lg = np.empty((T, E), np.float32)
    rc = lib().orc_bf16_moe_forward(_p(np.ascontiguousarray(x)), T, C.byref(L), degree,
                                    _p(out), _p(idx), _p(w), _p(lg))
    assert rc == 0
    return out, idx, w, lg


# ------------------------------------------------------------ bq attention
def bq_attn_prep(q_src, k_src, v_src, q_norm, k_norm, pos, slot, head_dim, num_q, num_kv,
                 rope_half, pair_stride, cos_table, sin_table, n_slots):
    """BqAttnPrepKernel for T tokens: returns q_i8, qi_bias, f_q and the K/V
    cache rows (int8 [n_slots][num_kv*head_dim], scales [n_slots][num_kv]) with
    the tokens' rows written at slot[t] (rows not written stay zero)."""
    T = q_src.shape[0]
    q_i8 = np.zeros((T, num_q * head_dim), np.int8)
    qb = np.zeros((T, num_q), np.float32)
    fq = np.zeros((T, num_q), np.float32)
    kc = np.zeros((n_slots, num_kv * head_dim), np.int8)
    ks = np.zeros((n_slots, num_kv), np.float32)
    vc = np.zeros_like(kc)
    vs = np.zeros_like(ks)
    a = [np.ascontiguousarray(v) for v in (q_src, k_src, v_src, q_norm, k_norm)]
    lib().orc_bq_attn_prep(*[_p(v) for v in a], T, _p(np.ascontiguousarray(pos, np.int32)),
                           _p(np.ascontiguousarray(slot, np.int32)), head_dim, num_q, num_kv,
                           rope_half, pair_stride, _p(np.ascontiguousarray(cos_table, np.float32)),
                           _p(np.ascontiguousarray(sin_table, np.float32)), _p(q_i8), _p(qb), _p(fq),
                           _p(kc), _p(ks), _p(vc), _p(vs))
    return q_i8, qb, fq, kc, ks, vc, vs


def bq_flash_decode(q_i8, qi_bias, f_q, k_cache, k_scale, v_cache, v_scale, slots, kv_len,
                    head_dim, num_q, num_kv, n_splits=1):
    """Flash decode of T query tokens over their cache rows `slots`
    ([T][max_kv], position order, kv_len[t] valid) with n_splits worker
    ranges merged as the reference does; bf16 [T][num_q*head_dim]."""
    T = q_i8.shape[0]
    slots = np.ascontiguousarray(slots, np.int32)
    out = np.empty((T, num_q * head_dim), np.uint16)
    a = [np.ascontiguousarray(v) for v in (q_i8, qi_bias, f_q, k_cache, k_scale, v_cache, v_scale)]
    lib().orc_bq_flash_decode(*[_p(v) for v in a], T, _p(slots), _p(np.ascontiguousarray(kv_len, np.int32)),
                              slots.shape[1], head_dim, num_q, num_kv, n_splits, _p(out))
    return out
