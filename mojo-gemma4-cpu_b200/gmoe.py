"""Python binding of libgmoe.so (include/gmoe.h) over ctypes.

Host-side mirror of the reference's MoE operator (dispatch_bq_moe,
modeling/gemma_4_moe_bq.mojo:630-713; dispatch_moe, modeling/gemma_4_moe.mojo:
493-566): `MoeBlock.forward(layer, x, out, T)` with the reference's argument
meaning (x_input -> moe_out, seq_len tokens).  Device buffers are passed as raw
addresses (torch tensors' data_ptr(), or any integer address); torch is only
the allocator used by tests and the benchmark, never a compute path here.

The library is required: importing this module on a machine without
libgmoe.so raises, and every call that returns a non-zero status raises
GmoeError with the library's error text.  There is no fallback path.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgmoe.so")

HIDDEN, NUM_EXPERTS, TOP_K, INTERMEDIATE, GATE_UP, DOWN_BLOCK = 2816, 128, 8, 704, 1408, 64
NB_DOWN = INTERMEDIATE // DOWN_BLOCK
ROUTE_CHUNK_BQ, ROUTE_CHUNK_BF16 = 16, 8

STATUS = {0: "GM_OK", -1: "GM_EINVAL", -2: "GM_ECUDA", -3: "GM_ENOMEM", -4: "GM_ENCCL",
          -5: "GM_ETIMEOUT", -6: "GM_ESTATE"}

# Every symbol include/gmoe.h declares, with its ctypes signature.
_vp, _i32, _i64, _sz = C.c_void_p, C.c_int, C.c_long, C.c_size_t


class StageStat(C.Structure):
    """gm_stage_stat_t: one stage label's statistics (times in ms)."""
    _fields_ = [("label", C.c_char * 32), ("calls", C.c_long), ("kernels", C.c_long),
                ("total_ms", C.c_double), ("min_ms", C.c_double), ("max_ms", C.c_double)]


SIGNATURES = {
    "gm_version": (C.c_char_p, []),
    "gm_last_error": (C.c_char_p, [_vp]),
    "gm_moe_create": (_i32, [C.POINTER(_vp), _i32, _i32, _i32, _i32, _i32]),
    "gm_moe_destroy": (_i32, [_vp]),
    "gm_moe_workspace_bytes": (_sz, [_i32]),
    "gm_router_workspace_bytes": (_sz, [_i32]),
    "gm_moe_register_layer_bq": (_i32, [_vp, _i32] + [_vp] * 8),
    "gm_moe_register_layer_bf16": (_i32, [_vp, _i32] + [_vp] * 6),
    "gm_moe_forward": (_i32, [_vp, _i32, _vp, _vp, _i32, _vp]),
    "gm_moe_forward_sync": (_i32, [_vp, _i32, _vp, _vp, _i32]),
    "gm_moe_set_option": (_i32, [_vp, _i32, _i64]),
    "gm_moe_register_post": (_i32, [_vp, _i32, _vp, _vp, _vp, C.c_float]),
    "gm_moe_forward_ffn": (_i32, [_vp, _i32, _vp, _vp, _i32, _vp]),
    "gm_moe_device_status": (_i32, [_vp, C.POINTER(_i32)]),
    "gm_ep_unique_id": (_i32, [_vp, _sz]),
    "gm_moe_ep_init": (_i32, [_vp, _vp, _i32]),
    "gm_moe_ep_set_placement": (_i32, [_vp, C.POINTER(_i32)]),
    "gm_moe_ep_init_group": (_i32, [C.POINTER(_vp), _i32]),
    "gm_moe_ep_forward_group": (_i32, [C.POINTER(_vp), _i32, _i32, C.POINTER(_vp), C.POINTER(_vp),
                                        C.POINTER(_i32), C.POINTER(_vp)]),
    "gm_moe_ep_set_placement_group": (_i32, [C.POINTER(_vp), _i32, C.POINTER(_i32)]),
    "gm_moe_profile_read": (_i32, [_vp, C.POINTER(StageStat), _i32, C.POINTER(_i32), C.POINTER(_i64)]),
    "gm_router_select": (_i32, [_vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    "gm_router_select_noalloc": (_i32, [_vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp]),
    "gm_build_expert_schedules": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "gm_rms_norm": (_i32, [_vp, _vp, _i32, _vp, _vp]),
    "gm_norm_residual_add": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "gm_bq_norm_quant": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp]),
    "gm_bq_phase1_gate_up": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "gm_bq_block_quant": (_i32, [_vp, _i64, _vp, _vp, _vp]),
    "gm_bq_phase2_down": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp]),
    "gm_phase1_gate_up_bf16": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp, _vp]),
    "gm_phase2_down_bf16": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp, _vp]),
    "gm_combine": (_i32, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "gm_bq_quantize_rows": (_i32, [_vp, _i64, _i32, _vp, _i32, _vp, _vp, _vp]),
    "gm_vnni_pack": (_i32, [_vp, _i64, _i32, _vp, _vp]),
    "gm_vnni_unpack": (_i32, [_vp, _i64, _i32, _vp, _vp]),
    "gm_router_center": (_i32, [_vp, _i32, _i32, _vp, _vp]),
    "gm_bake_split_gain": (_i32, [_vp, _vp, _i32, _vp]),
    "gm_bake_router_scale": (_i32, [_vp, _vp, _i32, _vp]),
    "gm_moe_register_dense_bq": (_i32, [_vp, _i32] + [_vp] * 7),
    "gm_dense_forward": (_i32, [_vp, _i32, _vp, _vp, _i32, _vp]),
    "gm_ffn_forward": (_i32, [_vp, _i32, _vp, _i32, _vp]),
    "gm_bq_dense_gate_up": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "gm_bq_block_linear": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    "gm_bq_linear": (_i32, [_vp, _vp, _i32, _vp, _vp, _i32, _vp, _vp]),
    "gm_bq_qkv": (_i32, [_vp, _vp, _i32, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    "gm_bq_block_quant_ex": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp]),
    "gm_bq_block_linear_ex": (_i32, [_vp, _vp, _i32, _i32, _i32, _vp, _vp, _i32, _vp, _vp]),
    "gm_bq_attn_prep": (_i32, [_vp] * 14 + [_vp, _i32, _vp] + [_i32] * 11 + [_vp]),
    "gm_bq_attention_decode": (_i32, [_vp] * 8 + [_i32] * 11 + [_vp, _vp, _sz, _vp]),
    "gm_bq_attention_prefill": (_i32, [_vp] * 7 + [_i32, _vp] + [_i32] * 8 + [_vp, _vp]),
    "gm_bq_attention_workspace_bytes": (_sz, [_i32] * 5),
    "gm_bq_attention_partial_bytes": (_sz, [_i32] * 3),
    "gm_bq_attention_partial": (_i32, [_vp] * 8 + [_i32] * 11 + [_vp, _vp, _sz, _vp]),
    "gm_bq_attention_merge": (_i32, [C.POINTER(_vp), _i32, _i32, _i32, _i32, _vp, _vp]),
    "gm_checkpoint_open": (_i32, [C.POINTER(_vp), C.c_char_p]),
    "gm_checkpoint_close": (_i32, [_vp]),
    "gm_checkpoint_tensor_count": (_i32, [_vp]),
    "gm_checkpoint_tensor_name": (C.c_char_p, [_vp, _i32]),
    "gm_checkpoint_tensor_info": (_i32, [_vp, C.c_char_p, C.POINTER(_i32), C.POINTER(_i32),
                                         C.POINTER(C.c_int64)]),
    "gm_checkpoint_read_rows": (_i32, [_vp, C.c_char_p, C.c_int64, C.c_int64, _vp, _sz]),
    "gm_moe_load_layer": (_i32, [_vp, _i32, _vp, _i32, C.c_char_p, _i32]),
}


class GmoeError(RuntimeError):
    pass


_LIB = None


def lib():
    """Load libgmoe.so (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise GmoeError("libgmoe.so not built at %s (run __graft_entry__.build())" % LIB_PATH)
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def _addr(t):
    """Raw address of a tensor-like (torch tensor, numpy array, int, None)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if hasattr(t, "cuda_stream"):  # torch.cuda.Stream
        return t.cuda_stream
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if hasattr(t, "ctypes"):
        return t.ctypes.data
    raise TypeError("cannot take the address of %r" % type(t))


def _stream(s):
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream  # torch.cuda.Stream


def check(rc, handle=None):
    if rc != 0:
        msg = lib().gm_last_error(handle)
        text = msg.decode(errors="backslashreplace") if msg else ""
        raise GmoeError("%s: %s" % (STATUS.get(rc, rc), text))
    return rc


def call(name, *args):
    """Call a stateless entry point; addresses/streams are converted."""
    fn = getattr(lib(), name)
    if len(args) != len(fn.argtypes):
        raise TypeError("%s takes %d arguments, %d given" % (name, len(fn.argtypes), len(args)))
    conv = []
    for a, ty in zip(args, fn.argtypes):
        conv.append(_addr(a) if ty is _vp else a)
    return check(fn(*conv))


class MoeBlock:
    """A gm_moe_t handle: weights of `num_layers` MoE blocks plus workspace for
    `max_tokens` tokens per call, expert shard `rank` of `degree`."""

    def __init__(self, max_tokens, num_layers=1, device=0, rank=0, degree=1):
        h = C.c_void_p()
        check(lib().gm_moe_create(C.byref(h), device, max_tokens, num_layers, rank, degree))
        self.h = h
        self.max_tokens, self.num_layers, self.rank, self.degree = max_tokens, num_layers, rank, degree
        self.epr = NUM_EXPERTS // degree

    def close(self):
        if self.h:
            lib().gm_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def register_bq(self, layer, gate_up, gate_up_scale, down, down_scale, router_centered,
                    router_scale, per_expert_scale, pre_ffn_norm_2):
        check(lib().gm_moe_register_layer_bq(
            self.h, layer, _addr(gate_up), _addr(gate_up_scale), _addr(down), _addr(down_scale),
            _addr(router_centered), _addr(router_scale), _addr(per_expert_scale),
            _addr(pre_ffn_norm_2)), self.h)

    def register_bf16(self, layer, gate_up, down, router_proj, router_scale, per_expert_scale,
                      pre_ffn_norm_2):
        check(lib().gm_moe_register_layer_bf16(
            self.h, layer, _addr(gate_up), _addr(down), _addr(router_proj), _addr(router_scale),
            _addr(per_expert_scale), _addr(pre_ffn_norm_2)), self.h)

    def forward(self, layer, x, out, T, stream=None):
        """Asynchronous on `stream`: x, out device bf16 [T][2816]."""
        check(lib().gm_moe_forward(self.h, layer, _addr(x), _addr(out), T, _stream(stream)), self.h)

    def register_post(self, layer, post_ffn_norm_1, post_ffn_norm_2, post_ffn_norm, layer_scalar):
        check(lib().gm_moe_register_post(self.h, layer, _addr(post_ffn_norm_1), _addr(post_ffn_norm_2),
                                         _addr(post_ffn_norm), float(layer_scalar)), self.h)

    def forward_ffn(self, layer, x_main, dense_out, T, stream=None):
        """MoE on x_main, then the post-MoE tail; x_main is updated in place."""
        check(lib().gm_moe_forward_ffn(self.h, layer, _addr(x_main), _addr(dense_out), T,
                                       _stream(stream)), self.h)

    def register_dense(self, layer, gate_proj, gate_scale, up_proj, up_scale, down_proj,
                       down_scale, pre_ffn_norm):
        """The layer's dense butterquant MLP (VNNI-packed weights, baked gain)."""
        check(lib().gm_moe_register_dense_bq(
            self.h, layer, _addr(gate_proj), _addr(gate_scale), _addr(up_proj), _addr(up_scale),
            _addr(down_proj), _addr(down_scale), _addr(pre_ffn_norm)), self.h)

    def dense_forward(self, layer, x, dense_out, T, stream=None):
        """The dense MLP alone: x -> dense_out (device bf16 [T][2816])."""
        check(lib().gm_dense_forward(self.h, layer, _addr(x), _addr(dense_out), T, _stream(stream)),
              self.h)

    def ffn_forward(self, layer, x_main, T, stream=None):
        """Dense MLP beside the MoE, then the post-MoE tail; x_main in place."""
        check(lib().gm_ffn_forward(self.h, layer, _addr(x_main), T, _stream(stream)), self.h)

    def forward_sync(self, layer, x, out, T):
        """Blocking; x/out may be host (e.g. pinned) or device buffers."""
        check(lib().gm_moe_forward_sync(self.h, layer, _addr(x), _addr(out), T), self.h)

    def set_option(self, option, value):
        check(lib().gm_moe_set_option(self.h, option, value), self.h)

    def profile(self, on=True):
        """Turns the per-stage event profiler on or off; clears the statistics
        and the kernel launch count either way."""
        self.set_option(OPT_PROFILE, 1 if on else 0)

    def profile_read(self):
        """(stats, kernel_launches): stats maps each stage label to a dict of
        calls, kernels, total_ms, min_ms, max_ms, avg_ms (first-seen order)."""
        n, launches = C.c_int(0), C.c_long(0)
        buf = (StageStat * 64)()
        check(lib().gm_moe_profile_read(self.h, buf, 64, C.byref(n), C.byref(launches)), self.h)
        stats = {}
        for st in buf[:min(n.value, 64)]:
            stats[st.label.decode()] = {
                "calls": st.calls, "kernels": st.kernels, "total_ms": st.total_ms,
                "min_ms": st.min_ms, "max_ms": st.max_ms,
                "avg_ms": st.total_ms / st.calls if st.calls else 0.0}
        return stats, launches.value

    def ep_init(self, unique_id, world):
        """Join the expert-parallel group (collective over `world` processes)."""
        buf = C.create_string_buffer(bytes(unique_id), len(unique_id))
        check(lib().gm_moe_ep_init(self.h, buf, world), self.h)

    def ep_set_placement(self, expert_rank):
        """Collective: expert e moves to rank expert_rank[e] (128/world each)."""
        arr = (C.c_int * NUM_EXPERTS)(*[int(r) for r in expert_rank])
        check(lib().gm_moe_ep_set_placement(self.h, arr), self.h)

    def device_status(self):
        """Synchronises; raises GmoeError(GM_ETIMEOUT) if a bounded wait expired."""
        e = C.c_int(0)
        check(lib().gm_moe_device_status(self.h, C.byref(e)), self.h)
        return e.value

    def load_layer(self, layer, ckpt, ckpt_layer=None, prefix=None, post=False, dense=False,
                   quantize=False):
        """One MoE layer from a Checkpoint (this handle's experts, load-time
        bakes and packing included); the format follows the file's
        experts.gate_up_proj dtype.  prefix None: the reference's
        "model.language_model.layers.%d." with %d = ckpt_layer (default: layer).
        post / dense: also the post-MoE gains / the dense MLP; quantize: a BF16
        checkpoint becomes the butterquant layer on the device."""
        if ckpt_layer is None:
            ckpt_layer = layer
        flags = (LOAD_POST if post else 0) | (LOAD_DENSE if dense else 0) | \
                (LOAD_QUANTIZE if quantize else 0)
        check(lib().gm_moe_load_layer(self.h, layer, ckpt.h, ckpt_layer,
                                      prefix.encode() if prefix is not None else None, flags),
              self.h)


DTYPES = {1: "BOOL", 2: "U8", 3: "I8", 4: "I16", 5: "U16", 6: "F16", 7: "BF16", 8: "I32", 9: "U32",
          10: "F32", 11: "I64", 12: "U64", 13: "F64", 14: "F8_E4M3", 15: "F8_E5M2"}
LOAD_POST = 1
LOAD_DENSE = 2
LOAD_QUANTIZE = 4
CKPT_MAX_DIMS = 8


class Checkpoint:
    """A gm_checkpoint_t: one .safetensors file or a directory of shards,
    headers parsed and checked at open, tensors read on demand (no GPU)."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().gm_checkpoint_open(C.byref(h), os.fsencode(path)))
        self.h = h

    def close(self):
        if self.h:
            lib().gm_checkpoint_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def names(self):
        L = lib()
        return [L.gm_checkpoint_tensor_name(self.h, i).decode()
                for i in range(L.gm_checkpoint_tensor_count(self.h))]

    def info(self, name):
        """(dtype tag, shape tuple)."""
        dt, nd = C.c_int(0), C.c_int(0)
        shape = (C.c_int64 * CKPT_MAX_DIMS)()
        check(lib().gm_checkpoint_tensor_info(self.h, name.encode(), C.byref(dt), C.byref(nd), shape))
        return DTYPES[dt.value], tuple(shape[:nd.value])

    def read_rows(self, name, row0, nrows, out):
        """Rows [row0, row0+nrows) of the tensor folded to 2-D into `out`
        (a writable host buffer: numpy array or address with its size)."""
        nbytes = out.nbytes if hasattr(out, "nbytes") else out.numel() * out.element_size()
        check(lib().gm_checkpoint_read_rows(self.h, name.encode(), row0, nrows, _addr(out), nbytes))
        return out


OPT_TC_MIN_TOKENS = 1
OPT_PROFILE = 2
OPT_PDL = 3
OPT_EP_TRANSPORT = 4
OPT_DENSE_TC_MIN_TOKENS = 5
OPT_EP_TIMEOUT_MS = 6
OPT_EP_INIT_TIMEOUT_MS = 7
EP_UNIQUE_ID_BYTES = 128


def _handles(blocks):
    arr = (C.c_void_p * len(blocks))(*[b.h.value for b in blocks])
    return arr


def ep_init_group(blocks):
    """Joins the MoeBlocks (rank g of degree len(blocks) at index g) into one
    in-process expert-parallel group (no NCCL; members may share a GPU)."""
    check(lib().gm_moe_ep_init_group(_handles(blocks), len(blocks)))


def ep_forward_group(blocks, layer, xs, outs, Ts, streams=None):
    """One layer on every member of an in-process group: member g's Ts[g]
    tokens xs[g] -> outs[g] on streams[g] (members sharing a GPU need the same
    stream; None = the default stream for every member)."""
    n = len(blocks)
    streams = [None] * n if streams is None else streams
    xa = (C.c_void_p * n)(*[_addr(x) for x in xs])
    oa = (C.c_void_p * n)(*[_addr(o) for o in outs])
    ta = (C.c_int * n)(*[int(t) for t in Ts])
    sa = (C.c_void_p * n)(*[_stream(s) for s in streams])
    check(lib().gm_moe_ep_forward_group(_handles(blocks), n, layer, xa, oa, ta, sa))


def ep_set_placement_group(blocks, expert_rank):
    """gm_moe_ep_set_placement for an in-process group (one call for all)."""
    arr = (C.c_int * NUM_EXPERTS)(*[int(r) for r in expert_rank])
    check(lib().gm_moe_ep_set_placement_group(_handles(blocks), len(blocks), arr))


def balanced_placement(load, world):
    """Expert -> rank map with 128/world experts per rank that evens out the
    given per-expert load: experts in descending load, each to the least-loaded
    rank that still has room (longest-processing-time first)."""
    epr = NUM_EXPERTS // world
    order = sorted(range(NUM_EXPERTS), key=lambda e: (-float(load[e]), e))
    total = [0.0] * world
    count = [0] * world
    rank = [0] * NUM_EXPERTS
    for e in order:
        r = min((r for r in range(world) if count[r] < epr), key=lambda r: (total[r], r))
        rank[e] = r
        total[r] += float(load[e])
        count[r] += 1
    return rank


def ep_unique_id():
    """A fresh NCCL unique id (bytes) for gm_moe_ep_init; made on one rank and
    sent to the others by the caller."""
    buf = C.create_string_buffer(EP_UNIQUE_ID_BYTES)
    check(lib().gm_ep_unique_id(buf, EP_UNIQUE_ID_BYTES))
    return buf.raw
