#!/usr/bin/env python
"""Benchmark of the B200 Gemma-4 MoE block (BASELINE metric: MoE-block tokens/s;
headline workload = configs[1], butterquant decode batch 64).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

A step is one MoE-block forward over one batch of synthetic tokens through the
C ABI (gm_moe_forward).  `value` is tokens/s with inputs resident in HBM;
`e2e` is the same metric through the blocking entry point gm_moe_forward_sync
with pinned host buffers (H2D of x and D2H of the output inside the timed
region).  `--impl reference` times the CPU restatement of the reference path
(oracle/, the Mojo reference cannot be built here) on the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mojo-gemma4-cpu_b200")
sys.path.insert(0, ROOT)
sys.path.insert(0, PKG)

H, E, TOPK, I, GU = 2816, 128, 8, 704, 1408
BQ_EXPERT_GU_BYTES = GU * H + GU * 4          # int8 rows + f32 row scales
BQ_EXPERT_DN_BYTES = H * I + H * 4
BQ_EXPERT_BYTES = BQ_EXPERT_GU_BYTES + BQ_EXPERT_DN_BYTES   # 5,964,288
BF16_EXPERT_BYTES = (GU * H + H * I) * 2                     # 11,894,784
FLOP_PER_TOKEN = TOPK * (2 * GU * H + 2 * H * I)              # 95,158,272

WORKLOADS = {
    # name: (tokens per step, weight format, parallelism)
    #   replicas:  N independent copies, tokens per GPU fixed (weak scaling)
    #   ep-weak:   expert parallel over the N GPUs, tokens per GPU fixed
    #   ep-strong: expert parallel, tokens per step fixed in total (split over N)
    # the default: on one GPU the plain forward; on N GPUs expert parallel
    # (each GPU holds 128/N experts and 64 tokens, dispatch/combine over NCCL)
    "bq-decode-b64": (64, "bq", "ep-weak"),
    "bq-decode-b8": (8, "bq", "replicas"),
    "bq-decode-b1": (1, "bq", "replicas"),
    "bf16-decode-b16": (16, "bf16", "replicas"),
    "bq-prefill-4k": (4096, "bq", "replicas"),
    "bf16-prefill-4k": (4096, "bf16", "replicas"),
    "bq-decode-b64-replicas": (64, "bq", "replicas"),
    # Zipf(1.1) routing (expert i-1 receives 8T*i^-1.1/sum of the routes, capped at T)
    "bq-prefill-4k-zipf": (4096, "bq", "replicas"),
    "bf16-prefill-4k-zipf": (4096, "bf16", "replicas"),
    "ep-prefill-16k": (16384, "bq", "ep-strong"),
}
ZIPF = {"bq-prefill-4k-zipf", "bf16-prefill-4k-zipf", "ep-prefill-16k"}
# config 5: one decode step of 64 sequences through 30 MoE layers (distinct
# weights per layer; the MoE blocks alone, as the config states it -- decoder-b64-30L runs the whole step)
WORKLOADS["bq-decode-b64-30L"] = (64, "bq", "replicas")
LAYERS = {"bq-decode-b64-30L": 30}
REF_SAMPLE_TOKENS = 512   # tokens per step of the --impl reference arm (CPU)
METRIC = "MoE-block tokens/s at 1/2/4/8 B200 (decode b=64, prefill 4k); % of roofline"
# Workloads of the rows widened beyond the MoE block (one GPU): the whole FFN
# (dense MLP beside the MoE, post-FFN tail; gm_ffn_forward) and butterquant
# decode attention over a full KV window (gm_bq_attention_decode).
EXTRA = {
    "ffn-decode-b64": ("ffn", 64),
    "ffn-prefill-4k": ("ffn", 4096),
    "attn-decode-sliding-b64": ("attn-sliding", 64),
    "attn-decode-full-b64": ("attn-full", 64),
    "attn-prefill-sliding-4k": ("attnp-sliding", 4096),
    "attn-prefill-full-4k": ("attnp-full", 4096),
    # config 5 as a whole decoder step: 64 sequences at 8k context through 30
    # layers of attention block + FFN (dense MLP, MoE, post-FFN tail)
    "decoder-b64-30L": ("decoder", 64),
}
EXTRA_TRAFFIC = {"attn-decode-full-b64": 541_900_000 + 14_200_000}
DENSE_I = 2112
DENSE_BYTES = 3 * DENSE_I * H + 2 * DENSE_I * 4 + H * 4       # int8 weights + row scales
ATTN = {  # head_dim, query heads, KV heads, window (0 = full), KV positions, pages per sequence
    "attn-sliding": (256, 16, 8, 1024, 1024, 2),
    "attn-full": (512, 16, 2, 0, 4096, 4),
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--workload", default="bq-decode-b64", choices=sorted(WORKLOADS) + sorted(EXTRA))
    p.add_argument("--impl", default="gmoe", choices=["gmoe", "reference"])
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="bounded CPU-baseline sample length")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--tokens", type=int, default=0,
                   help="profiling small cases: tokens per GPU instead of the workload's (the line's config "
                        "records the override; not a bench number)")
    p.add_argument("--batches", type=int, default=8, help="distinct token batches cycled")
    p.add_argument("--placement", default="balanced", choices=["balanced", "contiguous"],
                   help="expert placement of Zipf expert-parallel workloads")
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        import tempfile
        self.index = index
        self.proc = None
        # raw samples: GMOE_CLOCKS_DIR if set (to keep them), else a temp dir
        folder = os.environ.get("GMOE_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = os.path.join(folder, "clocks_bench_%d.csv" % os.getpid())

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[4:]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for _, _, r in rows:
            for n, v in zip(names, r[1:5]):
                if "Active" in v and "Not" not in v:
                    reasons.add(n)
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1],
                "reasons": sorted(reasons), "samples": len(rows)}


DEC_LAYERS, DEC_CTX = 30, 8192   # Gemma-4-26B-A4B: 30 layers, every 6th full attention


def run_decoder(args, T, stream, hbm):
    """One decode step of T sequences, each at position DEC_CTX - 1, through
    DEC_LAYERS decoder layers (modeling/gemma_4_moe_bq.mojo:1080-1110): per
    layer the attention block (norm-quant of x_main, q/k/v projections, head
    prep into the paged int8 cache, decode attention over the window (sliding
    layers: 1024 positions) or the whole context (full layers, (i+1) % 6 == 0:
    8192 positions), head-block quantisation, output projection into
    x_residual), the post-attention norm-residual into x_main, and the FFN
    (dense MLP beside the MoE, post-FFN tail) in place on x_main.  Every layer
    has its own weights and KV cache (random-init: the MoE, dense and q/k/v
    weights are N(0, 0.02) bf16 through the device quantizer; o_proj, whose
    K = heads x head_dim the device quantizer does not take, gets random int8
    codes and scales of the same magnitude; caches random int8)."""
    import numpy as np
    import torch
    import gmoe
    import synth
    PAGE, SHIFT = 1024, 10
    pos = DEC_CTX - 1
    g = torch.Generator(device="cuda").manual_seed(0xDEC)
    blk = gmoe.MoeBlock(T, DEC_LAYERS)
    gen = torch.Generator(device="cpu").manual_seed(0xDEC)

    def gain(n):
        return (1.0 + 0.1 * torch.randn(n, generator=gen)).to(torch.bfloat16).cuda()

    def quant(w, gamma):
        rows, cols = w.shape
        q = torch.empty(rows, cols, dtype=torch.int8, device="cuda")
        sc = torch.empty(rows, dtype=torch.float32, device="cuda")
        gmoe.call("gm_bq_quantize_rows", w, rows, cols, gamma, 128, q, sc, None)
        p = torch.empty_like(q)
        gmoe.call("gm_vnni_pack", q, rows, cols, p, None)
        return p, sc

    layers, kv_bytes, attn_w_bytes = [], 0, 0
    for l in range(DEC_LAYERS):
        full = (l + 1) % 6 == 0
        hd, nq, nkv, window, rope_half, pair_stride = (512, 16, 2, 0, 64, 256) if full else \
            (256, 16, 8, 1024, 128, 128)
        kv = DEC_CTX if full else window
        ppr = DEC_CTX // PAGE if full else 2     # sliding layers: a ring of two window-sized pages
        raw = synth.make_layer(seed=0x6E6D6F45 + 7919 * l, device="cuda")
        register(blk, "bq", synth.bq_layer(raw), layer=l)
        rawd = synth.make_dense(seed=0x0D3E + l, device="cuda")
        if l == 0:
            raw0, rawd0 = raw, rawd           # kept for the CPU leg's layers
        del raw
        D = synth.dense_layer(rawd)
        blk.register_dense(l, D["gate"], D["gate_scale"], D["up"], D["up_scale"], D["down"], D["down_scale"],
                           D["pre_ffn_norm"])
        blk.register_post(l, gain(H), gain(H), gain(H), 1.0)
        in_norm = gain(H)
        in_baked = torch.empty_like(in_norm)
        gmoe.call("gm_bake_split_gain", in_norm, in_baked, H, None)
        qn, kvn = nq * hd, nkv * hd
        wq = quant((torch.randn(qn, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16), in_norm)
        wk = quant((torch.randn(kvn, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16), in_norm)
        wv = None if full else quant((torch.randn(kvn, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16),
                                     in_norm)
        wo = (torch.randint(-127, 128, (H, qn), dtype=torch.int8, device="cuda", generator=g),
              torch.rand(H, device="cuda", generator=g) * 4e-4 + 4e-4)
        n_slots = T * ppr * PAGE
        kc = torch.randint(-127, 128, (n_slots, kvn), dtype=torch.int8, device="cuda", generator=g)
        vc = torch.randint(-127, 128, (n_slots, kvn), dtype=torch.int8, device="cuda", generator=g)
        ks = torch.rand(n_slots, nkv, device="cuda", generator=g) * 0.03
        vs = torch.rand(n_slots, nkv, device="cuda", generator=g) + 0.5
        base = (torch.randperm(T * ppr, device="cuda", generator=g).int() * PAGE).contiguous()
        ang = np.arange(DEC_CTX, dtype=np.float64)[:, None] * \
            (10000.0 ** (-np.arange(rope_half, dtype=np.float64) / rope_half))[None, :]
        kv_bytes += T * kv * nkv * (2 * hd + 8)
        attn_w_bytes += (qn + 2 * kvn if not full else qn + kvn) * (H + 4) + H * (qn + 4)
        layers.append(dict(
            full=full, hd=hd, nq=nq, nkv=nkv, window=window, kv=kv, rope_half=rope_half, pair_stride=pair_stride,
            page_mask=(ppr - 1) if window else -1, in_baked=in_baked, wq=wq, wk=wk, wv=wv, wo=wo,
            qnorm=gain(hd), knorm=gain(hd), post_attn=gain(H), kc=kc, vc=vc, ks=ks, vs=vs, base=base,
            cos=torch.from_numpy(np.cos(ang).astype(np.float32)).cuda(),
            sin=torch.from_numpy(np.sin(ang).astype(np.float32)).cuda(),
            runs=torch.tensor([[t, pos, t * ppr, ppr] for t in range(T)], dtype=torch.int32, device="cuda")))
    torch.cuda.empty_cache()
    # activations, sized for the largest layer kind
    xi8 = torch.empty(T, H, dtype=torch.int8, device="cuda")
    xsa = torch.empty(T, dtype=torch.float32, device="cuda")
    q_bf = torch.empty(T, 16 * 512, dtype=torch.bfloat16, device="cuda")
    k_bf = torch.empty(T, 8 * 256, dtype=torch.bfloat16, device="cuda")
    v_bf = torch.empty(T, 8 * 256, dtype=torch.bfloat16, device="cuda")
    q_i8 = torch.empty(T, 16 * 512, dtype=torch.int8, device="cuda")
    qb = torch.empty(T, 16, dtype=torch.float32, device="cuda")
    fq = torch.empty(T, 16, dtype=torch.float32, device="cuda")
    attn = torch.empty(T, 16 * 512, dtype=torch.bfloat16, device="cuda")
    o_i8 = torch.empty(T, 16 * 512, dtype=torch.int8, device="cuda")
    o_sa = torch.empty(T, 16, dtype=torch.float32, device="cuda")
    x_res = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    wsb = max(gmoe.lib().gm_bq_attention_workspace_bytes(T, c["hd"], c["nq"], c["nkv"], c["kv"]) for c in layers)
    ws = torch.empty(wsb // 4 + 1, dtype=torch.float32, device="cuda")

    ATTN_STAGES = ("norm_quant", "qkv", "prep", "decode", "head_quant", "o_proj", "norm_residual")

    def attention(c, x_main, stream, ev=None):
        """ev: None, or one CUDA event per stage boundary (len(ATTN_STAGES) + 1)."""
        hd, nq, nkv = c["hd"], c["nq"], c["nkv"]
        qn, kvn = nq * hd, nkv * hd
        mark = (lambda k: ev[k].record(stream)) if ev else (lambda k: None)
        mark(0)
        gmoe.call("gm_bq_norm_quant", x_main, c["in_baked"], T, xi8, xsa, stream)
        mark(1)
        wv = c["wv"]
        gmoe.call("gm_bq_qkv", xi8, xsa, T, c["wq"][0], c["wq"][1], qn, c["wk"][0], c["wk"][1],
                  wv[0] if wv else None, wv[1] if wv else None, kvn, q_bf, k_bf, v_bf if wv else None, stream)
        mark(2)
        gmoe.call("gm_bq_attn_prep", q_bf, k_bf, v_bf if wv else k_bf, c["qnorm"], c["knorm"], q_i8, qb, fq,
                  c["kc"], c["ks"], c["vc"], c["vs"], c["cos"], c["sin"], c["runs"], T, c["base"], T, hd, nq,
                  nkv, c["rope_half"], c["pair_stride"], 1, 0, SHIFT, PAGE - 1, c["page_mask"], stream)
        mark(3)
        gmoe.call("gm_bq_attention_decode", q_i8, fq, c["kc"], c["ks"], c["vc"], c["vs"], c["runs"], c["base"],
                  T, hd, nq, nkv, c["window"], 1, 0, SHIFT, PAGE - 1, c["page_mask"], c["kv"], attn, ws, wsb,
                  stream)
        mark(4)
        gmoe.call("gm_bq_block_quant_ex", attn, T, qn, hd, 0, o_i8, o_sa, stream)
        mark(5)
        gmoe.call("gm_bq_block_linear_ex", o_i8, o_sa, T, qn, hd, c["wo"][0], c["wo"][1], H, x_res, stream)
        mark(6)
        gmoe.call("gm_norm_residual_add", x_res, x_main, c["post_attn"], T, x_main, stream)
        mark(7)

    xs = [synth.make_tokens(T, seed=300 + b, device="cuda") for b in range(args.batches)]
    work = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")

    def run_layers(x_main, st, marks=None, stage_ev=None):
        for l, c in enumerate(layers):
            if marks:
                marks[l][0].record(st)
            attention(c, x_main, st, stage_ev[l] if stage_ev else None)
            if marks:
                marks[l][1].record(st)
            blk.ffn_forward(l, x_main, T, st)
        if marks:
            marks[-1][0].record(st)

    # The step's ~20 launches per layer are captured once into a CUDA graph
    # (after an eager run), so that the host's per-launch cost is paid once
    run_layers(work, stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="relaxed"):
        run_layers(work, torch.cuda.current_stream())
    torch.cuda.synchronize()

    def step(i):
        work.copy_(xs[i % len(xs)])
        graph.replay()
    ms = timed(step, args.steps, args.warmup, stream)
    per_step = ms / args.steps
    # kernels per step: 8 per attention block (norm-quant, qkv, prep, decode +
    # merge, head quant, o_proj, norm-residual) and the FFN's own count
    blk.profile(False)
    run_layers(work, stream)
    torch.cuda.synchronize()
    launches = (blk.profile_read()[1] + 8 * DEC_LAYERS) * args.steps
    # where the step goes: events around every layer's attention block and FFN
    marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(DEC_LAYERS + 1)]
    attn_ms, ffn_ms = 0.0, 0.0
    for i in range(3):
        work.copy_(xs[i % len(xs)])
        run_layers(work, stream, marks)
        torch.cuda.synchronize()
        for l in range(DEC_LAYERS):
            attn_ms += marks[l][0].elapsed_time(marks[l][1])
            ffn_ms += marks[l][1].elapsed_time(marks[l + 1][0])
    attn_ms, ffn_ms = attn_ms / 3, ffn_ms / 3
    # the attention block's stages, per layer kind (separate passes, so that
    # the stage events do not disturb the split above)
    stage_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(ATTN_STAGES) + 1)]
                for _ in range(DEC_LAYERS)]
    stage_us = {kind: {n: 0.0 for n in ATTN_STAGES} for kind in ("sliding", "full")}
    for i in range(3):
        work.copy_(xs[i % len(xs)])
        run_layers(work, stream, stage_ev=stage_ev)
        torch.cuda.synchronize()
        for l, c in enumerate(layers):
            kind = "full" if c["full"] else "sliding"
            n_kind = sum(1 for d in layers if d["full"] == c["full"])
            for k, n in enumerate(ATTN_STAGES):
                stage_us[kind][n] += 1e3 * stage_ev[l][k].elapsed_time(stage_ev[l][k + 1]) / (3 * n_kind)
    stage_us = {kind: {n: round(v, 1) for n, v in d.items()} for kind, d in stage_us.items()}
    # algorithmic bytes: every layer's routed experts (expected distinct of
    # T*8 uniform routes), dense MLP, attention weights and the KV it reads
    distinct = E * (1.0 - (1.0 - TOPK / E) ** T)
    moe_bytes = DEC_LAYERS * distinct * BQ_EXPERT_BYTES
    algo = moe_bytes + DEC_LAYERS * DENSE_BYTES + attn_w_bytes + kv_bytes
    roof = {"bound": "hbm", "achieved": algo / (per_step * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
            "note": "whole decoder step: %.2f GB of routed experts, %.2f GB dense MLP, %.2f GB attention "
                    "weights, %.2f GB KV cache per step" % (moe_bytes / 1e9, DEC_LAYERS * DENSE_BYTES / 1e9,
                                                          attn_w_bytes / 1e9, kv_bytes / 1e9)}
    xh = [x.cpu().pin_memory() for x in xs]
    oh = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()

    def e2e_step(i):
        work.copy_(xh[i % len(xh)], non_blocking=True)
        graph.replay()
        oh.copy_(work, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    for i in range(3):
        e2e_step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    e2e = T * args.steps / (time.perf_counter() - t0)
    cpu = None
    if not args.no_cpu_baseline:
        cpu = decoder_cpu_leg(args, layers, raw0, rawd0, xs[0])
    del graph
    blk.close()
    return {"metric": "decoder-step tokens/s (%d layers: attention block + FFN with the MoE block)" % DEC_LAYERS,
            "dtype": "i8", "config": {"workload": args.workload, "tokens_per_step": T, "layers": DEC_LAYERS,
                                      "context": DEC_CTX, "sliding_layers": sum(not c["full"] for c in layers),
                                      "full_layers": sum(c["full"] for c in layers), "parallelism": "single",
                                      "launch": "one CUDA graph per step (captured once)",
                                      "l2": "every layer's weights and KV cache distinct, %.1f GB read per step "
                                            "(larger than L2)" % (algo / 1e9)},
            "step_split": {"attention_ms": attn_ms, "ffn_ms": ffn_ms, "attention_stage_us_per_layer": stage_us,
                           "note": "CUDA events around each layer's attention block and FFN (MoE + dense "
                                   "MLP + tail), mean of 3 eager steps (the timed steps replay a CUDA graph)"},
            "_roof": roof, "_ms": ms, "_per_step": per_step, "_launches": launches,
            "_e2e": e2e, "_e2e_io": (T * H * 2, T * H * 2), "_cpu": cpu}


def decoder_cpu_leg(args, layers, raw, rawd, x):
    """The oracle (C++ restatement, all host threads) on a bounded sample: 4
    tokens through the first sliding and the first full layer (norm-quant,
    q/k/v products, flash decode over the layer's KV range, head quantisation,
    output projection, norm-residual, MoE, dense MLP, post-FFN tail; the head
    prep is left out), per-layer rates combined over the stack's 25 sliding
    and 5 full layers."""
    import numpy as np
    import synth
    O = oracle_native()
    h = synth.to_numpy
    Tc, PAGE, SHIFT, pos = 4, 1024, 10, DEC_CTX - 1
    Lo = oracle_bq_layer(O, {k: h(v) for k, v in raw.items()})
    Do = oracle_dense_layer(O, {k: h(v) for k, v in rawd.items()})
    rng = np.random.default_rng(5)
    xc = h(x[:Tc])
    nth = O.lib().orc_num_threads()

    def prepare(c):
        hd, nq, nkv, kv = c["hd"], c["nq"], c["nkv"], c["kv"]
        qn, kvn = nq * hd, nkv * hd
        w = {}
        for name, rows, cols, blk in (("wq", qn, H, None), ("wk", kvn, H, None), ("wv", kvn, H, None),
                                      ("wo", H, qn, hd)):
            if c[name] is None:
                continue
            q = O.vnni_unpack(h(c[name][0]), rows, cols)
            cs = O.colsum(q, cols, True).reshape(-1) if blk is None else O.colsum(q, blk, False)
            w[name] = (q, h(c[name][1]), cs)
        bh = h(c["base"])
        start = pos - kv + 1
        p = np.arange(start, start + kv)
        mask = c["page_mask"] if c["window"] else 0x7FFFFFFF
        slots = np.stack([bh[t * (len(bh) // len(h(c["runs"]))) + ((p >> SHIFT) & mask)] + (p & (PAGE - 1))
                          for t in range(Tc)]).astype(np.int32)
        caches = [h(c[k]) for k in ("kc", "ks", "vc", "vs")]
        qi = rng.integers(-127, 128, (Tc, qn), dtype=np.int8)
        qbias = (qi.reshape(Tc, nq, hd).astype(np.int64).sum(-1) * 128).astype(np.float32)
        fq = (rng.random((Tc, nq)) + 0.5).astype(np.float32)
        attn = O.f32_to_bf16(rng.standard_normal((Tc, qn)).astype(np.float32) * 0.3)
        gains = [h(c[k]) for k in ("in_baked", "post_attn")]

        def once():
            xi8, xsa = O.bq_norm_quant(xc, gains[0])
            for name in ("wq", "wk", "wv"):
                if name in w:
                    O.bq_linear(xi8, xsa, *w[name])
            O.bq_flash_decode(qi, qbias, fq, *caches, slots, np.full(Tc, kv, np.int32), hd, nq, nkv, nth)
            oq, osa = O.bq_block_quant_ex(attn, hd, False)
            xres = O.bq_block_linear_ex(oq, osa, *w["wo"], hd)
            xm = O.norm_residual_add(xres, xc, gains[1])
            moe = O.bq_forward(xm, Lo)[0]
            dense = O.dense_mlp(xm, Do)[0]
            O.post_moe(moe, dense, xm, gains[1], gains[1], gains[1], 1.0)
        return once

    sliding = next(c for c in layers if not c["full"])
    full = next(c for c in layers if c["full"])
    rate_s, n_s, w_s = median_rate(prepare(sliding), Tc, args.cpu_seconds / 2)
    rate_f, n_f, w_f = median_rate(prepare(full), Tc, args.cpu_seconds / 2)
    n_full = sum(c["full"] for c in layers)
    rate = 1.0 / ((len(layers) - n_full) / rate_s + n_full / rate_f)
    return dict({"value": rate, "unit": "tokens/s", "cores": nth, "kind": "port",
                 "sample": "%d tokens through one sliding layer (%d timed, %.0f tokens/s) and one full layer "
                           "(%d timed, %.0f tokens/s), combined over %d + %d layers; median (C++ restatement, "
                           "OpenMP)" % (Tc, n_s, rate_s, n_f, rate_f, len(layers) - n_full, n_full)},
                **host_info())


def build_layer(fmt, seed, device_rank, zipf=False):
    import synth
    raw = synth.make_layer(seed=seed, device="cuda")
    if zipf:
        raw = synth.apply_zipf(raw)
    if fmt == "bq":
        return synth.bq_layer(raw), raw
    return synth.bf16_layer(raw), raw


def register(blk, fmt, L, rank=0, degree=1, layer=0):
    """Registers this rank's experts [rank*128/degree, (rank+1)*128/degree)."""
    epr = E // degree
    lo, hi = rank * epr, (rank + 1) * epr
    if fmt == "bq":
        blk.register_bq(layer, L["gate_up"][lo * GU:hi * GU], L["gate_up_scale"][lo * GU:hi * GU],
                        L["down"][lo * H:hi * H], L["down_scale"][lo * H:hi * H],
                        L["router_centered"], L["router_scale"], L["per_expert_scale"],
                        L["pre_ffn_norm_2"])
    else:
        blk.register_bf16(layer, L["gate_up"][lo:hi], L["down"][lo:hi], L["router_proj"],
                          L["router_scale"], L["per_expert_scale"], L["pre_ffn_norm_2"])


def host_info():
    """nproc, CPU model and NUMA node count of this host."""
    model = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    try:
        numa = len([d for d in os.listdir("/sys/devices/system/node") if d.startswith("node")])
    except OSError:
        numa = None
    return {"nproc": os.cpu_count(), "cpu_model": model, "numa_nodes": numa}


def oracle_bq_layer(O, raw_cpu):
    """The reference quantizer and load-time bakes, run by the oracle on the host."""
    gu_q, gu_s = O.quantize_rows(raw_cpu["gate_up"].reshape(E * GU, H), 128, raw_cpu["pre_ffn_norm_2"])
    dn_q, dn_s = O.quantize_rows(raw_cpu["down"].reshape(E * H, I), 64)
    return {"router_centered": O.router_center(raw_cpu["router_proj"]),
            "router_scale": O.bake_router_scale(raw_cpu["router_scale"]),
            "pes": raw_cpu["per_expert_scale"], "gamma2": O.bake_split_gain(raw_cpu["pre_ffn_norm_2"]),
            "gu_q": gu_q, "gu_scale": gu_s, "gu_cs": O.colsum(gu_q, H, True).reshape(-1),
            "dn_q": dn_q, "dn_scale": dn_s, "dn_cs": O.colsum(dn_q, 64, False)}


def oracle_dense_layer(O, rawd_cpu):
    """DenseGateUp / DenseDown recipes on the host (row-major int8, colsums)."""
    wg, wgs = O.quantize_rows(rawd_cpu["gate"], 128, rawd_cpu["pre_ffn_norm"])
    wu, wus = O.quantize_rows(rawd_cpu["up"], 128, rawd_cpu["pre_ffn_norm"])
    wd, wds = O.quantize_rows(rawd_cpu["down"], 64)
    return {"wg": wg, "wgs": wgs, "wgcs": O.colsum(wg, H, True).reshape(-1),
            "wu": wu, "wus": wus, "wucs": O.colsum(wu, H, True).reshape(-1),
            "wd": wd, "wds": wds, "wdcs": O.colsum(wd, 64, False),
            "gamma": O.bake_split_gain(rawd_cpu["pre_ffn_norm"])}


def oracle_layer(fmt, raw_cpu):
    """The oracle's layer and forward for the workload's weight format."""
    from oracle import oracle as O
    if fmt == "bq":
        return oracle_bq_layer(O, raw_cpu), O.bq_forward
    L = {"router_proj": raw_cpu["router_proj"], "router_scale": O.bake_router_scale(raw_cpu["router_scale"]),
         "pes": raw_cpu["per_expert_scale"], "gamma2": raw_cpu["pre_ffn_norm_2"],
         "w_gu": raw_cpu["gate_up"], "w_dn": raw_cpu["down"]}
    return L, O.bf16_forward


def cpu_baseline_sample(fmt, T, seconds, raw_cpu, xs_cpu):
    """Time the oracle (CPU restatement of the reference path, all host cores)
    on forwards of the workload; returns (tokens/s at the median sample,
    samples, warm-up forwards, threads, per-forward ms at min / p50 / p90 /
    p99 as the reference harness reports them)."""
    from oracle import oracle as O
    import numpy as np
    L, fwd = oracle_layer(fmt, raw_cpu)
    # the reference harness protocol (benchmarks/bench_harness.mojo:7,62-84):
    # up to 30 warm-up forwards, then up to 600 timed samples, rate from the
    # median sample -- bounded here by `seconds` (a fifth for the warm-up)
    fwd(xs_cpu[0][:min(T, 4)], L)  # page the weights in
    t0, warm = time.perf_counter(), 0
    while warm < 30 and time.perf_counter() - t0 < 0.2 * seconds:
        fwd(xs_cpu[warm % len(xs_cpu)], L)
        warm += 1
    samples, t1 = [], time.perf_counter()
    while len(samples) < 600 and (time.perf_counter() - t1 < 0.8 * seconds or len(samples) < 3):
        x = xs_cpu[len(samples) % len(xs_cpu)]
        ts = time.perf_counter()
        fwd(x, L)
        samples.append(time.perf_counter() - ts)
    p50 = float(np.median(samples))
    ms = np.asarray(samples) * 1e3
    pct = {"min": round(float(ms.min()), 3), "p50": round(p50 * 1e3, 3),
           "p90": round(float(np.percentile(ms, 90)), 3), "p99": round(float(np.percentile(ms, 99)), 3)}
    return T / p50, len(samples), warm, O.lib().orc_num_threads(), pct


def run_reference(args):
    """--impl reference: the CPU restatement timed on this host (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    O = oracle_native()
    import synth
    T, fmt, _ = WORKLOADS[args.workload]
    zipf = args.workload in ZIPF
    layer = synth.make_layer(seed=0x6E6D6F45, device="cpu")
    if zipf:
        layer = synth.apply_zipf(layer)
    raw = {k: synth.to_numpy(v) for k, v in layer.items()}
    # each step is one forward of a bounded sample of the workload's tokens
    # (all of them up to REF_SAMPLE_TOKENS: the CPU's per-token rate is flat
    # beyond a few hundred tokens), so that --steps K --warmup W ends within
    # minutes even for the prefill workloads
    Ts = min(T, REF_SAMPLE_TOKENS)
    xs = [synth.to_numpy(synth.zipf_tokens(T, seed=s) if zipf else synth.make_tokens(T, seed=s))[:Ts]
          for s in range(2)]
    L, fwd = oracle_layer(fmt, raw)
    fwd(xs[0][:min(Ts, 4)], L)  # page the weights in
    for i in range(args.warmup):
        fwd(xs[i % 2], L)
    t0 = time.perf_counter()
    for i in range(args.steps):
        fwd(xs[i % 2], L)
    dt = time.perf_counter() - t0
    cores = O.lib().orc_num_threads()
    rate = args.steps * Ts / dt / LAYERS.get(args.workload, 1)
    sample = ("%d warm-up + %d timed forwards of %d of the workload's %d tokens (one per step), "
              "of the C++ restatement" % (args.warmup, args.steps, Ts, T))
    line = {"metric": METRIC, "value": rate, "unit": "tokens/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "i8" if fmt == "bq" else "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "tokens_per_step": T, "weights": fmt,
                       "reference_tokens_per_step": Ts},
            "cpu_baseline": dict({"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port",
                                  "sample": sample}, **host_info()),
            "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def timed(fn, steps, warmup, stream):
    """CUDA-event time of `steps` calls after a warm-up of >= 1 s."""
    import torch
    t_w, i = time.perf_counter(), 0
    while i < warmup or time.perf_counter() - t_w < 1.0:
        fn(i)
        i += 1
        if i % 8 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(steps):
        fn(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    return ev0.elapsed_time(ev1)


def oracle_native():
    """The oracle built for this host's instruction set (-march=native; the
    portable build if that fails), set to run on every host thread: the CPU
    legs run on rank 0 alone, and torchrun sets OMP_NUM_THREADS=1 per rank."""
    os.environ.setdefault("GMOE_ORACLE_VARIANT", "native")
    from oracle import build as ob
    try:
        ob.build("native")
    except Exception:
        os.environ["GMOE_ORACLE_VARIANT"] = "portable"
    from oracle import oracle as O
    O.lib().orc_set_num_threads(len(os.sched_getaffinity(0)))
    return O


def median_rate(fn, units, seconds):
    """The reference harness protocol, bounded: warm-up, then samples; units
    per second at the median sample."""
    import numpy as np
    fn()
    t0, warm = time.perf_counter(), 0
    while warm < 30 and time.perf_counter() - t0 < 0.2 * seconds:
        fn()
        warm += 1
    samples, t1 = [], time.perf_counter()
    while len(samples) < 600 and (time.perf_counter() - t1 < 0.8 * seconds or len(samples) < 3):
        ts = time.perf_counter()
        fn()
        samples.append(time.perf_counter() - ts)
    return units / float(np.median(samples)), len(samples), warm


def run_attn_prefill(args, kind, T, stream, hbm, tflops):
    """One prefill chunk of T tokens of one sequence (positions 0..T-1) through
    gm_bq_attention_prefill: sliding layer (head 256, 16 / 8 heads, window
    1024) or full layer (head 512, 16 / 2 heads, causal over the chunk).
    `batches` distinct (q, KV cache) sets are cycled so that the inputs exceed
    L2.  QK runs on int8 and PV on bf16 tensor-core instructions (mma.sync);
    the roofline counts both products of the algorithm."""
    import numpy as np
    import torch
    import gmoe
    hd, nq, nkv, window, _, _ = ATTN["attn" + kind[5:]]
    PAGE, SHIFT = 64, 6
    pages = (T + PAGE - 1) // PAGE
    g = torch.Generator(device="cuda").manual_seed(11)
    sets = []
    for _ in range(args.batches):
        kc = torch.randint(-127, 128, (pages * PAGE, nkv * hd), dtype=torch.int8, device="cuda", generator=g)
        vc = torch.randint(-127, 128, (pages * PAGE, nkv * hd), dtype=torch.int8, device="cuda", generator=g)
        ks = torch.rand(pages * PAGE, nkv, device="cuda", generator=g) * 0.03
        vs = torch.rand(pages * PAGE, nkv, device="cuda", generator=g) + 0.5
        q = torch.randint(-127, 128, (T, nq * hd), dtype=torch.int8, device="cuda", generator=g)
        fq = torch.rand(T, nq, device="cuda", generator=g) + 0.5
        sets.append((q, fq, kc, ks, vc, vs))
    base = (torch.randperm(pages, device="cuda", generator=g).int() * PAGE).contiguous()
    runs = torch.tensor([[0, 0, 0, pages]], dtype=torch.int32, device="cuda")
    out = torch.empty(T, nq * hd, dtype=torch.bfloat16, device="cuda")

    def call(st, q, o):
        gmoe.call("gm_bq_attention_prefill", q, st[1], st[2], st[3], st[4], st[5], runs, 1, base, T, hd, nq, nkv,
                  window, SHIFT, PAGE - 1, -1, o, stream)

    def step(i):
        st = sets[i % len(sets)]
        call(st, st[0], out)
    ms = timed(step, args.steps, args.warmup, stream)
    per_step = ms / args.steps
    positions = sum(min(p + 1, window) if window else p + 1 for p in range(T))
    # QK (int8) and PV (bf16 hi + lo weights) products, 2 FLOP per multiply-add
    # of the algorithm (the hi / lo split is not counted)
    flop = 2 * 2 * positions * nq * hd
    roof = {"bound": "tensor", "achieved": flop / (per_step * 1e-3) / 1e12, "peak": tflops, "unit": "TFLOP/s",
            "note": "QK and PV on mma.sync tensor-core instructions; peak = measured dense bf16 (tcgen05) rate"}
    qh = [st[0].cpu().pin_memory() for st in sets]
    oh = torch.empty(T, nq * hd, dtype=torch.bfloat16).pin_memory()
    qd = torch.empty_like(sets[0][0])

    def e2e_step(i):
        qd.copy_(qh[i % len(qh)], non_blocking=True)
        call(sets[i % len(sets)], qd, out)
        oh.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    for i in range(3):
        e2e_step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    e2e = T * args.steps / (time.perf_counter() - t0)
    cpu = None
    if not args.no_cpu_baseline:
        O = oracle_native()
        # a bounded sample: 8 tokens spread over the chunk, each over its own range
        sample = [int((i + 0.5) * T / 8) for i in range(8)]
        kv_len = np.array([min(p + 1, window) if window else p + 1 for p in sample], np.int32)
        slots = np.zeros((len(sample), int(kv_len.max())), np.int32)
        bh = base.cpu().numpy()
        for k, p in enumerate(sample):
            r = np.arange(p - kv_len[k] + 1, p + 1)
            slots[k, :kv_len[k]] = bh[r >> SHIFT] + (r & (PAGE - 1))
        st = sets[0]
        kch, ksh, vch, vsh = (x.cpu().numpy() for x in st[2:])
        qc = st[0][sample].cpu().numpy()
        fqc = st[1][sample].cpu().numpy()
        qbc = (qc.reshape(len(sample), nq, hd).astype(np.int64).sum(-1) * 128).astype(np.float32)
        rate, n, warm = median_rate(
            lambda: O.bq_flash_decode(qc, qbc, fqc, kch, ksh, vch, vsh, slots, kv_len, hd, nq, nkv,
                                      O.lib().orc_num_threads()),
            len(sample), args.cpu_seconds)
        # tokens/s of the whole chunk: the sample's mean range stands for the chunk's
        rate *= float(kv_len.mean()) / (positions / T)
        cpu = dict({"value": rate, "unit": "tokens/s", "cores": O.lib().orc_num_threads(), "kind": "port",
                    "sample": "%d warm-up + %d timed calls of 8 tokens spread over the chunk (mean %d KV "
                              "positions), scaled to the chunk's mean range, median (C++ restatement, "
                              "OpenMP)" % (warm, n, int(kv_len.mean()))}, **host_info())
    kv_mb = sum(x.numel() * x.element_size() for st in sets for x in st) / 1e6
    return {"metric": "prefill attention tokens/s (%s layer, %d-token chunk)" % (kind[6:], T),
            "dtype": "i8", "config": {"workload": args.workload, "tokens_per_step": T, "head_dim": hd,
                                      "q_heads": nq, "kv_heads": nkv, "window": window,
                                      "parallelism": "single",
                                      "l2": "%d distinct (q, KV cache) sets cycled, %.0f MB (larger than L2)"
                                            % (len(sets), kv_mb)},
            "_roof": roof, "_ms": ms, "_per_step": per_step, "_launches": args.steps,
            "_e2e": e2e, "_e2e_io": (T * nq * hd, T * nq * hd * 2), "_cpu": cpu}


def run_extra(args):
    """The FFN and attention workloads (one GPU; see EXTRA)."""
    import numpy as np
    import torch
    import gmoe
    import synth
    assert int(os.environ.get("WORLD_SIZE", "1")) == 1, "the FFN / attention workloads run on one GPU"
    assert args.warmup >= 3, "at least 3 warm-up steps"
    kind, T = EXTRA[args.workload]
    torch.cuda.set_device(0)
    hbm, tflops, peak_kind = peaks()
    stream = torch.cuda.current_stream()
    line = {"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "data": "synthetic (seeded; random-init, no checkpoint)"}
    with ClockSampler(0) as clk:
        if kind == "ffn":
            raw = synth.make_layer(seed=0x6E6D6F45, device="cuda")
            L = synth.bq_layer(raw)
            rawd = synth.make_dense(seed=0x0D3E, device="cuda")
            D = synth.dense_layer(rawd)
            g = torch.Generator(device="cpu").manual_seed(5)
            gains = [(1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).cuda() for _ in range(3)]
            blk = gmoe.MoeBlock(T, 1)
            register(blk, "bq", L)
            blk.register_post(0, gains[0], gains[1], gains[2], 1.0)
            blk.register_dense(0, D["gate"], D["gate_scale"], D["up"], D["up_scale"], D["down"],
                               D["down_scale"], D["pre_ffn_norm"])
            xs = [synth.make_tokens(T, seed=100 + b, device="cuda") for b in range(args.batches)]
            work = [x.clone() for x in xs]

            def step(i):
                w = work[i % len(work)]
                w.copy_(xs[i % len(xs)])          # fresh input (the FFN updates x_main in place)
                blk.ffn_forward(0, w, T, stream)
            ms = timed(step, args.steps, args.warmup, stream)
            blk.profile(False)               # zeroes the handle's launch count
            step(0)
            torch.cuda.synchronize()
            launches = blk.profile_read()[1] * args.steps   # kernels per step x timed steps
            per_step = ms / args.steps
            if T <= 256:
                moe_bytes = min(E, T * TOPK) * BQ_EXPERT_BYTES
                algo = moe_bytes + DENSE_BYTES + 4 * T * H * 2
                roof = {"bound": "hbm", "achieved": algo / (per_step * 1e-3) / 1e9, "peak": hbm,
                        "unit": "GB/s"}
            else:
                algo = T * (FLOP_PER_TOKEN + 2 * (2 * DENSE_I * H + H * DENSE_I))
                roof = {"bound": "tensor", "achieved": algo / (per_step * 1e-3) / 1e12, "peak": tflops,
                        "unit": "TFLOP/s"}
            # e2e: pinned host batch in, FFN, result out
            xh = [x.cpu().pin_memory() for x in xs]
            oh = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
            w = work[0]

            def e2e_step(i):
                w.copy_(xh[i % len(xh)], non_blocking=True)
                blk.ffn_forward(0, w, T, stream)
                oh.copy_(w, non_blocking=True)
                torch.cuda.current_stream().synchronize()
            for i in range(3):
                e2e_step(i)
            t0 = time.perf_counter()
            for i in range(args.steps):
                e2e_step(i)
            e2e = T * args.steps / (time.perf_counter() - t0)
            e2e_io = (T * H * 2, T * H * 2)
            cpu = None
            if not args.no_cpu_baseline:
                O = oracle_native()
                Lo = oracle_bq_layer(O, {k: synth.to_numpy(v) for k, v in raw.items()})
                Do = oracle_dense_layer(O, {k: synth.to_numpy(v) for k, v in rawd.items()})
                gn = [synth.to_numpy(v) for v in gains]
                Tc = min(T, 64)   # a bounded sample: at most 64 tokens per timed FFN
                xc = synth.to_numpy(xs[0][:Tc])

                def ffn_once():
                    moe = O.bq_forward(xc, Lo)[0]
                    dense = O.dense_mlp(xc, Do)[0]
                    O.post_moe(moe, dense, xc, gn[0], gn[1], gn[2], 1.0)
                rate, n, warm = median_rate(ffn_once, Tc, args.cpu_seconds)
                cpu = dict({"value": rate, "unit": "tokens/s", "cores": O.lib().orc_num_threads(),
                            "kind": "port",
                            "sample": "%d warm-up + %d timed FFNs of %d tokens (MoE + dense MLP + post tail), "
                                      "median (C++ restatement, OpenMP)" % (warm, n, Tc)}, **host_info())
            line.update({"metric": "FFN tokens/s (dense MLP + MoE + post-FFN tail, gm_ffn_forward)",
                         "dtype": "i8", "config": {"workload": args.workload, "tokens_per_step": T,
                                                   "weights": "bq", "layers": 1, "parallelism": "single"}})
            blk.close()
        elif kind == "decoder":
            line.update(run_decoder(args, T, stream, hbm))
            roof, ms, per_step, launches = line.pop("_roof"), line.pop("_ms"), line.pop("_per_step"), line.pop("_launches")
            e2e, e2e_io, cpu = line.pop("_e2e"), line.pop("_e2e_io"), line.pop("_cpu")
        elif kind.startswith("attnp"):
            line.update(run_attn_prefill(args, kind, T, stream, hbm, tflops))
            roof, ms, per_step, launches = line.pop("_roof"), line.pop("_ms"), line.pop("_per_step"), line.pop("_launches")
            e2e, e2e_io, cpu = line.pop("_e2e"), line.pop("_e2e_io"), line.pop("_cpu")
        else:
            hd, nq, nkv, window, kv, ppr = ATTN[kind]
            PAGE, SHIFT = 1024, 10
            g = torch.Generator(device="cuda").manual_seed(9)
            n_slots = T * ppr * PAGE
            kc = torch.randint(-127, 128, (n_slots, nkv * hd), dtype=torch.int8, device="cuda", generator=g)
            vc = torch.randint(-127, 128, (n_slots, nkv * hd), dtype=torch.int8, device="cuda", generator=g)
            ks = torch.rand(n_slots, nkv, device="cuda", generator=g) * 0.03
            vs = torch.rand(n_slots, nkv, device="cuda", generator=g) + 0.5
            qs = [torch.randint(-127, 128, (T, nq * hd), dtype=torch.int8, device="cuda", generator=g)
                  for _ in range(args.batches)]
            fq = torch.rand(T, nq, device="cuda", generator=g) + 0.5
            pos = (5000 if window else kv - 1)
            base = (torch.randperm(T * ppr, device="cuda", generator=g).int() * PAGE).contiguous()
            runs = torch.tensor([[t, pos, t * ppr, ppr] for t in range(T)], dtype=torch.int32, device="cuda")
            pmask = ppr - 1 if window else -1
            wsb = gmoe.lib().gm_bq_attention_workspace_bytes(T, hd, nq, nkv, kv)
            ws = torch.empty(wsb // 4 + 1, device="cuda")
            out = torch.empty(T, nq * hd, dtype=torch.bfloat16, device="cuda")

            def call(q, o):
                gmoe.call("gm_bq_attention_decode", q, fq, kc, ks, vc, vs, runs, base, T, hd, nq, nkv,
                          window, 1, 0, SHIFT, PAGE - 1, pmask, kv, o, ws, wsb, stream)

            def step(i):
                call(qs[i % len(qs)], out)
            ms = timed(step, args.steps, args.warmup, stream)
            launches = 2 * args.steps  # decode + merge kernels per call
            per_step = ms / args.steps
            algo = T * kv * nkv * (2 * hd + 8) + T * nq * hd * 3
            roof = {"bound": "hbm", "achieved": algo / (per_step * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s"}
            qh = [q.cpu().pin_memory() for q in qs]
            oh = torch.empty(T, nq * hd, dtype=torch.bfloat16).pin_memory()
            qd = torch.empty_like(qs[0])

            def e2e_step(i):
                qd.copy_(qh[i % len(qh)], non_blocking=True)
                call(qd, out)
                oh.copy_(out, non_blocking=True)
                torch.cuda.current_stream().synchronize()
            for i in range(3):
                e2e_step(i)
            t0 = time.perf_counter()
            for i in range(args.steps):
                e2e_step(i)
            e2e = T * args.steps / (time.perf_counter() - t0)
            e2e_io = (T * nq * hd, T * nq * hd * 2)
            cpu = None
            if not args.no_cpu_baseline:
                O = oracle_native()
                # a bounded sample: the oracle's flash decode of 4 of the tokens
                Tc = 4
                slots = np.zeros((Tc, kv), np.int32)
                bh = base.cpu().numpy()
                start = pos - kv + 1 if window else 0
                for t in range(Tc):
                    p = np.arange(start, start + kv)
                    slots[t] = bh[t * ppr + ((p >> SHIFT) & (pmask if window else 0x7FFFFFFF))] + (p & (PAGE - 1))
                kch, ksh, vch, vsh = kc.cpu().numpy(), ks.cpu().numpy(), vc.cpu().numpy(), vs.cpu().numpy()
                qc = qs[0][:Tc].cpu().numpy()
                fqc = fq[:Tc].cpu().numpy()
                qbc = (qc.reshape(Tc, nq, hd).astype(np.int64).sum(-1) * 128).astype(np.float32)
                kvl = np.full(Tc, kv, np.int32)
                rate, n, warm = median_rate(
                    lambda: O.bq_flash_decode(qc, qbc, fqc, kch, ksh, vch, vsh, slots, kvl, hd, nq, nkv,
                                              O.lib().orc_num_threads()),
                    Tc, args.cpu_seconds)
                cpu = dict({"value": rate, "unit": "tokens/s", "cores": O.lib().orc_num_threads(),
                            "kind": "port",
                            "sample": "%d warm-up + %d timed decode calls of %d tokens x %d KV positions, "
                                      "median (C++ restatement, OpenMP)" % (warm, n, Tc, kv)}, **host_info())
            line.update({"metric": "decode attention tokens/s (%s layer, %d KV positions)" % (kind[5:], kv),
                         "dtype": "i8", "config": {"workload": args.workload, "tokens_per_step": T,
                                                   "head_dim": hd, "q_heads": nq, "kv_heads": nkv,
                                                   "kv_positions": kv, "parallelism": "single",
                                                   "l2": "KV cache %.0f MB per step (larger than L2)"
                                                         % (T * kv * nkv * 2 * hd / 1e6)}})
    roof["frac"] = roof["achieved"] / roof["peak"]
    # DRAM bytes per call of the dominant kernel from the ncu capture of the
    # same command (profiles/attn_decode_full_b64.md); None elsewhere
    roof["traffic"] = EXTRA_TRAFFIC.get(args.workload)
    line.update({"value": T * args.steps / (ms / 1e3), "unit": "tokens/s", "ms_per_step": per_step,
                 "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": e2e_io[0],
                         "d2h_bytes_per_step": e2e_io[1]},
                 "gpu_launches": launches, "roofline": roof, "peak_source": peak_kind,
                 "clocks": clk.summary()})
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.workload in EXTRA:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm covers the MoE-block "
                              "workloads; this workload's CPU leg is its cpu_baseline"}))
            return
        return run_extra(args)
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import gmoe

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    T, fmt, mode = WORKLOADS[args.workload]
    if args.tokens > 0:
        T = args.tokens * (world if mode == "ep-strong" else 1)
    assert args.warmup >= 3, "at least 3 warm-up steps"
    ep = mode.startswith("ep")
    if mode == "ep-strong":
        assert T % world == 0, "tokens per step must split evenly over the GPUs"
        T //= world
    degree = world if ep else 1

    zipf = args.workload in ZIPF
    nl = LAYERS.get(args.workload, 1)
    L, raw = build_layer(fmt, 0x6E6D6F45, local, zipf)
    blk = gmoe.MoeBlock(T, nl, device=local, rank=rank if ep else 0, degree=degree)
    register(blk, fmt, L, rank if ep else 0, degree)
    for layer in range(1, nl):
        Ll, _ = build_layer(fmt, 0x6E6D6F45 + 7919 * layer, local, zipf)
        register(blk, fmt, Ll, rank if ep else 0, degree, layer=layer)
        del Ll
    torch.cuda.empty_cache()
    if ep and world > 1:
        # the NCCL id of the library's communicator, made on rank 0
        uid = torch.tensor(list(gmoe.ep_unique_id()) if rank == 0 else [0] * gmoe.EP_UNIQUE_ID_BYTES,
                           dtype=torch.uint8, device="cuda")
        dist.broadcast(uid, 0)
        blk.ep_init(bytes(uid.cpu().tolist()), world)
    placement, rank_of = "contiguous", None
    if ep and world > 1 and zipf and args.placement == "balanced":
        # experts spread by their expected Zipf load (the C ABI still takes the
        # reference's contiguous blocks; the library moves the weights)
        import synth
        rank_of = gmoe.balanced_placement(synth.zipf_targets(T * world), world)
        blk.ep_set_placement(rank_of)
        placement = "balanced (Zipf target load, longest-processing-time first)"
    g = torch.Generator(device="cuda")
    g.manual_seed(1000 + rank)
    if zipf:
        import synth
        xs = [synth.zipf_tokens(T, seed=1000 + 97 * rank + b, device="cuda") for b in range(args.batches)]
    else:
        xs = [torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16) for _ in range(args.batches)]
    outs = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in range(args.batches)]
    stream = torch.cuda.current_stream()

    tmp = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in range(2)]

    def step(i, x=None, out=None):
        """One step: the MoE block of every layer, each layer's output the next
        layer's input."""
        x = xs[i % len(xs)] if x is None else x
        out = outs[i % len(xs)] if out is None else out
        for layer in range(nl):
            dst = out if layer == nl - 1 else tmp[layer % 2]
            blk.forward(layer, x, dst, T, stream)
            x = dst

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # The clock sampler runs from the warm-up through the timed region; the
    # warm-up lasts at least 1 s so that the GPU's power and clocks have settled
    # under this load (and nvidia-smi sees it) before the timed region.
    with ClockSampler(local) as clk:
        if dist:
            # every rank must run the same forwards (the expert-parallel forward
            # holds collectives): the warm-up length comes from the slowest rank
            for i in range(3):
                step(i)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for i in range(3):
                step(i)
            torch.cuda.synchronize()
            per = torch.tensor([(time.perf_counter() - t0) / 3], device="cuda")
            dist.all_reduce(per, op=dist.ReduceOp.MAX)
            n_warm = max(args.warmup, int(1.0 / max(float(per.item()), 1e-6)) + 1)
            for i in range(n_warm):
                step(i)
                if i % 8 == 7:
                    torch.cuda.synchronize()
        else:
            t_w = time.perf_counter()
            i = 0
            while i < args.warmup or time.perf_counter() - t_w < 1.0:
                step(i)
                i += 1
                if i % 8 == 0:
                    torch.cuda.synchronize()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        blk.profile(False)           # profiler off; zeroes the handle's kernel launch count
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        torch.cuda.synchronize()
        _, timed_launches = blk.profile_read()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    value = world * T * args.steps / (ms / 1e3)

    # ---- end to end through the public API with pinned host buffers: the
    # blocking entry point for one layer; with several layers the host batch is
    # copied in, every layer runs on the device and the result is copied out
    xh = [x.cpu().pin_memory() for x in xs]
    oh = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    xin = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    yout = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")

    def e2e_step(i):
        if nl == 1:
            blk.forward_sync(0, xh[i % len(xh)], oh, T)
        else:
            xin.copy_(xh[i % len(xh)], non_blocking=True)
            step(i, xin, yout)
            oh.copy_(yout, non_blocking=True)
            torch.cuda.current_stream().synchronize()

    for i in range(3):
        e2e_step(i)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * T * args.steps / e2e_s

    # ---- roofline of the dominant kernel: CUDA events on the forward's stream
    # around each stage of the same forward (handle's stage profiler)
    roof = roofline(blk, fmt, L, xs, outs, T, args.steps, stream, args.workload, rank, world, ep, dist,
                    rank_of)

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if mode == "ep-strong" else "weak", "vs_baseline": None,
        "dtype": "i8" if fmt == "bq" else "bf16",
        "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights; random-init, no checkpoint)",
        "config": {"workload": args.workload + (" (tokens override %d)" % args.tokens if args.tokens else ""),
                   "tokens_per_step": T * world, "tokens_per_gpu": T,
                   "weights": fmt, "layers": nl, "expert_placement": placement if ep and world > 1 else None,
                   "parallelism": ("ep%d" % world) if ep and world > 1 else ("replicas" if world > 1 else "single"),
                   "l2": "inputs larger than L2: %d distinct token batches, routed expert weights %.0f MB per step"
                         % (len(xs), roof.get("weight_mb", 0))},
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2},
        "gpu_launches": timed_launches,
        "roofline": {k: roof[k] for k in ("bound", "achieved", "peak", "unit", "frac", "traffic")},
        "roofline_detail": roof["detail"],
        "routing": dict(roof["routing"], kind="zipf(1.1)" if zipf else "uniform"),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_leg(fmt, T, args, raw)
    if rank == 0:
        print(json.dumps(line), flush=True)
    blk.close()
    if dist:
        dist.destroy_process_group()


def cpu_leg(fmt, T, args, raw_dev):
    import synth
    oracle_native()
    raw_cpu = {k: synth.to_numpy(v) for k, v in raw_dev.items()}
    import torch
    g = torch.Generator(device="cpu")
    g.manual_seed(7)
    if args.workload in ZIPF:
        xs = [synth.to_numpy(synth.zipf_tokens(T, seed=7 + b)) for b in range(2)]
    else:
        xs = [synth.to_numpy(torch.randn(T, H, generator=g).to(torch.bfloat16)) for _ in range(2)]
    rate, n, warm, cores, pct = cpu_baseline_sample(fmt, T, args.cpu_seconds, raw_cpu, xs)
    nl = LAYERS.get(args.workload, 1)
    return dict({"value": rate / nl, "unit": "tokens/s", "cores": cores, "kind": "port",
                 "forward_ms": pct,
                 "sample": "%d warm-up + %d timed forwards of %d tokens, median (C++ restatement of "
                           "the reference path, OpenMP)%s" % (warm, n, T, (
                               "; one layer timed, rate divided by %d layers" % nl) if nl > 1 else "")},
                **host_info())


# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) of
# the dominant kernel, from the ncu captures of the same bench command
# summarised under profiles/ (bq_decode_b64.md, bq_prefill_4k_zipf_tcgen05.md,
# bf16_prefill_4k_tcgen05.md); None where no capture of the current kernel
# and workload exists.
NCU_TRAFFIC = {
    ("bq-decode-b64", "bq_phase1_gate_up"): 508_446_720 + 7_229_952,
    ("bq-prefill-4k-zipf", "bq_phase2_down.tc"): 280_055_808 + 353_800_192,
    ("bf16-prefill-4k", "phase1_gate_up.tc"): 1_229_532_000 + 45_981_184,
}


def stage_model(label, fmt, T, distinct, R):
    """(bound, algorithmic bytes or FLOPs per launch) of one forward stage.
    T: this GPU's tokens; R: routes into this GPU's experts (T*8 without
    expert parallelism); distinct: this GPU's experts that receive a route.
    Bytes count every operand once: routed expert weights (distinct experts
    x bytes per expert), activations read, results written."""
    ksplit = H // 256
    if label == "bq_phase1_gate_up":
        return "hbm", distinct * BQ_EXPERT_GU_BYTES + R * (H + 4) // TOPK + R * (I + 11 * 4)
    if label == "bq_phase2_down":
        return "hbm", distinct * BQ_EXPERT_DN_BYTES + R * (I + 11 * 4) + R * H * 4
    if label == "bq_phase1_gate_up.tc":
        return "tensor", 2.0 * R * GU * H
    if label == "bq_phase2_down.tc":
        return "tensor", 2.0 * R * H * I
    if label == "phase1_gate_up.tc":
        return "tensor", 2.0 * R * GU * H
    if label == "phase2_down.tc":
        return "tensor", 2.0 * R * H * I
    if label == "phase1_gate_up":
        if R >= 8 * 1024:
            return "tensor", 2.0 * R * GU * H
        return "hbm", distinct * GU * H * 2 + R * H * 2 // TOPK + R * I * 2
    if label == "phase2_down":
        if R >= 8 * 1024:
            return "tensor", 2.0 * R * H * I
        return "hbm", distinct * H * I * 2 + R * I * 2 + R * H * 4
    if label == "router_expert":
        return "hbm", E * H * 2 + T * H * 2 + H * 2 + T * 4 + ksplit * T * E * 4
    if label in ("router_merge.schedule", "router_merge"):
        return "hbm", ksplit * T * E * 4 + T * TOPK * (4 + 4 + 8 + 4)
    if label == "bq_norm_quant":
        return "hbm", T * H * 2 + H * 2 + T * H + T * 8
    if label == "rms_norm":
        return "hbm", T * H * 2 + H * 2 + T * H * 2 + T * 4
    if label == "bq_norm_gather":
        return "hbm", T * H * 2 + H * 2 + T * 4 + T * TOPK * 4 + R * (H + 4)
    if label == "rms_norm_gather":
        return "hbm", T * H * 2 + H * 2 + T * 4 + T * TOPK * 4 + R * H * 2
    if label == "gather_rows":
        return "hbm", R * (H + 4) * 2 + R * 8
    if label == "combine":
        return "hbm", R * H * 4 + (R // TOPK) * H * 2 + R * 8
    return "hbm", None


def roofline(blk, fmt, L, xs, outs, T, steps, stream, workload, rank=0, world=1, ep=False, dist=None,
             rank_of=None):
    """Per-stage device times of the forward itself: the handle's stage
    profiler (GM_OPT_PROFILE) records CUDA events on the forward's stream
    around every stage; L2 is flushed (256 MB write) before each profiled
    forward.  The dominant kernel stage (largest share of the step among the
    stages that launch this library's kernels) is reported against its
    roofline; every stage is listed in the detail, the expert-parallel
    exchanges with their NVLink bytes per second."""
    import torch
    import gmoe
    hbm, tf, src = peaks()
    s = stream
    import numpy as np
    epr = E // world if ep else E
    if rank_of is None:
        rank_of = [e // epr for e in range(E)] if ep else [0] * E
    owner = np.asarray(rank_of)
    mine_idx = torch.tensor(np.nonzero(owner == (rank if ep else 0))[0], device="cuda")
    # routes into this GPU's experts and the distinct experts they reach, per
    # batch (with expert parallelism: over every rank's tokens)
    lg = torch.empty(gmoe.lib().gm_router_workspace_bytes(T) // 4, dtype=torch.float32, device="cuda")
    idx = torch.empty(T, TOPK, dtype=torch.int32, device="cuda")
    w = torch.empty(T, TOPK, dtype=torch.float32, device="cuda")
    rw = L["router_centered"] if fmt == "bq" else L["router_proj"]
    per_batch = []
    hist_sum = torch.zeros(E, dtype=torch.long, device="cuda")
    covered = torch.zeros((), dtype=torch.long, device="cuda")
    for x in xs:
        gmoe.call("gm_router_select", x, rw, L["router_scale"], L["per_expert_scale"], T, lg, idx, w, s)
        # tokens whose 8th/9th logit margin exceeds 1e-3 (the parity tests'
        # rule for a selection that must match the reference bit for bit)
        top9 = torch.topk(lg[:T * E].view(T, E), 9, dim=1).values
        covered += ((top9[:, 7] - top9[:, 8]) > 1e-3).sum()
        hist = torch.bincount(idx.reshape(-1).long(), minlength=E)
        if ep and dist is not None:
            dist.all_reduce(hist)
        hist_sum += hist
        mine = hist[mine_idx]
        per_batch.append((int((mine > 0).sum()), int(mine.sum())))
    torch.cuda.synchronize()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    n = max(5, min(steps, 50))
    blk.profile(True)
    for i in range(n):
        flush.zero_()
        blk.forward(0, xs[i % len(xs)], outs[i % len(xs)], T, s)
    torch.cuda.synchronize()
    stats, launches = blk.profile_read()
    blk.profile(False)
    mean_distinct = sum(per_batch[i % len(xs)][0] for i in range(n)) / n
    mean_R = sum(per_batch[i % len(xs)][1] for i in range(n)) / n
    step_ms = sum(v["avg_ms"] for v in stats.values())
    row_bytes = (H + 4 + 64) if fmt == "bq" else (2 * H + 64)
    stages = {}
    for label, v in stats.items():
        bound, amount = stage_model(label, fmt, T, mean_distinct, mean_R)
        sec = v["avg_ms"] / 1e3
        e = {"avg_us": round(v["avg_ms"] * 1e3, 2), "share": round(v["avg_ms"] / step_ms, 4),
             "kernels_per_call": v["kernels"] / max(v["calls"], 1)}
        if amount is not None:
            if bound == "tensor":
                e["tflops"] = round(amount / sec / 1e12, 1)
                e["frac"] = round(amount / sec / 1e12 / tf, 3)
            else:
                e["gbs"] = round(amount / sec / 1e9, 1)
                e["frac"] = round(amount / sec / 1e9 / hbm, 3)
        if label in ("ep_dispatch", "ep_combine") and world > 1:
            # bytes this GPU sends over NVLink (blocks of T rows to every peer)
            per_row = row_bytes if label == "ep_dispatch" else 2 * H
            e["nvlink_bytes_sent"] = (world - 1) * T * per_row
            e["nvlink_gbs"] = round((world - 1) * T * per_row / sec / 1e9, 1)
        stages[label] = e
    cand = [k for k in stats if stats[k]["kernels"] > 0 and stage_model(k, fmt, T, 1, 1)[1] is not None]
    top = max(cand, key=lambda k: stats[k]["avg_ms"])
    bound, amount = stage_model(top, fmt, T, mean_distinct, mean_R)
    sec = stats[top]["avg_ms"] / 1e3
    traffic = NCU_TRAFFIC.get((workload, top))
    detail = {"kernel": top, "avg_launch_us": stats[top]["avg_ms"] * 1e3, "launches_timed": n,
              "distinct_experts": mean_distinct, "routes_to_this_gpu": mean_R, "stages": stages,
              "kernels_per_forward": launches / n}
    if bound == "tensor":
        ach = amount / sec / 1e12
        detail.update({"flop_per_launch": amount, "peak_source": src + " (bf16 dense, burst)"})
        roof = {"bound": "tensor", "achieved": ach, "peak": tf, "unit": "TFLOP/s", "frac": ach / tf}
    else:
        ach = amount / sec / 1e9
        per_expert = {"bq_phase1_gate_up": BQ_EXPERT_GU_BYTES, "bq_phase2_down": BQ_EXPERT_DN_BYTES,
                      "phase1_gate_up": GU * H * 2, "phase2_down": H * I * 2}.get(top, 0)
        detail.update({"bytes_per_launch": amount, "bytes_per_expert": per_expert,
                       "peak_source": src + " (hbm copy)"})
        roof = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm}
    roof["traffic"] = traffic
    roof["detail"] = detail
    roof["weight_mb"] = mean_distinct * (BQ_EXPERT_BYTES if fmt == "bq" else BF16_EXPERT_BYTES) / 1e6
    # realised routing of the timed batches (all ranks' tokens with expert parallelism)
    h = (hist_sum.double() / len(xs)).cpu().numpy()
    tokens = T * (world if ep else 1)
    load = {"max_expert_share": round(float(h.max() / h.sum()), 4),
            "expert_routes_top8": [int(v) for v in h[:8]],
            "expert_routes_last4": [int(v) for v in h[-4:]],
            "top8_margin_above_1e-3": round(float(covered.item()) / (T * len(xs)), 4)}
    if ep and world > 1:
        load["routes_per_gpu"] = [int(h[owner == r].sum()) for r in range(world)]
    if workload in ZIPF:
        import synth
        load["zipf_target_top8"] = [int(round(v)) for v in synth.zipf_targets(tokens)[:8]]
    roof["routing"] = load
    return roof


if __name__ == "__main__":
    main()
