#!/usr/bin/env python
"""Benchmark of the reference's headline metric on B200:

    prefill+decode tok/s at B32/L1024 (27B hybrid, bf16); sum of call medians
    = (32*1024 + 32) tokens / (median prefill-call time + median decode-call time)

One step = one ``forward_step`` prefill of 32 requests x 1024 tokens into a fresh cache
(``new_cache(32, initial_capacity=64)``, so cache growth is inside the call, as in the
reference benchmark) followed by one decode ``forward_step`` of 32 tokens at 1024 prior
context. Weights: seeded N(0, 0.02) random init of the 27B geometry (54 GB, larger than
L2, streamed by every call). Token ids: the reference case ``batch_32_length_1024``
(uniform ids, seeds 26/27).

``value`` is device time (CUDA events around each call on the launching stream);
``e2e`` is wall time of the same public calls with the host token lists as input and the
logits read back to host memory. With N GPUs (torchrun) every rank runs its own B32/L1024
requests on its own replica (weak scaling, no collective on the data path); times are the
max over ranks. ``--impl reference`` times the CPU restatement of the reference
(oracle/) on a bounded sample of the same workload and extrapolates.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "prefill+decode tok/s at B32/L1024 (27B hybrid, bf16); sum of call medians"
UNIT = "tok/s"
# The reference GPU path's published number for this exact metric on one B200
# (results/shapes.csv: 1298.65 ms prefill + 35.26 ms decode at B32/L1024).
BASELINE_TOK_S = 24589.0
# results/shapes.csv:22-27, (batch, length) -> (prefill ms, decode ms): the same metric at
# the other shapes the reference publishes (configs[1] is B16 x L2048)
PUBLISHED_MS = {(16, 2048): (1292.67, 30.287), (32, 1024): (1298.65, 35.257), (64, 512): (1302.68, 44.580)}


def published_tok_s(B, L):
    p = PUBLISHED_MS.get((B, L))
    return None if p is None else (B * L + B) / ((p[0] + p[1]) * 1e-3)


EPI_NAMES = {0: "bf16", 1: "f32-of-bf16", 2: "SwiGLU"}


def _ncu_traffic(shape):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the GEMM of
    this shape, from the ncu summary committed for it (None when there is none)."""
    M, N, K, kind = shape
    path = os.path.join(ROOT, "profiles", f"gemm_{EPI_NAMES.get(kind, kind).lower()}_M{M}_N{N}_K{K}.md")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":")[1].strip().replace(",", ""))
    except OSError:
        pass
    return None


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        self.f.flush()
        rows = []
        with open(self.f.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


class HostReader:
    """Reads a call's result (the logits) into one page-locked host buffer that is allocated
    on first use (in the warm-up calls) and reused, so the device-to-host copy of every timed
    call runs at the rate of pinned memory instead of paying for a fresh pageable array."""

    def __init__(self):
        self.buf = None

    def __call__(self, t):
        import torch
        n = t.numel()
        if self.buf is None or self.buf.numel() < n or self.buf.dtype != t.dtype:
            self.buf = torch.empty(n, dtype=t.dtype, pin_memory=True)
        out = self.buf[:n].view(t.shape)
        out.copy_(t)
        return out


def make_inputs(V, B, L, rank):
    import torch
    g = torch.Generator().manual_seed(26 + 1000 * rank)
    ids = torch.randint(V, (B * L,), generator=g)
    prefill = [r.tolist() for r in ids.split([L] * B)]
    g = torch.Generator().manual_seed(27 + 1000 * rank)
    decode = [[t] for t in torch.randint(V, (B,), generator=g).tolist()]
    return prefill, decode


def reduce_step_times(rec, world, device):
    """This rank's median per-call times, then the maximum over ranks (a weak-scaling job
    is as slow as its slowest replica). Returns (step_ms, e2e_ms, prefill_ms, decode_ms)."""
    import torch
    import torch.distributed as dist
    med_p, med_d = statistics.median(rec["p"]), statistics.median(rec["d"])
    med_pw, med_dw = statistics.median(rec["p_wall"]), statistics.median(rec["d_wall"])
    t = torch.tensor([med_p + med_d, med_pw + med_dw, med_p, med_d], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return tuple(t.tolist())


# ------------------------------------------------------------------------- CPU baseline
def cpu_baseline(B=32, L=1024, sample_tokens=512, decode_ctx=128):
    """CPU restatement (oracle/) of the 27B step on a bounded sample: one GDN layer, one
    attention layer and one MLP at full 27B width for a prefill of 2 requests of
    sample_tokens/2 tokens and a decode of B requests at decode_ctx context, plus the
    lm_head; extrapolated by layer counts and (prefill) linearly in tokens."""
    import torch

    from oracle import ops as O
    from qwen38_inference_b200.config import qwen38_27b
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    c = qwen38_27b()
    g = torch.Generator().manual_seed(0)

    def W(*shape):
        return (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16).float()

    H = c.hidden_size
    gdn = dict(qkvz=W(c.qkvz_dim, H), ba=W(c.ba_dim, H), conv=W(c.conv_dim, 4), A_log=torch.zeros(48),
               dt_bias=W(48), norm=W(128) + 1, out=W(H, c.gdn_v_dim))
    att = dict(qkv=W(c.qkv_dim, H), out=W(H, c.attn_out_dim), q_norm=W(256), k_norm=W(256))
    mlp = dict(gate_up=W(2 * c.intermediate_size, H), down=W(H, c.intermediate_size))
    lm = W(c.vocab_size, H)
    rope = torch.randn(8192, 64)
    rnd = O.bf16

    def gdn_layer(x, n_req, decode):
        T = x.shape[0]
        qkvz = O.linear(x, gdn["qkvz"], rnd)
        ba = O.linear(x, gdn["ba"], rnd)
        st = torch.zeros(n_req, c.conv_dim, 3, dtype=torch.bfloat16)
        rec = torch.zeros(n_req, 48, 128, 128)
        gg, beta = O.gdn_gating(gdn["A_log"], ba[:, 48:], ba[:, :48], gdn["dt_bias"], rnd)
        if decode:
            mixed = O.conv_decode(qkvz[:, :c.conv_dim], gdn["conv"], st, list(range(n_req)), rnd)
        else:
            per = T // n_req
            mixed = O.conv_prefill(qkvz[:, :c.conv_dim], gdn["conv"], st, [i * per for i in range(n_req + 1)],
                                   list(range(n_req)), [False] * n_req, rnd)
        q = O.l2norm(mixed[:, :2048].reshape(T, 16, 128))
        k = O.l2norm(mixed[:, 2048:4096].reshape(T, 16, 128))
        v = mixed[:, 4096:].reshape(T, 48, 128)
        per = T // n_req
        o = torch.empty(T, 48, 128)
        for i in range(n_req):
            s = slice(i * per, (i + 1) * per)
            o[s], rec[i] = O.gdn_recurrence(q[s], k[s], v[s], gg[s], beta[s], rec[i], 128 ** -0.5, 3)
        y = O.gated_rmsnorm(rnd(o).reshape(-1, 128), gdn["norm"], qkvz[:, c.conv_dim:].reshape(-1, 128), 1e-6, rnd)
        return O.linear(y.reshape(T, -1), gdn["out"], rnd)

    def attn_layer(x, n_req, ctx):
        T = x.shape[0]
        proj = O.linear(x, att["qkv"], rnd)
        qg, k, v = proj.split([c.q_gate_dim, c.kv_dim, c.kv_dim], dim=-1)
        pos = torch.arange(T) % 4096
        q, k, gate = O.qk_norm_rope_gate(qg, k, att["q_norm"], att["k_norm"], rope, pos, 1e-6, 24, 4, 256, 64, rnd)
        per = T // n_req
        rows = n_req * (ctx + per) + 64
        kc = torch.zeros(rows, 4, 256, dtype=torch.bfloat16)
        vc = torch.zeros(rows, 4, 256, dtype=torch.bfloat16)
        starts = [64 + i * (ctx + per) for i in range(n_req)]
        loc = torch.tensor([starts[i] + ctx + j for i in range(n_req) for j in range(per)])
        kc[loc] = k.to(torch.bfloat16)
        vc[loc] = v.reshape(-1, 4, 256).to(torch.bfloat16)
        a = O.paged_attention(q, kc, vc, starts, [ctx] * n_req, [per] * n_req, 256 ** -0.5, rnd)
        out = O.sigmoid_mul(a.reshape(T, -1), gate.reshape(T, -1), rnd)
        return O.linear(out, att["out"], rnd)

    def mlp_layer(x):
        return O.linear(O.silu_mul(O.linear(x, mlp["gate_up"], rnd), rnd), mlp["down"], rnd)

    def timed(fn):
        t = time.perf_counter()
        fn()
        return time.perf_counter() - t

    x = torch.randn(sample_tokens, H).to(torch.bfloat16).float()
    tp = {"gdn": timed(lambda: gdn_layer(x, 2, False)), "attn": timed(lambda: attn_layer(x, 2, 0)),
          "mlp": timed(lambda: mlp_layer(x)), "lm": timed(lambda: O.linear(x[:2], lm, rnd))}
    xd = torch.randn(B, H).to(torch.bfloat16).float()
    td = {"gdn": timed(lambda: gdn_layer(xd, B, True)), "attn": timed(lambda: attn_layer(xd, B, decode_ctx)),
          "mlp": timed(lambda: mlp_layer(xd)), "lm": timed(lambda: O.linear(xd, lm, rnd))}
    scale = B * L / sample_tokens
    prefill_s = scale * (48 * tp["gdn"] + 16 * tp["attn"] + 64 * tp["mlp"]) + (B / 2) * tp["lm"]
    decode_s = 48 * td["gdn"] + 16 * td["attn"] + 64 * td["mlp"] + td["lm"]
    value = (B * L + B) / (prefill_s + decode_s)
    sample = (f"CPU restatement (oracle/, fp32 math with bf16 rounding points), extrapolated: one GDN, one "
              f"attention and one MLP layer at 27B width on a {sample_tokens}-token prefill (2 requests) and a "
              f"B{B} decode at {decode_ctx} context, plus lm_head; scaled by layer counts (48/16/64) and linearly "
              f"to {B}x{L} tokens; est. prefill {prefill_s:.1f} s + decode {decode_s:.2f} s")
    return {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
            "sample_seconds": sum(tp.values()) + sum(td.values())}


# ------------------------------------------------------------------------- GPU arm
def run_gpu(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    from qwen38_inference_b200 import Qwen38, ops
    from qwen38_inference_b200.config import qwen38_27b

    cfg = qwen38_27b()
    B, L = args.batch, args.length
    model = Qwen38(config=cfg, seed=0, device=f"cuda:{local}", max_context=max(8192, 2 * L))
    prefill, decode = make_inputs(cfg.vocab_size, B, L, rank)
    stream = torch.cuda.current_stream()
    read = HostReader()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def one_step(record):
        cache = model.new_cache(B, initial_capacity=64)
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        t0 = time.perf_counter()
        ev[0].record(stream)
        lg = model.forward_step(prefill, cache)
        t_issue_p = time.perf_counter()
        ev[1].record(stream)
        h2d = model._engine.last_h2d_bytes
        host_p = read(lg)
        t1 = time.perf_counter()
        t_dec = time.perf_counter()
        ev[2].record(stream)
        lg = model.forward_step(decode, cache)
        t_issue_d = time.perf_counter()
        ev[3].record(stream)
        h2d += model._engine.last_h2d_bytes
        host_d = read(lg)
        t2 = time.perf_counter()
        torch.cuda.synchronize()
        if record is not None:
            record["p"].append(ev[0].elapsed_time(ev[1]))
            record["d"].append(ev[2].elapsed_time(ev[3]))
            record["p_wall"].append((t1 - t0) * 1e3)
            record["d_wall"].append((t2 - t1) * 1e3)
            record["p_issue"].append((t_issue_p - t0) * 1e3)
            record["d_issue"].append((t_issue_d - t_dec) * 1e3)
        return h2d, host_p.numel() * 4 + host_d.numel() * 4
    for _ in range(args.warmup):
        one_step(None)
    rec = {"p": [], "d": [], "p_wall": [], "d_wall": [], "p_issue": [], "d_issue": []}
    ops.LAUNCHES[0] = 0
    barrier()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            h2d, d2h = one_step(rec)
        barrier()
    launches = ops.LAUNCHES[0] // max(1, args.steps)
    clocks = clk.summary()
    step_ms, e2e_ms, mp, md = reduce_step_times(rec, world, "cuda")
    tokens = world * (B * L + B)

    # ---- roofline of the dominant kernel (the tcgen05 GEMM): one instrumented prefill
    from qwen38_inference_b200 import _lib
    prof, per_op = [], []
    ops.PROFILE, _lib.PROFILE = prof, per_op
    cache = model.new_cache(B, initial_capacity=64)
    model.forward_step(prefill, cache)
    torch.cuda.synchronize()
    ops.PROFILE, _lib.PROFILE = None, None
    breakdown = {}
    for name, a, b in per_op:
        breakdown[name] = breakdown.get(name, 0.0) + a.elapsed_time(b)
    dec_ops = []
    _lib.PROFILE = dec_ops
    model._engine.use_graphs = False  # per-op events need the eager launch sequence
    model.forward_step(decode, cache)
    torch.cuda.synchronize()
    model._engine.use_graphs = True
    _lib.PROFILE = None
    dec_breakdown = {}
    for name, a, b in dec_ops:
        dec_breakdown[name] = dec_breakdown.get(name, 0.0) + a.elapsed_time(b)
    hbm, tf_burst, tf_sust, src = _peaks()
    # GEMM launches grouped by (M, N, K, epilogue); the group with the most device time is
    # the dominant kernel of the step (the MLP gate_up projection with the SwiGLU epilogue)
    groups = {}
    for f, a, b, shape in prof:
        g = groups.setdefault(shape, [0.0, 0.0, 0])
        g[0] += f
        g[1] += a.elapsed_time(b)
        g[2] += 1
    all_flops = sum(g[0] for g in groups.values())
    all_ms = sum(g[1] for g in groups.values())
    shape, (g_flops, g_ms, g_n) = max(groups.items(), key=lambda kv: kv[1][1])
    M_, N_, K_, kind = shape
    per_launch_ms = g_ms / g_n
    achieved = (g_flops / g_n) / (per_launch_ms * 1e-3) / 1e12
    traffic = _ncu_traffic(shape)
    roof = {"bound": "tensor",
            "kernel": f"gemm_tcgen05_kernel {EPI_NAMES.get(kind, kind)} M={M_} N={N_} K={K_}",
            "achieved": round(achieved, 1), "peak": tf_sust, "unit": "TFLOP/s",
            "frac": round(achieved / tf_sust, 4),
            "peak_source": f"{src} bf16_tflops_sustained (kernel timed inside a long step)",
            "flop_per_launch": g_flops / g_n, "launches_per_prefill": g_n, "avg_launch_ms": round(per_launch_ms, 4),
            "traffic": traffic, "algorithmic_bytes_per_launch": 2 * (M_ * K_ + N_ * K_ + M_ * (N_ // 2 if kind == 2 else N_)),
            "share_of_prefill": round(g_ms / mp, 4) if mp else None,
            "all_gemms": {"achieved": round(all_flops / (all_ms * 1e-3) / 1e12, 1), "launches": len(prof),
                          "share_of_prefill": round(all_ms / mp, 4) if mp else None}}
    pub = published_tok_s(B, L)
    metric = METRIC if (B, L) == (32, 1024) else METRIC.replace("B32/L1024", f"B{B}/L{L}")
    out = {"metric": metric, "value": round(tokens / (step_ms * 1e-3), 1), "unit": UNIT, "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": round(tokens / (step_ms * 1e-3) / pub, 4) if pub else None,
           "dtype": "bf16", "data": "synthetic (random-init N(0,0.02) 27B weights; uniform token ids, reference case seeds 26/27)",
           "config": {"workload": f"B{B}xL{L} prefill into a fresh cache + B{B} decode at {L} context, 27B hybrid",
                      "model": "Qwen3.8-27B hybrid geometry (48 GDN + 16 gated GQA), random init",
                      "global_batch": world * B, "seq_len": L, "parallelism": f"replicas x{world} (requests sharded)",
                      "l2": "inputs larger than L2 (54 GB of weights streamed per call)"},
           "median_ms": {"prefill": round(mp, 3), "decode": round(md, 3),
                         "prefill_host_issue": round(statistics.median(rec["p_issue"]), 3),
                         "decode_host_issue": round(statistics.median(rec["d_issue"]), 3)},
           "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h},
           "gpu_launches": launches, "clocks": clocks, "roofline": roof,
           "op_ms": {"prefill": {k[3:]: round(v, 2) for k, v in sorted(breakdown.items(), key=lambda x: -x[1])},
                     "decode": {k[3:]: round(v, 3) for k, v in sorted(dec_breakdown.items(), key=lambda x: -x[1])}}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(B, L)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _rank_weight_bytes(model):
    """Bytes of this rank's weights that a decode step streams (every linear layer and the
    lm_head; the embedding is a row gather)."""
    seen, total = set(), 0
    for w in model.layers:
        for k, t in w.items():
            if k in ("qkvz", "ba"):  # views into qkvzba
                continue
            if t.data_ptr() not in seen:
                seen.add(t.data_ptr())
                total += t.numel() * t.element_size()
    return total + model.final_norm.numel() * 2 + model.lm_head.numel() * 2


def run_long(args):
    """One long request with head-wise tensor parallelism over the N GPUs (torchrun): a
    B1 prompt of ``--long-tokens`` tokens fed in ``--chunk``-token forward_step calls into a
    fresh cache, then decode steps at that context (the reference configuration "B1 prefill
    of 131071 tokens in 512-token chunks, then decode"). One step = the whole chunked prefill
    plus ``--decode-steps`` decodes (the first two set up the decode graph and are untimed).
    Warm-up steps run the first 8 chunks only. Times are per-call CUDA events summed over the
    chunks, max over ranks (strong scaling: the same request whatever N)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    from qwen38_inference_b200 import Qwen38, ops
    from qwen38_inference_b200.config import qwen38_27b

    cfg = qwen38_27b()
    n_tok, chunk = args.long_tokens, args.chunk
    n_dec = max(3, args.decode_steps)
    model = Qwen38(config=cfg, seed=0, device=f"cuda:{local}", max_context=n_tok + n_dec + 2 * chunk + 64,
                   tensor_parallel=True if world > 1 else None)
    if world > 1 and args.tp_allreduce == "peer":
        model.enable_peer_allreduce()
    g = torch.Generator().manual_seed(26)
    prompt = torch.randint(cfg.vocab_size, (n_tok,), generator=g).tolist()  # same tokens on every rank
    g = torch.Generator().manual_seed(27)
    dec_tokens = torch.randint(cfg.vocab_size, (n_dec,), generator=g).tolist()
    chunks = [prompt[i:i + chunk] for i in range(0, n_tok, chunk)]
    stream = torch.cuda.current_stream()
    read = HostReader()

    def one_step(n_chunks, rec):
        cache = model.new_cache(1, initial_capacity=64)
        pf, pw, dd, dw = [], [], [], []
        h2d = d2h = 0
        torch.cuda.synchronize()
        for c in chunks[:n_chunks]:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            e0.record(stream)
            lg = model.forward_step([c], cache)
            e1.record(stream)
            h2d += model._engine.last_h2d_bytes
            host = read(lg)
            pw.append((time.perf_counter() - t0) * 1e3)
            d2h += host.numel() * 4
            pf.append((e0, e1))
        for i, t in enumerate(dec_tokens):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            e0.record(stream)
            lg = model.forward_step([[t]], cache)
            e1.record(stream)
            host = read(lg)
            if i >= 2:  # graph set-up calls are untimed
                dw.append((time.perf_counter() - t0) * 1e3)
                dd.append((e0, e1))
        torch.cuda.synchronize()
        if rec is not None:
            rec["p"].append(sum(a.elapsed_time(b) for a, b in pf))
            rec["p_wall"].append(sum(pw))
            rec["d"].append(statistics.median(a.elapsed_time(b) for a, b in dd))
            rec["d_wall"].append(statistics.median(dw))
            rec["io"] = (h2d, d2h)
        return cache

    for _ in range(args.warmup):
        one_step(min(8, len(chunks)), None)
    rec = {"p": [], "d": [], "p_wall": [], "d_wall": []}
    ops.LAUNCHES[0] = 0
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            cache = one_step(len(chunks), rec)
        torch.cuda.synchronize()
    launches = ops.LAUNCHES[0] // max(1, args.steps)
    step_ms, e2e_ms, mp, md = reduce_step_times(rec, world, "cuda")
    # per-op device time of one more chunk and one more decode at the full context, eager
    from qwen38_inference_b200 import _lib
    op_ms = {}
    model._engine.use_graphs = False
    for name, toks in (("chunk", [chunks[0]]), ("decode", [[dec_tokens[0]]])):
        prof = []
        _lib.PROFILE = prof
        model.forward_step(toks, cache)
        torch.cuda.synchronize()
        _lib.PROFILE = None
        agg = {}
        for n, a, b in prof:
            agg[n[3:]] = agg.get(n[3:], 0.0) + a.elapsed_time(b)
        op_ms[name] = {k: round(v, 3) for k, v in sorted(agg.items(), key=lambda kv: -kv[1])}
    model._engine.use_graphs = True
    # decode roofline (HBM): this rank's weights + its KV heads over the context + its GDN
    # states (read and written), per decode step
    c = model.cfg
    ctx = n_tok + n_dec
    kv_bytes = sum(1 for k in model.layer_types if k == "full_attention") * 2 * c.num_key_value_heads * c.head_dim * 2 * ctx
    st_bytes = sum(1 for k in model.layer_types if k != "full_attention") * c.linear_num_value_heads * \
        c.linear_value_head_dim * c.linear_key_head_dim * 4 * 2
    dec_bytes = _rank_weight_bytes(model) + kv_bytes + st_bytes
    hbm, _, _, src = _peaks()
    achieved = dec_bytes / (md * 1e-3) / 1e9
    h2d, d2h = rec["io"]
    out = {"metric": f"B1 long-context chunked prefill tok/s ({n_tok} tokens in {chunk}-token calls), 27B hybrid, "
                     f"head-wise tensor parallel", "value": round(n_tok / (mp * 1e-3), 1), "unit": UNIT,
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (random-init N(0,0.02) 27B weights; uniform token ids, seeds 26/27)",
           "config": {"workload": f"B1 x {n_tok} tokens in {chunk}-token chunks into a fresh cache, then decode at "
                                  f"{n_tok} context", "global_batch": 1, "seq_len": n_tok,
                      "parallelism": (f"tp{world} (head-wise; fp32 all-reduce after each row-parallel projection: "
                                      + ("NCCL in prefill, in the projection kernel over peer memory in decode)"
                                         if args.tp_allreduce == "peer" else "NCCL)")) if world > 1 else "single GPU",
                      "warmup_steps": "first 8 chunks + decodes", "l2": "inputs larger than L2 (weights streamed per call)"},
           "median_ms": {"prefill_total": round(mp, 2), "decode": round(md, 3)},
           "reference_published": {"prefill_ms_one_131072_token_call": 7753.7, "decode_ms_at_131k": 15.79},
           "e2e": {"value": round(n_tok / (statistics.median(rec["p_wall"]) * 1e-3), 1), "unit": UNIT,
                   "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                   "decode_ms": round(statistics.median(rec["d_wall"]), 3)},
           "gpu_launches": launches, "clocks": clk.summary(), "op_ms_at_full_context": op_ms,
           "roofline": {"bound": "hbm", "kernel": "decode step at the long context (all kernels of one step)",
                        "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                        "peak_source": f"{src} hbm_gbs", "bytes_per_rank_step": dec_bytes, "traffic": None}}
    if rank == 0:
        print(json.dumps(out), flush=True)
    del cache
    model.close()  # graphs holding NCCL calls and the peer buffers go before the process group
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _dist_setup(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    return world, rank, local


def _max_over_ranks(vals, world):
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run_continuous(args):
    """configs[2], continuous batching on the 27B model: 32 requests with prompt lengths
    uniform in [512, 1536] prefilled in one ragged call into a fresh cache, then 64 decode
    steps; before every 8th step 4 requests (slots 4j..4j+3 at the j-th refill) are reset and
    refilled with new prompts of uniform random length, in the same call as the other 28
    requests' decode tokens (a mixed call, which the reference runs as prefill, REF:5027).
    Exercises cache growth and slot reuse. One step = that whole sequence; ``value`` = tokens
    consumed / device time (CUDA events per call, summed), max over ranks (each rank its own
    replica and requests)."""
    import torch
    import torch.distributed as dist
    world, rank, local = _dist_setup(args)
    from qwen38_inference_b200 import Qwen38, ops
    from qwen38_inference_b200.config import qwen38_27b
    cfg = qwen38_27b()
    B, V = 32, cfg.vocab_size
    model = Qwen38(config=cfg, seed=0, device=f"cuda:{local}", max_context=8192)
    g = torch.Generator().manual_seed(26 + 1000 * rank)
    plan = [("prefill", [torch.randint(V, (int(n),), generator=g).tolist()
                         for n in torch.randint(512, 1537, (B,), generator=g)], None)]
    for step in range(64):
        if step % 8 == 7:
            j = step // 8
            slots = list(range(4 * j, 4 * j + 4))
            rows = [torch.randint(V, (int(torch.randint(512, 1537, (1,), generator=g)),), generator=g).tolist()
                    if s in slots else [int(torch.randint(V, (1,), generator=g))] for s in range(B)]
            plan.append(("mixed", rows, slots))
        else:
            plan.append(("decode", [[int(t)] for t in torch.randint(V, (B,), generator=g)], None))
    stream = torch.cuda.current_stream()
    read = HostReader()

    def one_run(rec):
        cache = model.new_cache(B, initial_capacity=64)
        evs, tok, wall = [], 0, 0.0
        h2d = d2h = 0
        torch.cuda.synchronize()
        for kind, rows, reset in plan:
            if reset:
                cache.reset(reset)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            e0.record(stream)
            lg = model.forward_step(rows, cache)
            e1.record(stream)
            h2d += model._engine.last_h2d_bytes
            host = read(lg)
            wall += time.perf_counter() - t0
            d2h += host.numel() * 4
            evs.append((kind, e0, e1))
            tok += sum(len(r) for r in rows)
        torch.cuda.synchronize()
        if rec is not None:
            ms = {k: [a.elapsed_time(b) for kk, a, b in evs if kk == k] for k in ("prefill", "decode", "mixed")}
            rec.append((sum(sum(v) for v in ms.values()), wall * 1e3, ms, tok, h2d, d2h))

    for _ in range(args.warmup):
        one_run(None)
    rec = []
    ops.LAUNCHES[0] = 0
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            one_run(rec)
    launches = ops.LAUNCHES[0] // max(1, args.steps)
    dev_ms = statistics.median(r[0] for r in rec)
    wall_ms = statistics.median(r[1] for r in rec)
    dev_ms, wall_ms = _max_over_ranks([dev_ms, wall_ms], world)
    ms, tok, h2d, d2h = rec[-1][2], rec[-1][3], rec[-1][4], rec[-1][5]
    out = {"metric": "continuous-batching tok/s (27B hybrid, bf16; B32, prompts U[512,1536], 64 decode steps, "
                     "4 slots refilled every 8 steps)", "value": round(world * tok / (dev_ms * 1e-3), 1),
           "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (random-init N(0,0.02) 27B weights; uniform token ids and prompt lengths, seed 26)",
           "config": {"workload": "configs[2]: ragged B32 prefill, 56 decode calls and 8 mixed refill calls into "
                                  "one cache", "global_batch": world * B, "seq_len": "512-1536",
                      "parallelism": f"replicas x{world} (requests sharded)",
                      "l2": "inputs larger than L2 (54 GB of weights streamed per call)"},
           "tokens_per_step_per_rank": tok,
           "median_ms": {"prefill_call": round(ms["prefill"][0], 3), "decode_call": round(statistics.median(ms["decode"]), 3),
                         "mixed_call": round(statistics.median(ms["mixed"]), 3)},
           "e2e": {"value": round(world * tok / (wall_ms * 1e-3), 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h},
           "gpu_launches": launches, "clocks": clk.summary()}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_split(args):
    """configs[4], throughput half: decode of B64 requests at 512 tokens of context with the
    requests split across the N GPUs of the job (B64/N per replica; strong scaling: the same
    64 requests whatever N). One step = a prefill of each rank's requests (512 tokens each)
    into a fresh cache, then ``--decode-steps`` decode calls (the first two set up the decode
    graph, untimed). ``value`` = 64 / (median decode call, max over ranks) tokens per second;
    the prefill is reported beside it. No collective on the data path."""
    import torch
    import torch.distributed as dist
    world, rank, local = _dist_setup(args)
    from qwen38_inference_b200 import Qwen38, ops
    from qwen38_inference_b200.config import qwen38_27b
    cfg = qwen38_27b()
    B_all, L = 64, 512
    if B_all % world:
        raise SystemExit("the 64 requests must split evenly over the GPUs")
    B = B_all // world
    n_dec = max(3, args.decode_steps)
    model = Qwen38(config=cfg, seed=0, device=f"cuda:{local}", max_context=8192)
    g = torch.Generator().manual_seed(26)
    ids = torch.randint(cfg.vocab_size, (B_all, L), generator=g)
    prompts = [r.tolist() for r in ids[rank * B:(rank + 1) * B]]
    g = torch.Generator().manual_seed(27)
    dec = torch.randint(cfg.vocab_size, (n_dec, B_all), generator=g)[:, rank * B:(rank + 1) * B].tolist()
    stream = torch.cuda.current_stream()
    read = HostReader()

    rec_io = [0]

    def one_step(rec):
        cache = model.new_cache(B, initial_capacity=64)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        lg = model.forward_step(prompts, cache)
        e1.record(stream)
        read(lg)
        dd, dw = [], []
        for i, t in enumerate(dec):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            a.record(stream)
            lg = model.forward_step([[x] for x in t], cache)
            b.record(stream)
            read(lg)  # the device-timed region ends before the copy; the wall time includes it
            rec_io[0] = model._engine.last_h2d_bytes
            if i >= 2:
                dw.append((time.perf_counter() - t0) * 1e3)
                dd.append((a, b))
        torch.cuda.synchronize()
        if rec is not None:
            rec["p"].append(e0.elapsed_time(e1))
            rec["d"].append(statistics.median(a.elapsed_time(b) for a, b in dd))
            rec["d_wall"].append(statistics.median(dw))

    for _ in range(args.warmup):
        one_step(None)
    rec = {"p": [], "d": [], "d_wall": []}
    ops.LAUNCHES[0] = 0
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            one_step(rec)
    launches = ops.LAUNCHES[0] // max(1, args.steps)
    mp, md, mdw = _max_over_ranks([statistics.median(rec["p"]), statistics.median(rec["d"]),
                                   statistics.median(rec["d_wall"])], world)
    pub = PUBLISHED_MS[(64, 512)][1]
    out = {"metric": "decode tok/s at B64/L512 (27B hybrid, bf16), requests split across GPUs",
           "value": round(B_all / (md * 1e-3), 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(md, 3), "higher_is_better": True, "scaling": "strong",
           "vs_baseline": round(pub / md, 4) if world == 1 else None, "dtype": "bf16",
           "data": "synthetic (random-init N(0,0.02) 27B weights; uniform token ids, seeds 26/27)",
           "config": {"workload": f"configs[4]: B64 x L512 split {B} requests per GPU; prefill, then decode at 512",
                      "global_batch": B_all, "seq_len": L, "parallelism": f"replicas x{world} (requests split)",
                      "l2": "inputs larger than L2 (54 GB of weights streamed per call)"},
           "median_ms": {"prefill_per_rank": round(mp, 3), "decode": round(md, 3)},
           "reference_published_ms": {"prefill_b64_l512": PUBLISHED_MS[(64, 512)][0], "decode_b64_l512": pub},
           "e2e": {"value": round(B_all / (mdw * 1e-3), 1), "unit": UNIT, "per": "decode call",
                   "h2d_bytes_per_step": rec_io[0], "d2h_bytes_per_step": 4 * B * cfg.vocab_size},
           "gpu_launches": launches, "clocks": clk.summary()}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_step_cublas(args):
    """Comparator (not the product path): the B32 x L1024 prefill of the headline step with
    every projection done by cuBLAS through torch (plain bf16 GEMMs; the SwiGLU, the logits'
    fp32 widening, the add-norms and q/k norm + RoPE + KV store then run as separate steps,
    the last two as this library's kernels), alternated call by call with the product's own
    prefill on the same model, inputs and box, so both see the same power-capped clocks.
    Prints both medians (CUDA events) and the clocks seen."""
    import torch
    import torch.nn.functional as F
    from qwen38_inference_b200 import Qwen38, ops
    from qwen38_inference_b200.config import qwen38_27b
    cfg = qwen38_27b()
    B, L = args.batch, args.length
    model = Qwen38(config=cfg, seed=0, device="cuda:0", max_context=max(8192, 2 * L))
    prefill, _ = make_inputs(cfg.vocab_size, B, L, 0)
    own = {k: getattr(ops, k) for k in ("gemm", "gemm_qkv_rope_store", "gemm_add_rmsnorm")}

    def lib_gemm(x, w, out=None, *, out_kind=ops.OUT_BF16, ws=None):
        y = torch.matmul(x, w.t())
        if out_kind == ops.OUT_SWIGLU:
            if fused_silu is not None:
                r = torch.empty(y.shape[0], y.shape[1] // 2, dtype=y.dtype, device=y.device)
                fused_silu(r, y)
            else:
                g, u = y.chunk(2, dim=-1)
                r = F.silu(g) * u
        elif out_kind in (ops.OUT_F32_OF_BF16, ops.OUT_F32):
            r = y.float()
        else:
            r = y
        if out is None:
            return r
        out.copy_(r)
        return out

    def lib_qkv(x, w, qkv, nq, nkv, d, q_w, k_w, rope, positions, locations, kc, vc, eps, ws):
        qkv.copy_(torch.matmul(x, w.t()))
        ops.qk_norm_rope_store(qkv, nq, nkv, d, q_w, k_w, rope, positions, locations, kc, vc, eps)
        return qkv

    def lib_add_norm(x, w, resid, norm_w, hidden, eps, ws):
        hidden.copy_(torch.matmul(x, w.t()))
        ops.add_rmsnorm(hidden, resid, norm_w, eps)

    lib = {"gemm": lib_gemm, "gemm_qkv_rope_store": lib_qkv, "gemm_add_rmsnorm": lib_add_norm}
    swiglu_kind = "torch bf16 elementwise"
    try:  # a fused silu-and-mul kernel, as the reference's stack has (sgl_kernel); vllm's if importable
        import vllm._C  # noqa: F401
        fused_silu = torch.ops._C.silu_and_mul
        swiglu_kind = "vllm silu_and_mul (one fused kernel)"
    except Exception:
        fused_silu = None
    stream = torch.cuda.current_stream()

    def one(which):
        for k, v in (lib if which == "cublas" else own).items():
            setattr(ops, k, v)
        cache = model.new_cache(B, initial_capacity=64)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        model.forward_step(prefill, cache)
        e1.record(stream)
        torch.cuda.synchronize()
        for k, v in own.items():
            setattr(ops, k, v)
        return e0.elapsed_time(e1)

    for _ in range(args.warmup):
        one("ours")
        one("cublas")
    t = {"ours": [], "cublas": []}
    with ClockSampler(0) as clk:
        for _ in range(args.steps):
            for which in ("ours", "cublas"):
                t[which].append(one(which))
    mo, mc = statistics.median(t["ours"]), statistics.median(t["cublas"])
    print(json.dumps({"op": "step_cublas", "batch": B, "length": L, "prefill_ms": {"ours": round(mo, 2),
                      "cublas_gemms": round(mc, 2)}, "ratio_cublas_over_ours": round(mc / mo, 4),
                      "samples": {k: [round(x, 1) for x in v] for k, v in t.items()}, "swiglu": swiglu_kind,
                      "clocks": clk.summary()}),
          flush=True)


def run_decode_step(args):
    """The B32 decode step at 1024 tokens of context alone, for a launch list: three rounds of
    prefill + decode on fresh caches (which the buffer arena places at the same addresses,
    so the decodes run eagerly, then capture, then replay the decode graph), a fourth
    prefill, and its decode from the graph bracketed by the CUDA profiler API, so that
    ``ncu --profile-from-start off`` captures exactly that call's kernels. ``--layers N``
    builds the 27B geometry with N layers (every layer's kernels keep their 27B shapes; the
    small-footprint case for counter captures)."""
    import dataclasses

    import torch
    from qwen38_inference_b200 import Qwen38
    from qwen38_inference_b200.config import qwen38_27b

    cfg = qwen38_27b()
    if args.layers:
        cfg = dataclasses.replace(cfg, num_hidden_layers=args.layers)
    B, L = args.batch, args.length
    model = Qwen38(config=cfg, seed=0, device="cuda:0", max_context=max(8192, 2 * L))
    prefill, decode = make_inputs(cfg.vocab_size, B, L, 0)
    for _ in range(3):
        cache = model.new_cache(B, initial_capacity=64)
        model.forward_step(prefill, cache)
        model.forward_step(decode, cache)
        del cache
    cache = model.new_cache(B, initial_capacity=64)
    model.forward_step(prefill, cache)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.cudart().cudaProfilerStart()
    e0.record()
    model.forward_step(decode, cache)
    e1.record()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"op": "decode_step", "batch": B, "context": L, "ms": round(e0.elapsed_time(e1), 3),
                      "graph_replays": model._engine.replays}), flush=True)


def run_op(args):
    """One kernel of the step alone, at the step's shape, on random data: the case the ncu
    captures under profiles/ run (``--op gate_up``: the MLP gate_up GEMM with the SwiGLU
    epilogue, M = batch*length tokens; ``--op gdn_prefill``: the chunked delta rule with
    the fused gated RMSNorm over batch requests of length tokens, 27B head geometry)."""
    import torch
    from qwen38_inference_b200 import ops
    from qwen38_inference_b200.config import qwen38_27b

    cfg = qwen38_27b()
    B, L = args.batch, args.length
    T = B * L
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    if args.op == "gate_up":
        x = torch.randn(T, cfg.hidden_size, device=dev, generator=g).bfloat16()
        w = (torch.randn(2 * cfg.intermediate_size, cfg.hidden_size, device=dev, generator=g) * 0.02).bfloat16()
        y = torch.empty(T, cfg.intermediate_size, device=dev, dtype=torch.bfloat16)
        work = 2.0 * T * w.shape[0] * cfg.hidden_size
        unit = "TFLOP/s"

        def launch():
            ops.gemm(x, w, y, out_kind=ops.OUT_SWIGLU)
    elif args.op in ("qkvz_proj", "down_proj"):
        # the GDN input projection (CTA-pair kernel) and the MLP down projection (256-row
        # tiles) of the prefill, bf16 output
        N, K = (cfg.qkvz_dim + cfg.ba_dim, cfg.hidden_size) if args.op == "qkvz_proj" else \
            (cfg.hidden_size, cfg.intermediate_size)
        x = torch.randn(T, K, device=dev, generator=g).bfloat16()
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
        y = torch.empty(T, N, device=dev, dtype=torch.bfloat16)
        work = 2.0 * T * N * K
        unit = "TFLOP/s"

        def launch():
            ops.gemm(x, w, y)
    elif args.op == "conv_prefill":
        C = cfg.conv_dim
        x = torch.randn(T, cfg.qkvz_dim, device=dev, generator=g).bfloat16()
        w = (torch.randn(C, cfg.linear_conv_kernel_dim, device=dev, generator=g) * 0.5).bfloat16()
        cs = torch.zeros(B, C, cfg.linear_conv_kernel_dim - 1, device=dev).bfloat16()
        cu = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
        slots = torch.arange(B, dtype=torch.int32, device=dev)
        has = torch.zeros(B, dtype=torch.int32, device=dev)
        qo = torch.empty(T, cfg.gdn_qk_dim, device=dev).bfloat16()
        ko = torch.empty_like(qo)
        vo = torch.empty(T, cfg.gdn_v_dim, device=dev).bfloat16()
        work = 2.0 * T * C * 2  # read the conv channels of x, write q, k, v
        unit = "GB/s"

        def launch():
            ops.conv_prefill(x, w, cs, cu, slots, has, B, L, qo, ko, vo, cfg.gdn_qk_dim, cfg.gdn_v_dim,
                             cfg.linear_key_head_dim)
    elif args.op == "attn_prefill":
        from qwen38_inference_b200.model import build_metadata
        nq, nkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        cap = L
        kc = torch.randn(B * cap + 64, nkv, d, device=dev, generator=g).bfloat16()
        vc = torch.randn(B * cap + 64, nkv, d, device=dev, generator=g).bfloat16()
        qkv = torch.randn(T, cfg.qkv_dim, device=dev, generator=g).bfloat16()
        packed, offs, _ = build_metadata(list(range(B)), [0] * B, [L] * B, cap)
        md = {k_: torch.from_numpy(packed[o:o + n]).to(dev) for k_, (o, n) in offs.items()}
        out = torch.empty(T, nq * d, device=dev).bfloat16()
        work = 2.0 * 2 * B * (L * (L + 1) / 2) * d * nq  # causal QK^T and PV
        unit = "TFLOP/s"

        def launch():
            ops.attn_prefill(qkv, nq, nkv, d, kc, vc, md["tiles"], md["cu"], md["prefix"], md["kv_base"], out,
                             d ** -0.5)
    elif args.op == "gdn_decode":
        launch, work, unit, extra = _gdn_decode_case(cfg, B, g)
    elif args.op == "gdn_prefill_flashinfer":
        launch, work, unit, extra = _gdn_prefill_case(cfg, B, L, g, flashinfer=True)
    else:
        launch, work, unit, extra = _gdn_prefill_case(cfg, B, L, g)
    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    for i in range(args.steps):
        ev[2 * i].record()
        launch()
        ev[2 * i + 1].record()
    torch.cuda.synchronize()
    ms = statistics.median(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps))
    rate = work / (ms * 1e-3) / (1e12 if unit == "TFLOP/s" else 1e9)
    line = {"op": args.op, "batch": B, "length": L, "median_ms": round(ms, 4), "achieved": round(rate, 1),
            "unit": unit, "work_per_launch": work}
    hbm, tf_burst, _, src = _peaks()
    line["frac_of_peak"] = round(rate / (hbm if unit == "GB/s" else tf_burst), 4)
    line["peak_source"] = f"{src} {'hbm_gbs' if unit == 'GB/s' else 'bf16_tflops (burst: kernel timed alone)'}"
    if "extra" in locals():
        line.update(extra)
    print(json.dumps(line), flush=True)
    return line


class Unavailable(Exception):
    """A library comparator that cannot run on this box (the reason goes into the JSON line)."""


def _gdn_gating_inputs(T, HV, dev, g):
    """configs[3] gating: g = -softplus(N(0,1)), beta = sigmoid(N(0,1)). The kernels compute
    g = -exp(A_log) softplus(a + dt_bias) and beta = sigmoid(b) from the projection's b and a
    columns (REF:1274-1289), so A_log = 0 and dt_bias = 0 with a, b ~ N(0,1) give exactly
    those distributions."""
    import torch
    ba = torch.randn(T, 2 * HV, device=dev, generator=g).bfloat16()  # [b | a]
    A_log = torch.zeros(HV, device=dev)
    dt_bias = torch.zeros(HV, device=dev).bfloat16()
    return ba, A_log, dt_bias


def _gdn_prefill_case(cfg, B, L, g, flashinfer=False):
    """The chunked delta rule with the fused gating and gated RMSNorm over B requests of L
    tokens, 27B head geometry, configs[3] inputs: q and k L2-normalised, v ~ N(0,1), the
    gating above, zero initial state (a fresh prefill). ``flashinfer``: the same recurrence
    through flashinfer's sm100 chunked kernel (the reference's REF:5084 kernel), given
    alpha = exp(g) and beta in fp32 like the reference passes them; it computes o only
    (no gating, no norm), so its algorithmic bytes omit z, y and ba and count o."""
    import torch
    from qwen38_inference_b200 import ops
    dev = "cuda"
    T = B * L
    H, HV, dk, dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, \
        cfg.linear_value_head_dim
    nrm = torch.nn.functional.normalize
    q = nrm(torch.randn(T, H, dk, device=dev, generator=g), dim=-1).bfloat16().view(T, H * dk)
    k = nrm(torch.randn(T, H, dk, device=dev, generator=g), dim=-1).bfloat16().view(T, H * dk)
    v = torch.randn(T, HV * dv, device=dev, generator=g).bfloat16()
    ba, A_log, dt_bias = _gdn_gating_inputs(T, HV, dev, g)
    a = ba[:, HV:].float()
    gg = -torch.nn.functional.softplus(a)
    extra = {"gating": "g = -softplus(a), a ~ N(0,1) (A_log = 0, dt_bias = 0); beta = sigmoid(b), b ~ N(0,1)",
             "g_mean": round(float(gg.mean()), 4), "beta_mean": round(float(torch.sigmoid(ba[:, :HV].float()).mean()), 4)}
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
    state = torch.zeros(B, HV, dv, dk, device=dev)
    if flashinfer:
        try:
            from flashinfer.gdn_kernels import chunk_gated_delta_rule_sm100
        except Exception as e:
            raise Unavailable(f"flashinfer sm100 chunked GDN not importable: {type(e).__name__}: {e}") from None
        alpha = torch.exp(gg).contiguous()
        beta = torch.sigmoid(ba[:, :HV].float()).bfloat16().float().contiguous()
        o = torch.empty(T, HV, dv, device=dev, dtype=torch.bfloat16)
        out_state = torch.empty(B, HV, dv, dk, device=dev)
        q3, k3, v3 = q.view(T, H, dk), k.view(T, H, dk), v.view(T, HV, dv)
        extra["kernel"] = "flashinfer chunk_gated_delta_rule_sm100 (CuTe DSL), o only"
        work = 2.0 * T * (2 * H * dk + HV * dv) + 4.0 * T * HV * 2 + 2.0 * T * HV * dv + 2.0 * B * HV * dv * dk * 4

        def launch():
            chunk_gated_delta_rule_sm100(q3, k3, v3, alpha, beta, o, cu, state, out_state, dk ** -0.5)
        try:
            launch()  # the CuTe DSL kernel compiles at its first call
            torch.cuda.synchronize()
        except Exception as e:
            msg = str(e).strip().splitlines()
            raise Unavailable(f"flashinfer chunk_gated_delta_rule_sm100 failed at its first call: {type(e).__name__}: "
                              f"{msg[0][:200] if msg else ''}") from None
        return launch, work, "GB/s", extra
    z = torch.randn(T, HV * dv, device=dev, generator=g).bfloat16()
    nw = torch.ones(dv, device=dev).bfloat16()
    y = torch.empty(T, HV * dv, device=dev, dtype=torch.bfloat16)
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    # algorithmic bytes: q, k, v, z, ba read once, y written once, state read + written
    work = 2.0 * T * (2 * H * dk + 2 * HV * dv + 2 * HV) + 2.0 * T * HV * dv + 2.0 * B * HV * dv * dk * 4
    extra["flop_per_launch"] = (8 * dk * dv + 10 * 64 * dv) * T * HV  # (8 d^2 + 10 C d) FLOP per token and value head
    extra["kernel"] = "qw gdn_prefill_kernel (chunked delta rule + gating + gated RMSNorm)"

    def launch():
        ops.gdn_prefill(q, k, v, ba, A_log, dt_bias, cu, slots, B, state, z, nw, y, H, HV, dk, dv, dk ** -0.5,
                        cfg.rms_norm_eps)
    return launch, work, "GB/s", extra


def _gdn_decode_case(cfg, B, g):
    """The fused decode step of B requests (conv update, L2 norm of q and k, gating, one
    recurrent step of the fp32 state, gated RMSNorm), 27B head geometry, configs[3] inputs
    (projection rows ~ N(0,1), the gating above, a state of a previous prefill ~ N(0, 0.05)).
    Algorithmic bytes: the state read and written, the conv state read and written, the
    projection row and ba read, y written."""
    import torch
    from qwen38_inference_b200 import ops
    dev = "cuda"
    H, HV, dk, dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, \
        cfg.linear_value_head_dim
    C = cfg.conv_dim
    qkvz = torch.randn(B, cfg.qkvz_dim, device=dev, generator=g).bfloat16()
    ba, A_log, dt_bias = _gdn_gating_inputs(B, HV, dev, g)
    conv_w = (torch.randn(C, 4, device=dev, generator=g) * 0.5).bfloat16()
    conv_state = torch.randn(B, C, 3, device=dev, generator=g).bfloat16()
    state = torch.randn(B, HV, dv, dk, device=dev, generator=g) * 0.05
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    nw = torch.ones(dv, device=dev).bfloat16()
    y = torch.empty(B, HV * dv, device=dev, dtype=torch.bfloat16)
    work = 2.0 * B * HV * dv * dk * 4 + 2.0 * B * C * 3 * 2 + 2.0 * B * (cfg.qkvz_dim + 2 * HV) + 2.0 * B * HV * dv
    extra = {"gating": "g = -softplus(a), a ~ N(0,1) (A_log = 0, dt_bias = 0); beta = sigmoid(b), b ~ N(0,1)",
             "kernel": "qw gdn_decode_kernel (conv + L2 norm + gating + recurrent step + gated RMSNorm)"}

    def launch():
        ops.gdn_decode(qkvz, ba, conv_w, conv_state, state, slots, B, A_log, dt_bias, nw, y, H, HV, dk, dv,
                       cfg.rms_norm_eps)
    return launch, work, "GB/s", extra


def run_gdn_sweep(args):
    """the gated-delta-rule op sweep, B in {16, 32, 64} x L in {2048, 1024, 512}
    for the chunked prefill and B in {16, 32, 64} for the single-token decode step; one JSON
    line per case (each with its fraction of the measured HBM peak)."""
    lines = []
    for B in (16, 32, 64):
        for L in (2048, 1024, 512):
            args.batch, args.length, args.op = B, L, "gdn_prefill"
            lines.append(run_op(args))
    for B in (16, 32, 64):
        args.batch, args.length, args.op = B, 1, "gdn_decode"
        lines.append(run_op(args))
    return lines


# the prefill step's projection shapes at B32 x L1024 and their launches per prefill
# (qkv and o_proj in 16 attention layers, qkvz|ba and out_proj in 48 GDN layers, gate_up
# and down in all 64, lm_head once on the 32 last rows)
STEP_GEMMS = [("qkv", 32768, 14336, 5120, 0, 16), ("qkvz_ba", 32768, 16480, 5120, 0, 48),
              ("o_proj", 32768, 5120, 6144, 0, 16), ("out_proj", 32768, 5120, 6144, 0, 48),
              ("gate_up", 32768, 34816, 5120, 2, 64), ("down", 32768, 5120, 17408, 0, 64),
              ("lm_head", 32, 248320, 5120, 1, 1)]


def run_gemm_cublas(args):
    """Comparator (outside the product path and its timed region): each projection shape of
    the B32 x L1024 prefill through this library's tcgen05 GEMM and through cuBLAS
    (torch F.linear, bf16 in and out), alternately in the same process at the same clocks,
    CUDA events, median of ``--steps``. The SwiGLU shape is timed as our fused GEMM against
    the plain cuBLAS GEMM of the same [T, 2I] product (cuBLAS then still owes the SwiGLU).
    Totals weight each shape by its launches per prefill."""
    import torch
    import torch.nn.functional as F
    from qwen38_inference_b200 import ops
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    ws = ops.Workspace(dev)
    rows, ours_tot, cub_tot, flop_tot = [], 0.0, 0.0, 0.0
    for name, M, N, K, kind, per in STEP_GEMMS:
        if args.gemm_shape and name != args.gemm_shape:
            continue
        x = torch.randn(M, K, device=dev, generator=g).bfloat16()
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
        n_out = N // 2 if kind == 2 else N
        y = torch.empty(M, n_out, device=dev, dtype=torch.float32 if kind == 1 else torch.bfloat16)
        yc = torch.empty(M, N, device=dev, dtype=torch.bfloat16)

        def ours():
            ops.gemm(x, w, y, out_kind=kind, ws=ws)

        def cub():
            torch.matmul(x, w.t(), out=yc)
        for fn in (ours, cub, ours, cub, ours, cub):
            fn()
        torch.cuda.synchronize()
        t = {"ours": [], "cublas": []}
        for _ in range(args.steps):
            for key, fn in (("ours", ours), ("cublas", cub)):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                e1.synchronize()
                t[key].append(e0.elapsed_time(e1))
        mo, mc = statistics.median(t["ours"]), statistics.median(t["cublas"])
        flop = 2.0 * M * N * K
        rows.append({"shape": name, "M": M, "N": N, "K": K, "launches_per_prefill": per, "ours_ms": round(mo, 4),
                     "cublas_ms": round(mc, 4), "ours_tflops": round(flop / mo / 1e9, 1),
                     "cublas_tflops": round(flop / mc / 1e9, 1), "ratio_cublas_over_ours": round(mc / mo, 4)})
        ours_tot += per * mo
        cub_tot += per * mc
        flop_tot += per * flop
        del x, w, y, yc
    out = {"op": "gemm_cublas", "shapes": rows, "prefill_gemm_ms": {"ours": round(ours_tot, 2),
                                                                     "cublas": round(cub_tot, 2)},
           "prefill_gemm_tflops": {"ours": round(flop_tot / ours_tot / 1e9, 1),
                                   "cublas": round(flop_tot / cub_tot / 1e9, 1)},
           "ratio_cublas_over_ours": round(cub_tot / ours_tot, 4),
           "note": "alternating launches; inputs larger than L2 (each A panel >= 335 MB)"}
    print(json.dumps(out), flush=True)


def run_gemm_sustained(args):
    """The four large-M projection shapes of the B32 x L1024 prefill (gate_up with the SwiGLU
    epilogue, qkvz|ba, down, out_proj), launched back to back as in the step so that the
    GPU sits at its power cap: 40 warm rounds, then ``--steps`` timed rounds with CUDA events
    around every launch; medians per shape. The GEMM tuning knobs (QW_GEMM_WIDE,
    QW_GEMM_GROUP, QW_GEMM_PAIR) apply, so runs with different settings compare the shapes
    under the same kind of load."""
    import torch
    from qwen38_inference_b200 import ops
    from qwen38_inference_b200.config import qwen38_27b
    cfg = qwen38_27b()
    dev = "cuda"
    T = args.batch * args.length
    g = torch.Generator(device=dev).manual_seed(0)
    shapes = [("gate_up", 2 * cfg.intermediate_size, cfg.hidden_size, ops.OUT_SWIGLU),
              ("qkvz_ba", cfg.qkvz_dim + cfg.ba_dim, cfg.hidden_size, ops.OUT_BF16),
              ("down", cfg.hidden_size, cfg.intermediate_size, ops.OUT_BF16),
              ("out_proj", cfg.hidden_size, cfg.gdn_v_dim, ops.OUT_BF16)]
    bufs = {}
    for name, N, K, kind in shapes:
        x = torch.randn(T, K, device=dev, generator=g).bfloat16()
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
        y = torch.empty(T, N // 2 if kind == ops.OUT_SWIGLU else N, device=dev, dtype=torch.bfloat16)
        bufs[name] = (x, w, y, kind)
    ws = ops.Workspace(dev)
    for _ in range(40):
        for x, w, y, kind in bufs.values():
            ops.gemm(x, w, y, out_kind=kind, ws=ws)
    torch.cuda.synchronize()
    ev = {n: [] for n in bufs}
    with ClockSampler(0) as clk:
        for _ in range(args.steps):
            for name, (x, w, y, kind) in bufs.items():
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                ops.gemm(x, w, y, out_kind=kind, ws=ws)
                b.record()
                ev[name].append((a, b))
        torch.cuda.synchronize()
    out = {"op": "gemm_sustained", "tokens": T,
           "knobs": {k: os.environ.get(k) for k in ("QW_GEMM_WIDE", "QW_GEMM_GROUP", "QW_GEMM_PAIR")},
           "median_ms": {n: round(statistics.median(a.elapsed_time(b) for a, b in e), 4) for n, e in ev.items()},
           "clocks": clk.summary()}
    print(json.dumps(out), flush=True)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    t0 = time.perf_counter()
    cb = cpu_baseline(args.batch, args.length)
    wall = time.perf_counter() - t0
    out = {"metric": METRIC, "value": round(cb["value"], 2), "unit": UNIT, "impl": "reference",
           "n_gpus": args.gpus, "steps": 1, "warmup": 0, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": f"B{args.batch}xL{args.length} prefill + B{args.batch} decode, 27B hybrid (CPU sample)"},
           "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
           "e2e": {"value": round(cb["value"], 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "wall_s": round(wall, 1)}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--length", type=int, default=1024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["step", "long", "continuous", "split"], default="step",
                    help="step: the headline B32/L1024 prefill+decode (replicas over N GPUs; --batch 16 "
                         "--length 2048 is configs[1]); long: one long request with head-wise tensor parallelism "
                         "over N GPUs; continuous: configs[2] continuous batching; split: configs[4] decode of "
                         "B64 at L512 with the requests split across the N GPUs")
    ap.add_argument("--long-tokens", type=int, default=131071)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--decode-steps", type=int, default=10)
    ap.add_argument("--tp-allreduce", choices=["peer", "nccl"], default="peer",
                    help="long workload, N > 1: decode all-reduce inside the projection kernels (peer) or NCCL")
    ap.add_argument("--layers", type=int, default=0, help="--op decode_step: layers of the 27B geometry (0: all 64)")
    ap.add_argument("--gemm-shape", default=None, choices=[g[0] for g in STEP_GEMMS],
                    help="--op gemm_cublas: time only this projection shape")
    ap.add_argument("--op", choices=["gate_up", "qkvz_proj", "down_proj", "gdn_prefill", "gdn_decode",
                                     "gdn_sweep", "gdn_prefill_flashinfer", "gemm_cublas", "step_cublas",
                                     "gemm_sustained",
                                     "conv_prefill",
                                     "attn_prefill", "decode_step"],
                    default=None,
                    help="time one kernel of the step alone (the case the ncu captures run); gdn_sweep: the "
                         "configs[3] sweep; gdn_prefill_flashinfer and gemm_cublas: library comparators")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    if args.op == "decode_step":
        run_decode_step(args)
    elif args.op == "gdn_sweep":
        run_gdn_sweep(args)
    elif args.op == "gemm_cublas":
        run_gemm_cublas(args)
    elif args.op == "step_cublas":
        run_step_cublas(args)
    elif args.op == "gemm_sustained":
        run_gemm_sustained(args)
    elif args.op:
        try:
            run_op(args)
        except Unavailable as e:
            print(json.dumps({"op": args.op, "unavailable": str(e)}), flush=True)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "long":
        run_long(args)
    elif args.workload == "continuous":
        run_continuous(args)
    elif args.workload == "split":
        run_split(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
