#!/usr/bin/env python3
"""Prefill tokens/s per attention layer of exact-max shared-selection thresholded attention.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--variant shared]
    python bench.py --impl reference ...      # the reference algorithm on the host cores

Workload (default): benchmark config 2 -- Llama-3-8B-shaped GQA layer (32 q / 8 kv heads,
D=128), S=32768, B=1, bf16, YaRN factor 4 (orig 8192, mscale 1.1386), exact max, tau=5,
top 30% with the 25/20% fallback, cap 2048, query tile 64.  Synthetic seeded inputs
(sta.synth) stand in for the model activations.  A "step" is one call of the attention op on
pre-projected q, k, v: RoPE prologue + Kernel A (2 passes) + selection + attend.

Multi-GPU: one process per GPU (torchrun); the layer is partitioned across ranks by kv-head
range and/or query slab (sta.partition) with no data-path collective (strong scaling: the
job's total work is fixed).
Timing: CUDA events on torch's current stream, W untimed warm-up steps, K timed steps between
barrier + synchronize, max over ranks.  Inputs (268 MB of q alone) exceed L2 (126 MB).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "sparse-thresholded-attention_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "prefill tokens/s per attention layer"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["sta", "reference", "reference_gpu"], default="sta",
                    help="reference: the reference algorithm on the host cores (oracle port); "
                         "reference_gpu: the reference's own Triton kernels on this GPU, from "
                         "the unmodified install in baseline/_ref")
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--variant", choices=["shared", "pq_union", "pq_stream", "dca_dense"],
                    default="shared",
                    help="dca_dense: the dense Dual Chunk Attention prefill (config 3 geometry)")
    ap.add_argument("--seq-len", type=int, default=None, help="override S (profiling only)")
    ap.add_argument("--heads", type=int, default=None, help="override q heads (profiling only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-compare", action="store_true",
                    help="reference_gpu: skip the comparison with this build's results")
    ap.add_argument("--ref-heads", type=int, default=2,
                    help="reference_gpu, configs 3 / 4: (batch, head) units timed")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--partition", choices=["auto", "heads", "slabs", "grid"], default="auto",
                    help="multi-GPU unit: kv-head ranges, query slabs, or both (sta.partition)")
    ap.add_argument("--decode", action="store_true",
                    help="time one decode step (the last position against the whole cache) "
                         "instead of the prefill op; its own metric line")
    ap.add_argument("--e2e-groups", default="auto",
                    help="kv-head groups of the host-buffer pipeline (transfer / compute overlap): "
                         "a count, comma-separated kv-head counts, or auto (one kv head first and "
                         "last, the rest in two groups)")
    ap.add_argument("--max-workspace-gb", type=int, default=48,
                    help="scratch cap; larger problems run over groups of kv heads")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def workload(args):
    """Inputs + geometry of the benchmark config (full tensors, on the CPU)."""
    import torch
    from sta.synth import config_geometry, make_config_inputs
    q, k, v, c = make_config_inputs(args.config, seq_len=args.seq_len, n_heads=args.heads)
    geo, geo_c = config_geometry(c, args.variant)
    tau = torch.full((c["H"],), float(c["tau"]))
    return q, k, v, tau, geo, geo_c, c


def workload_desc(c, args, world, unit=None):
    name = c["name"] + ("" if args.variant == "shared" else f"-{args.variant}")
    return {"workload": name, "batch": c["B"], "q_heads": c["H"], "kv_heads": c["Hkv"],
            "seq_len": c["S"], "head_dim": c["D"], "tile": c["T"] if args.variant == "shared" else 32,
            "k_max": c["k_max"], "tau": c["tau"], "pct": c.get("pct", 30.0),
            "geometry": c["geom"],
            "parallelism": (f"{unit['mode']} partition x{world} ({unit['head_parts']} kv-head parts"
                            f" x {unit['slab_parts']} query slabs)") if world > 1 and unit else "single GPU",
            "l2": "no flush: inputs exceed L2 (q alone %.0f MB > 126 MB)" % (c["B"] * c["H"] * c["S"] * c["D"] * 2 / 1e6)}


# ---------------------------------------------------------------------------------------------
# CPU baseline: the oracle restatement of the reference algorithm on a bounded sample
# ---------------------------------------------------------------------------------------------
def cpu_sample(q, k, v, tau, geo, c, n_tiles=12, head=0, seed=0, geo_c=None):
    """Run the reference algorithm (oracle port) on `n_tiles` query tiles of one q head and
    extrapolate to the whole layer by causal work (cost of a tile ~ its key count).
    Returns (tokens/s estimate, seconds spent, description)."""
    import numpy as np
    from oracle import sta_oracle as oracle
    T, N, D, H, Hk = c["T"], c["S"], c["D"], c["H"], c["Hkv"]
    nt = (N + T - 1) // T
    rng = np.random.default_rng(seed)
    tiles = sorted(rng.choice(nt, size=min(n_tiles, nt), replace=False).tolist())
    kv = head // (H // Hk)
    qh = q[0, head:head + 1].float().numpy()
    kh = k[0, kv:kv + 1].float().numpy()
    vh = v[0, kv:kv + 1].float().numpy()
    geo_c = geo_c or geo
    invf = geo["inv_freq"].numpy()
    sm = 1.0 / math.sqrt(D)
    t0 = time.perf_counter()
    sel = oracle.select_vote(qh, kh, tau[head:head + 1].numpy(), invf, geo["pos_scale"],
                             geo["rope_scale"], sm, T, tiles=tiles, dca=geo.get("dca"))
    idx = np.full((1, nt, c["k_max"]), N, np.int32)
    npk = np.zeros((1, nt, c["k_max"]), np.float32)
    npq = np.zeros((1, nt, T), np.float32)
    for t in tiles:
        s = oracle.build_sets(sel["votes"][:, t:t + 1], geo_c["pos_scale"], 32, 32, c["pct"], T,
                              c["k_max"], q_pos_base=t * T)
        idx[:, t], npk[:, t], npq[:, t] = s[0][:, 0], s[1][:, 0], s[2][:, 0]
    oracle.gather_attn(qh, kh, vh, geo_c["inv_freq"].numpy(), idx, npk, npq, sm,
                       geo_c["rope_scale"], T, v_is_bf16=True, tiles=tiles)
    dt = time.perf_counter() - t0
    work_sample = sum(min((t + 1) * T, N) for t in tiles)
    work_total = H * c["B"] * sum(min((t + 1) * T, N) for t in range(nt))
    est = dt * work_total / work_sample
    tok_s = c["B"] * N / est
    desc = (f"oracle port (numpy) on {len(tiles)} of {nt} query tiles of 1 of {H} q heads, "
            f"{dt:.1f} s; extrapolated by causal key count to the whole layer ({est:.0f} s)")
    return tok_s, dt, desc


class _Capture:
    """Record the inputs / result of one module-level function of the reference for one call."""

    def __init__(self, module, name):
        self.module, self.name, self.orig = module, name, getattr(module, name)
        self.args = self.result = None

    def __enter__(self):
        def wrapped(*a, **kw):
            self.args = a
            self.result = self.orig(*a, **kw)
            return self.result
        setattr(self.module, self.name, wrapped)
        return self

    def __exit__(self, *exc):
        setattr(self.module, self.name, self.orig)


def _time_calls(fn, warmup, steps):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _compare_with_reference(c, q, k, v, tau, geo, geo_c, ref_out, ref_votes, ref_stats):
    """This build vs the reference's Triton op on identical inputs (the reference receives
    repeat_kv-expanded k / v, this build the GQA-native ones): Kernel A votes, per-tile
    statistics, and outputs overall and on the tiles whose votes agree exactly."""
    import numpy as np
    import torch
    from sta import core
    from sta.core import Geometry
    dev = q.device
    H, N, T = c["H"], c["S"], c["T"]
    nt = (N + T - 1) // T
    ga = Geometry(geo["inv_freq"], geo["pos_scale"], geo["rope_scale"])
    gc = Geometry(geo_c["inv_freq"], geo_c["pos_scale"], geo_c["rope_scale"])
    out, st, _ = core.forward("shared", q, k, v, tau, ga, gc, tile=T, k_max=c["k_max"],
                              pct=c["pct"])
    sel = core.select(q[0], k[0], tau, ga, tile=T)
    hi = torch.clamp((torch.arange(nt, device=dev) + 1) * T, max=N)
    mask = torch.arange(N, device=dev)[None, :] < hi[:, None]            # (nt, N)
    ours = sel["votes"].view(H, -1).int()
    d = (ref_votes[0][:, mask].int() - ours).abs() if ref_votes.dim() == 4 else \
        (ref_votes[:, mask].int() - ours).abs()
    seg = torch.cumsum(hi, 0)
    csum = torch.cumsum(d.long(), 1)
    ends = csum[:, seg - 1]
    per_tile = torch.diff(ends, dim=1, prepend=torch.zeros_like(ends[:, :1]))  # (H, nt)
    agree = per_tile == 0
    res = {"vote_entries": int(d.numel()), "vote_entries_differing": int((d > 0).sum()),
           "vote_abs_diff_sum": int(d.sum()), "tiles": int(agree.numel()),
           "tiles_votes_identical": int(agree.sum())}
    for name in ("shared_size", "kept_size"):
        r = ref_stats[name].to(dev).reshape(H, nt)
        o = st[name][0].to(r.dtype)
        res[f"{name}_equal_tiles"] = int((r == o).sum())
        res[f"{name}_equal_on_identical_vote_tiles"] = bool((r == o)[agree].all())
    err = (out[0].float() - ref_out[0].float()).abs()                    # (H, N, D)
    res["out_max_abs"] = float(err.max())
    res["out_mean_abs"] = float(err.mean())
    row_agree = agree.repeat_interleave(T, 1)[:, :N]
    e_ok = err[row_agree]
    res["out_max_abs_identical_vote_tiles"] = float(e_ok.max()) if e_ok.numel() else None
    res["out_mean_abs_identical_vote_tiles"] = float(e_ok.mean()) if e_ok.numel() else None
    # Is every vote difference a near-threshold key?  keep = s >= m - tau, so this build's votes
    # at tau - delta and tau + delta bracket every vote that score errors of at most delta can
    # produce: a reference vote inside the bracket is explained by such errors.
    for delta in (1e-3, 1e-2):
        lo = core.select(q[0], k[0], tau - delta, ga, tile=T)["votes"].view(H, -1).int()
        hi_ = core.select(q[0], k[0], tau + delta, ga, tile=T)["votes"].view(H, -1).int()
        r = ref_votes[:, mask].int()
        inside = (r >= lo) & (r <= hi_)
        diff = d > 0
        res[f"differing_explained_within_{delta:g}"] = int((diff & inside).sum())
        del lo, hi_, r, inside
    res["note"] = ("reference scores with tl.dot (TF32 on this GPU); this build with three bf16 "
                   "products (~2^-16).  differing_explained_within_x: differing vote entries "
                   "that lie between this build's votes at tau - x and tau + x, i.e. that score "
                   "errors of at most x around the threshold account for")
    return res


def run_reference_gpu(args):
    """--impl reference_gpu: the reference's own Triton prefill ops on this GPU, unmodified,
    imported from baseline/_ref, same seeded inputs and CUDA-events protocol.  The reference
    receives repeat_kv-expanded k / v as its hooks pass them (exact_2.py:644-646).

    configs 1 / 2 (shared): the whole layer, plus a comparison with this build on the same
    inputs (votes, statistics, outputs).  Config 3 (the reference's two-geometry hybrid kernel,
    shared_selection_triton_hybrid_exact.py:450-510; the reference has no thresholded DCA) and
    config 4 (PQ-Union, perquery.py:459-525; PQ-Stream, pqstream_kernel.py:498-564): the
    reference's (H, n_tiles, N) buffers do not fit a whole layer (68 GiB per array at 128k), so
    the op runs per (batch element, head) -- exact, every head is independent -- on a few
    heads, and the layer time is that per-head time x batch x heads (`extrapolated`).
    Rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    line = {"impl": "reference_gpu", "metric": METRIC, "unit": "tokens/s"}
    if not os.path.isdir(ref_dir):
        line["unavailable"] = "reference install missing (baseline/_ref)"
        emit(line)
        return
    import tempfile as _tf
    os.environ.setdefault("TRITON_CACHE_DIR", _tf.mkdtemp(prefix="ref_triton_"))
    sys.path.insert(0, ref_dir)
    import torch
    q, k, v, tau, geo, geo_c, c = workload(args)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, H, Hk, N = c["B"], c["H"], c["Hkv"], c["S"]
    G = H // Hk
    taud = tau.to(dev)
    ia = geo["inv_freq"].to(dev)
    ic = geo_c["inv_freq"].to(dev)
    extra = {}
    if args.config in (1, 2) and args.variant == "shared":
        mod = __import__("shared_selection_triton_YaRN_exact" if c["geom"] == "yarn"
                         else "shared_selection_triton_exact_2")
        qd = q.to(dev)
        kd = k.to(dev).repeat_interleave(G, 1)
        vd = v.to(dev).repeat_interleave(G, 1)

        def step():
            return mod.shared_pi_attention(qd, kd, vd, taud, ia, pos_scale=geo["pos_scale"],
                                           pct=c["pct"], rope_scale=geo["rope_scale"],
                                           tile=c["T"], k_max=c["k_max"])
        ms = _time_calls(step, args.warmup, args.steps)
        est = False
        if not args.no_compare:
            with _Capture(mod, "_build_sets") as cap:
                r = step()
            torch.cuda.synchronize()
            stats = {"shared_size": r[1], "kept_size": r[2]}
            votes = cap.args[0]
            del kd, vd
            extra["vs_this_build"] = _compare_with_reference(
                c, qd, k.to(dev), v.to(dev), tau, geo, geo_c, r[0], votes, stats)
    else:
        n_units = max(1, args.ref_heads)
        units = [(b, h) for b in range(B) for h in range(H)]
        step_idx = [int(i * (len(units) - 1) / max(n_units - 1, 1)) for i in range(n_units)]
        picks = [units[i] for i in step_idx]
        per = []
        for b, h in picks:
            qd = q[b:b + 1, h:h + 1].to(dev)
            kd = k[b:b + 1, h // G:h // G + 1].to(dev)
            vd = v[b:b + 1, h // G:h // G + 1].to(dev)
            t1 = taud[h:h + 1]
            if args.variant == "shared":
                mod = __import__("shared_selection_triton_hybrid_exact")
                fn = lambda: mod.shared_pi_attention(  # noqa: E731
                    qd, kd, vd, t1, ia, geo["pos_scale"], geo["rope_scale"], ic,
                    geo_c["pos_scale"], geo_c["rope_scale"], pct=c["pct"], tile=c["T"],
                    k_max=c["k_max"])
            elif args.variant == "pq_union":
                mod = __import__("shared_selection_triton_perquery")
                fn = lambda: mod.shared_pq_attention(  # noqa: E731
                    qd, kd, vd, t1, ia, ic, geo["pos_scale"], geo["rope_scale"],
                    k_max=c["k_max"], select_score="expmass")
            else:
                mod = __import__("pqstream_kernel")
                fn = lambda: mod.pqstream_attention(  # noqa: E731
                    qd, kd, vd, t1, ia, ic, geo["pos_scale"], geo["rope_scale"], block_n=32)
            per.append(_time_calls(fn, 1, max(1, min(args.steps, 2))))
            del qd, kd, vd
            torch.cuda.empty_cache()
        ms = statistics.mean(per) * B * H
        est = True
        extra["per_head_ms"] = per
        extra["sampled_units"] = [list(x) for x in picks]
        extra["extrapolated"] = True
        extra["how"] = "per-(batch, head) calls of the reference op, mean x batch x heads"
    line.update({"value": B * N / (ms / 1e3), "ms_per_step": ms, "n_gpus": 1,
                 "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                 "dtype": "bf16 inputs (reference Triton: fp32 RoPE, tl.dot)",
                 "config": workload_desc(c, args, 1), "extrapolated": est,
                 "source": "unmodified reference modules installed by pip into baseline/_ref"})
    line.update(extra)
    emit(line)


def parity_block(q, k, v, tau, geo, geo_c, c, qd, kd, out, ga, n_tiles=12, seed=7):
    """Checker beside the CPU baseline: this run's output against the oracle on a seeded
    sample of query tiles (plus the last tile) of q head 0 at the benchmark's full length.
    Kernel A's votes of head 0 (read back through sta_select) must equal the oracle's except
    keys whose score is within 1e-3 of the threshold; the oracle then selects and attends on
    those device votes, and the op's output rows must be within max-abs 2e-2 / mean-abs 1e-3."""
    import numpy as np
    from oracle import sta_oracle as oracle
    from sta import core
    T, N, D, k_max = c["T"], c["S"], c["D"], c["k_max"]
    nt = (N + T - 1) // T
    rng = np.random.default_rng(seed)
    tiles = sorted(set(int(x) for x in rng.choice(nt, size=min(n_tiles, nt), replace=False)) | {nt - 1})
    sel = core.select(qd[0, 0:1], kd[0, 0:1], tau[0:1], ga, tile=T)
    votes = sel["votes"].cpu().numpy()
    sm = 1.0 / math.sqrt(D)
    qx, kx, vx = q[0, 0].float().numpy(), k[0, 0].float().numpy(), v[0, 0].float().numpy()
    ora = oracle.select_tiles(qx, kx, c["tau"], geo["inv_freq"].numpy(), geo["pos_scale"],
                              geo["rope_scale"], sm, T, tiles, dca=geo.get("dca"))
    outside = flips = 0
    idx = np.full((1, nt, k_max), N, np.int32)
    npk = np.zeros((1, nt, k_max), np.float32)
    npq = np.zeros((1, nt, T), np.float32)
    for t in tiles:
        o = ora[t]
        off = T * t * (t + 1) // 2
        dv = votes[off:off + o["hi"]].astype(np.int64)
        d = np.abs(dv - o["votes"])
        outside += int((d > o["near"]).sum())
        flips += int(d.sum())
        v1 = np.zeros((1, 1, N), np.int64)
        v1[0, 0, :o["hi"]] = dv
        s_ = oracle.build_sets(v1, geo_c["pos_scale"], 32, 32, c["pct"], T, k_max, q_pos_base=t * T)
        idx[0, t], npk[0, t], npq[0, t] = s_[0][0, 0], s_[1][0, 0], s_[2][0, 0]
    ref = oracle.gather_attn(qx[None], kx[None], vx[None], geo_c["inv_freq"].numpy(), idx, npk,
                             npq, sm, geo_c["rope_scale"], T, v_is_bf16=True, tiles=tiles)
    got = out[0, 0].float().cpu().numpy()
    rows = np.concatenate([np.arange(t * T, min((t + 1) * T, N)) for t in tiles])
    err = np.abs(got[rows] - ref[0, rows])
    return {"head": 0, "tiles": len(tiles), "vote_keys_outside_boundary": outside,
            "boundary_vote_flips": flips, "out_max_abs": float(err.max()),
            "out_mean_abs": float(err.mean()), "tolerance": "max-abs 2e-2, mean-abs 1e-3",
            "pass": bool(outside == 0 and err.max() <= 2e-2 and err.mean() <= 1e-3)}


def run_reference(args):
    """--impl reference: the reference's algorithm on the host cores (oracle port).

    A full cfg2 layer would take minutes of CPU time per step, so each step is a bounded sample
    (48 query tiles of one q head) whose time is extrapolated by causal key count to the whole
    layer.  The line says so: `extrapolated` is true, `steps` / `ms_per_step` are the timed
    samples themselves, `value` is the extrapolated whole-layer throughput."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.config == 0:
        return run_reference_interpreter(args)
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    q, k, v, tau, geo, geo_c, c = workload(args)
    world = args.gpus
    for i in range(args.warmup):
        cpu_sample(q, k, v, tau, geo, c, n_tiles=2, seed=100 + i, geo_c=geo_c)
    vals, secs = [], []
    t0 = time.perf_counter()
    desc = ""
    n_tiles = 48
    for i in range(args.steps):
        tok, dt, desc = cpu_sample(q, k, v, tau, geo, c, n_tiles=n_tiles, seed=i, geo_c=geo_c)
        vals.append(tok)
        secs.append(dt)
    value = statistics.median(vals)
    cores = os.cpu_count() or 1
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.median(secs),
            "extrapolated": True,
            "sample_per_step": f"{n_tiles} query tiles of 1 of {c['H'] * c['B']} q heads",
            "est_ms_per_layer": 1e3 * c["B"] * c["S"] / value,
            "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32 (numpy oracle on bf16 inputs)",
            "data": "synthetic (seeded, sta.synth)", "config": workload_desc(c, args, 1),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "cpu_model": cpu_model(), "sample": desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t0}
    emit(line)


def run_reference_interpreter(args):
    """--impl reference --config 0: the UNMODIFIED reference (shared_pi_attention of
    shared_selection_triton_exact_2.py, from baseline/_ref) under TRITON_INTERPRET=1 on the host
    cores, on the whole config-0 layer (fp32, 4 heads x 1024 tokens): every step is a complete
    timed call, nothing is extrapolated."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    line = {"impl": "reference", "metric": METRIC, "unit": "tokens/s"}
    if not os.path.isdir(ref_dir):
        line["unavailable"] = "reference install missing (baseline/_ref)"
        emit(line)
        return
    os.environ["TRITON_INTERPRET"] = "1"  # before triton is imported by the reference module
    import tempfile as _tf
    os.environ.setdefault("TRITON_CACHE_DIR", _tf.mkdtemp(prefix="ref_triton_"))
    sys.path.insert(0, ref_dir)
    import torch
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    q, k, v, tau, geo, geo_c, c = workload(args)
    mod = __import__("shared_selection_triton_exact_2")

    def step():
        return mod.shared_pi_attention(q, k, v, tau, geo["inv_freq"], pos_scale=geo["pos_scale"],
                                       pct=c["pct"], rope_scale=geo["rope_scale"], tile=c["T"],
                                       k_max=c["k_max"])
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = c["B"] * c["S"] / dt
    line.update({"value": value, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                 "ms_per_step": 1e3 * dt, "extrapolated": False, "higher_is_better": True,
                 "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                 "data": "synthetic (seeded, sta.synth)", "config": workload_desc(c, args, 1),
                 "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores,
                                  "kind": "reference", "cpu_model": cpu_model(),
                                  "sample": "the whole config-0 layer per step, reference "
                                            "Triton kernels under TRITON_INTERPRET=1"},
                 "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0}})
    emit(line)


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        load = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def run_gpu(args):
    import torch
    import torch.distributed as dist
    from sta import core
    from sta.core import Geometry

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", device_id=dev)
    q, k, v, tau, geo, geo_c, c = workload(args)
    H, Hk, N, D, B = c["H"], c["Hkv"], c["S"], c["D"], c["B"]
    from sta.partition import plan
    unit = plan(Hk, N, world, rank, args.partition)
    G = H // Hk
    k0, k1 = unit["kv"]
    s0, s1 = unit["slab"]
    qs = q[:, k0 * G:k1 * G, s0:s1].contiguous()
    ks = k[:, k0:k1, :s1].contiguous()
    vs = v[:, k0:k1, :s1].contiguous()
    taus = tau[k0 * G:k1 * G]
    qd, kd, vd = qs.to(dev), ks.to(dev), vs.to(dev)
    ga = Geometry(geo["inv_freq"], geo["pos_scale"], geo["rope_scale"], geo.get("dca"))
    gc = Geometry(geo_c["inv_freq"], geo_c["pos_scale"], geo_c["rope_scale"])
    T = c["T"] if args.variant == "shared" else 32
    kw = dict(tile=T, k_max=c["k_max"], pct=c.get("pct", 30.0),
              select_score="freq" if args.variant == "shared" else "expmass", block_n=32,
              max_workspace_bytes=args.max_workspace_gb << 30, q_pos_base=s0)

    def step(qq, kk, vv, evs=None):
        return core.forward(args.variant, qq, kk, vv, taus, ga, gc, stage_events=evs, **kw)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        out, st, _ = step(qd, kd, vd)
    torch.cuda.synchronize()

    K = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(K)]
    for row in evs:
        for e in row:
            e.record()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        start.record()
        for i in range(K):
            out, st, _ = step(qd, kd, vd, evs[i])
        end.record()
        torch.cuda.synchronize()
        barrier()
    ms_total = start.elapsed_time(end)
    # the op runs once per batch element and per group of kv heads (scratch cap); the events
    # bracket the last group of the last element: scale by both counts
    ngroups = int(st.get("kv_head_groups", 1))
    stage_ms = [0.0] * 4
    for row in evs:
        for j in range(4):
            stage_ms[j] += B * ngroups * row[j].elapsed_time(row[j + 1]) / K
    t = torch.tensor([ms_total], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / K
    tokens = B * N
    value = tokens / (ms_step / 1e3)

    # ---- end to end through the public API with host buffers: sta.core.forward_host copies
    # pinned q / k / v in and the output back every step, overlapped with the compute by
    # kv-head group (H2D + op + D2H inside the timed region)
    e2e = None
    if not args.no_e2e:
        qh, kh, vh = qs.pin_memory(), ks.pin_memory(), vs.pin_memory()
        ekw = dict(kw)
        ekw.pop("max_workspace_bytes")
        ekw["max_workspace_bytes"] = args.max_workspace_gb << 30

        units = ks.shape[1] if ks.shape[1] > 1 else qs.shape[1]  # kv heads, or q heads
        if args.e2e_groups == "auto":
            mid = units - 2     # one unit first and last, the rest in two groups
            groups = ([1] + [x for x in (mid - mid // 2, mid // 2) if x] + [1]) if units > 2 \
                else units
        elif "," in args.e2e_groups:
            groups = [int(x) for x in args.e2e_groups.split(",")]
        else:
            groups = int(args.e2e_groups)

        def step_host():
            return core.forward_host(args.variant, qh, kh, vh, taus, ga, gc, groups=groups, **ekw)
        for _ in range(2):
            out_h, _ = step_host()
        torch.cuda.synchronize()
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(K):
            out_h, _ = step_host()
        e2.record()
        torch.cuda.synchronize()
        t2 = torch.tensor([s2.elapsed_time(e2)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        e2e_ms = float(t2.item()) / K
        nb = torch.tensor([sum(x.numel() * x.element_size() for x in (qs, ks, vs)),
                           out_h.numel() * out_h.element_size()], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(nb)  # bytes copied by all ranks together
        e2e = {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(nb[0].item()), "d2h_bytes_per_step": int(nb[1].item()),
               "api": f"sta.core.forward_host, pinned host buffers, kv-head groups {groups} "
                      "overlapping H2D / compute / D2H"}

    # ---- roofline of the dominant kernel (Kernel A on tensor cores)
    # screened scoring runs for unweighted selections (shared freq votes, PQ-Stream bits)
    screened = os.environ.get("STA_SELECT_SCREEN", "0") == "1" and args.variant != "pq_union"
    pk, pk_kind = peaks()
    Hr = qs.shape[1]
    pairs = (s1 * (s1 + 1) - s0 * (s0 + 1)) / 2   # causal (query, key) pairs of this rank's slab
    flops_sel = 2 * 2 * D * Hr * B * pairs      # two passes for every variant
    sel_ms = stage_ms[1]
    achieved = flops_sel / (sel_ms / 1e3) / 1e12
    peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
    traffic, traffic_src = select_traffic_bytes(c, Hr, s0, s1)
    roof = {"kernel": "select_kernel (tcgen05 exact-max Kernel A)", "bound": "tensor",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_kind": f"{pk_kind} bf16 sustained", "traffic": traffic,
            "traffic_source": traffic_src,
            "algorithmic_flops_per_launch": flops_sel, "launch_ms": sel_ms,
            "tensor_flops_issued_per_launch": (1.5 if screened else 3) * flops_sel,
            "note": ("screened scoring: 3 passes of ONE fp16 product per pair (screened max, "
                     "exact max of the candidates, votes); pairs within the proven bound of the "
                     "max / threshold rescored exactly on the CUDA cores; the launch time "
                     "includes the fp16-operand / norm prep kernel") if screened else
                    "3 bf16 products per fp32-accurate score (hi*hi + hi*lo + lo*hi)"}

    # per op call: the cos/sin table, then per kv-head group the RoPE prologue of q and k (q in
    # 3 planes for DCA), Kernel A, the selection and the attend (PQ-Stream: pass 2 fused)
    per_group = {"shared": 5, "pq_union": 5, "pq_stream": 4}[args.variant] + (2 if geo.get("dca") else 0)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import torch as _t
        _t.set_num_threads(os.cpu_count() or 1)
        tok_cpu, _, desc = cpu_sample(q, k, v, tau, geo, c, n_tiles=240, geo_c=geo_c)
        cpu = {"value": tok_cpu, "unit": "tokens/s", "cores": os.cpu_count() or 1,
               "kind": "port", "sample": desc}
        if args.variant == "shared" and s0 == 0 and k0 == 0:
            cpu["parity"] = parity_block(q, k, v, tau, geo, geo_c, c, qd, kd, out, ga)
    stats = {}
    if args.variant == "shared":
        ks_ = st["kept_size"].float()
        stats = {"mean_kept_size": float(ks_.mean()), "max_kept_size": float(ks_.max()),
                 "overflow_frac": float(st["overflow"].float().mean()),
                 "unresolved_frac": float(st["overflow20"].float().mean()),
                 "fallback_tiles": int(((st["chosen"] > 0) & (st["chosen"] < 30)).sum())}
    elif args.variant == "pq_union":
        stats = {"mean_usize": float(st["usize"].float().mean()),
                 "mean_kept_size": float(st["kept_size"].float().mean()),
                 "overflow_frac": float(st["overflow"].float().mean())}
    else:
        used = (st["blocks"] - st["skipped"]).float()
        stats = {"mean_kept_per_query": float(st["kept"].float().mean()),
                 "mean_blocks_per_tile": float(st["blocks"].float().mean()),
                 "mean_advancing_blocks_per_tile": float(used.mean()),
                 "mean_span": float(st["span"].float().mean())}
    clocks = clk.summary()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": K, "warmup": args.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded generator sta.synth, BASELINE config shapes)",
                "config": workload_desc(c, args, world, unit), "clocks": clocks, "e2e": e2e,
                "gpu_launches": K * B * (1 + per_group * ngroups),
                "kv_head_groups": ngroups,
                "stage_ms": {"rope_prologue": stage_ms[0], "select_tcgen05": stage_ms[1],
                             "build_sets": stage_ms[2], "attend": stage_ms[3]},
                "roofline": roof, "cpu_baseline": cpu, "selection": stats,
                "parity": (cpu or {}).get("parity")}
        emit(line)
    if world > 1:
        dist.destroy_process_group()


def run_gpu_dca(args):
    """--variant dca_dense: the dense Dual Chunk Attention prefill (sta_dca_forward, the
    reference's dca_forward core) on the config's inputs and DCA geometry (config 3: chunk
    6144, local window 1024, mscale of the sequence length), 1 GPU, CUDA events."""
    import torch
    from sta import core
    q, k, v, tau, geo, geo_c, c = workload(args)
    if not geo.get("dca"):
        raise SystemExit("--variant dca_dense needs a DCA geometry (config 3)")
    dev = torch.device("cuda", 0)
    B, H, N, D = c["B"], c["H"], c["S"], c["D"]
    qd, kd, vd = q.to(dev), k.to(dev), v.to(dev)
    s_, w_ = geo["dca"]

    def step():
        return core.dca_dense(qd, kd, vd, geo["inv_freq"], chunk_size=s_, local_window=w_,
                              rope_scale=geo["rope_scale"])
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    pk, pk_kind = peaks()
    flops = 4 * D * B * H * N * (N + 1) / 2     # S = Q.K^T and O = P.V over causal pairs
    achieved = flops / (ms / 1e3) / 1e12
    peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
    emit({"metric": METRIC, "value": B * N / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
          "data": "synthetic (seeded generator sta.synth, BASELINE config shapes)",
          "config": dict(workload_desc(c, args, 1), chunk_size=s_, local_window=w_),
          "clocks": clk.summary(), "gpu_launches": args.steps * B * 6,
          "roofline": {"kernel": "dca_dense_kernel (tcgen05 S = Q.K^T, O = P.V, P in TMEM)",
                       "bound": "tensor", "achieved": achieved, "peak": peak,
                       "unit": "TFLOP/s", "frac": achieved / peak,
                       "peak_kind": f"{pk_kind} bf16 sustained",
                       "algorithmic_flops_per_launch": flops / B}})


def run_decode(args):
    """--decode: one decode step of the variant's rule (shared -> PI cap + reposition, pq_union
    -> dense ranks, pq_stream -> streamed positions) for the config's last position against the
    whole cache, CUDA events, 1 GPU.  HBM traffic: the cache's K once (scores) + the kept rows."""
    import torch
    from sta import core
    from sta.core import Geometry
    q, k, v, tau, geo, geo_c, c = workload(args)
    dev = torch.device("cuda", 0)
    N = c["S"]
    qd = q[:, :, N - 1].contiguous().to(dev)
    kd, vd = k.to(dev), v.to(dev)
    ga = Geometry(geo["inv_freq"], geo["pos_scale"], geo["rope_scale"])
    gc = Geometry(geo_c["inv_freq"], geo_c["pos_scale"], geo_c["rope_scale"])
    mode = {"shared": "pi", "pq_union": "rank", "pq_stream": "stream"}[args.variant]
    kw = dict(k_max=c["k_max"], block_n=32)
    for _ in range(max(args.warmup, 3)):
        out, st, _ = core.decode(mode, qd, kd, vd, tau, ga, gc, **kw)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out, st, _ = core.decode(mode, qd, kd, vd, tau, ga, gc, **kw)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    kv_bytes = kd.numel() * kd.element_size()
    pk, pk_kind = peaks()
    gbs = kv_bytes / (ms / 1e3) / 1e9
    emit({"metric": "decode steps/s per attention layer", "value": 1e3 / ms, "unit": "steps/s",
          "ms_per_step": ms, "n_gpus": 1, "steps": args.steps, "higher_is_better": True,
          "config": dict(workload_desc(c, args, 1), context=N, mode=mode),
          "mean_kept": float(st["kept"].float().mean()),
          "roofline": {"bound": "hbm", "achieved": gbs, "peak": float(pk["hbm_gbs"]),
                       "unit": "GB/s", "frac": gbs / float(pk["hbm_gbs"]),
                       "note": f"K cache read once for the scores ({kv_bytes} bytes); {pk_kind} peak"}})


def select_traffic_bytes(c, heads, s0, s1):
    """DRAM bytes of one select launch.  A committed ncu measurement at the same shape is used
    as is; otherwise the committed small-case measurement is split into the part that grows
    with the rows (first reads of the q / k hi + lo operands: S) and the rest (K re-reads that
    miss L2 and the compact vote writes: causal pairs, S^2), and each part is scaled by its
    own law."""
    p = os.path.join(ROOT, "profiles", "select_kernel_traffic.json")
    if not os.path.exists(p):
        return None, None
    with open(p) as f:
        d = json.load(f)
    D, G = c["D"], c["H"] // c["Hkv"]
    if d.get("seq_len") == s1 and s0 == 0 and d.get("heads") == heads and d.get("head_dim", D) == D:
        return d["dram_bytes"], "ncu at this shape"
    n0, h0 = d["seq_len"], d["heads"]
    lin0 = 4 * D * n0 * (h0 + h0 // G)                  # q hi + lo, k hi + lo (bf16)
    quad0 = max(d["dram_bytes"] - lin0, 0)
    rows = s1 - s0
    lin = 4 * D * (rows * heads + s1 * max(heads // G, 1))
    pairs = (s1 * (s1 + 1) - s0 * (s0 + 1)) / 2
    quad = quad0 * (heads * pairs) / (h0 * n0 * (n0 + 1) / 2)
    return lin + quad, f"ncu at S={n0}, split into S and S^2 parts and scaled"


_JSON_FD = None


def emit(line: dict):
    """Print the one JSON result line on the original stdout."""
    data = (json.dumps(line) + "\n").encode()
    if _JSON_FD is not None:
        os.write(_JSON_FD, data)
    else:
        sys.stdout.write(data.decode())
        sys.stdout.flush()


def main():
    global _JSON_FD
    args = parse()
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # libraries (NCCL's version banner) write to fd 1; keep stdout for the JSON line only
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)
    if args.decode:
        run_decode(args)
    elif args.variant == "dca_dense" and args.impl == "sta":
        run_gpu_dca(args)
    elif args.impl == "reference_gpu":
        run_reference_gpu(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
