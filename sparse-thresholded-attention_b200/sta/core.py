"""Torch-facing plumbing around the C ABI: argument normalisation, output allocation,
workspace allocation (torch caching allocator) and the launch on torch's current stream.

Everything numeric runs in libsta.so; this module only moves pointers.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib as L


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return L.STA_DTYPE_F32
    if dt == torch.bfloat16:
        return L.STA_DTYPE_BF16
    raise TypeError(f"unsupported dtype {dt} (float32 or bfloat16)")


def _rows(x: torch.Tensor) -> torch.Tensor:
    """(heads, n, d) view with a contiguous last dim (copy only when needed)."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


@dataclass
class Geometry:
    """RoPE geometry: frequencies, position compression, cos/sin scale (YaRN mscale)."""
    inv_freq: torch.Tensor
    pos_scale: float = 1.0
    rope_scale: float = 1.0
    # (chunk_size, local_window): Dual Chunk Attention position ids (selection geometry only)
    dca: tuple | None = None


def _dev_f32(x, device):
    return x.to(device=device, dtype=torch.float32).contiguous()


def _check_inputs(q, k, v, q_pos_base=0):
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("q, k, v must be CUDA tensors (there is no CPU path)")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be (Z, H, N, D)")
    Z, H, Nq, D = q.shape
    N = k.shape[2]
    if k.shape[0] != Z or v.shape != k.shape or Nq + q_pos_base != N or k.shape[3] != D:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if H % k.shape[1]:
        raise ValueError("number of q heads must be a multiple of the number of kv heads")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share one dtype")
    dtype_code(q.dtype)
    return Z, H, k.shape[1], N, D


def forward(variant: str, q, k, v, tau, ga: Geometry, gc: Geometry, *, sm_scale=None,
            pct=30.0, n_global=32, n_local=32, tile=32, k_max=1024, select_score="freq",
            measure=False, block_n=32, pos_advance="max", use_skip=True, keep_sets=False,
            max_workspace_bytes=0, stage_events=None, chunk_size=16, n_chunk=0,
            chunk_agg="sum", q_pos_base=0):
    """Run one prefill op.  variant: 'shared' | 'pq_union' | 'pq_stream' | 'chunk'.
    q (Z,H,N,D); k, v (Z,Hkv,N,D) with H % Hkv == 0 (Hkv == H for repeat_kv-expanded input).
    q_pos_base > 0 (a multiple of 128): q holds only the queries at positions
    q_pos_base..N-1 (a query slab, (Z,H,N-q_pos_base,D)); k / v hold all N keys and the
    statistics cover the slab's tiles.  Every query tile is independent of the others, so slabs
    reproduce the whole-sequence call exactly.
    Returns (out (Z,H,Nq,D), dict of per-(head, tile) statistics [+ sets when keep_sets])."""
    q_pos_base = int(q_pos_base)
    if q_pos_base < 0 or q_pos_base % 128:
        raise ValueError("q_pos_base must be a non-negative multiple of 128")
    Z, H, Hk, N, D = _check_inputs(q, k, v, q_pos_base)
    Nq = N - q_pos_base
    dev = q.device
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    T = int(tile)
    nt = (Nq + T - 1) // T
    tau_d = _dev_f32(tau, dev).reshape(-1)
    if tau_d.numel() != H:
        raise ValueError(f"tau must have one entry per q head ({H}), got {tau_d.numel()}")
    ia = _dev_f32(ga.inv_freq, dev)
    ic = _dev_f32(gc.inv_freq, dev)
    same_geometry = int(ia.shape == ic.shape and float(ga.rope_scale) == float(gc.rope_scale)
                        and bool(torch.equal(ga.inv_freq.detach().float().cpu(),
                                             gc.inv_freq.detach().float().cpu())))
    if ia.numel() != D // 2 or ic.numel() != D // 2:
        raise ValueError("inv_freq must have head_dim/2 entries")
    out = torch.empty((Z, H, Nq, D), dtype=q.dtype, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    st = {}
    if variant == "shared":
        for name in ("shared_size", "kept_size", "chosen", "kpct_meas"):
            st[name] = torch.empty((Z, H, nt), **i32)
        st["overflow"] = torch.empty((Z, H, nt), dtype=torch.uint8, device=dev)
        st["overflow20"] = torch.empty((Z, H, nt), dtype=torch.uint8, device=dev)
    elif variant == "pq_union":
        st["usize"] = torch.empty((Z, H, nt), **i32)
        st["kept_size"] = torch.empty((Z, H, nt), **i32)
        st["overflow"] = torch.empty((Z, H, nt), dtype=torch.uint8, device=dev)
    elif variant == "chunk":
        st["usize"] = torch.empty((Z, H, nt), **i32)
        st["kept_size"] = torch.empty((Z, H, nt), **i32)
    elif variant == "pq_stream":
        f32 = dict(dtype=torch.float32, device=dev)
        st["span"] = torch.empty((Z, H, nt), **f32)
        st["kept"] = torch.empty((Z, H, Nq), **i32)
        st["blocks"] = torch.empty((Z, H, nt), **f32)
        st["skipped"] = torch.empty((Z, H, nt), **f32)
    else:
        raise ValueError(variant)
    sets = {}
    if keep_sets and variant != "pq_stream":
        sets["idx"] = torch.empty((Z, H, nt, k_max), **i32)
        sets["newpos_k"] = torch.empty((Z, H, nt, k_max), dtype=torch.float32, device=dev)
        sets["newpos_q"] = torch.empty((Z, H, nt, T), dtype=torch.float32, device=dev)
        if variant in ("pq_union", "chunk"):
            sets["mask"] = torch.empty((Z, H, nt, k_max), **i32)
    lib = L.lib()
    fn_ws = getattr(lib, f"sta_{variant}_workspace_bytes")
    fn = getattr(lib, f"sta_{variant}_forward")
    stream = _stream()
    ws = None
    for b in range(Z):
        qb, kb, vb = _rows(q[b]), _rows(k[b]), _rows(v[b])
        a = L.ForwardArgs()
        a.q, a.q_stride_h, a.q_stride_n = qb.data_ptr(), qb.stride(0), qb.stride(1)
        a.k, a.k_stride_h, a.k_stride_n = kb.data_ptr(), kb.stride(0), kb.stride(1)
        a.v, a.v_stride_h, a.v_stride_n = vb.data_ptr(), vb.stride(0), vb.stride(1)
        a.out = out[b].data_ptr()
        a.dtype = dtype_code(q.dtype)
        a.batch, a.n_heads, a.n_kv_heads, a.n, a.d = 1, H, Hk, N, D
        a.tau = tau_d.data_ptr()
        a.inv_freq_a, a.pos_scale_a, a.rope_scale_a = ia.data_ptr(), float(ga.pos_scale), float(ga.rope_scale)
        a.inv_freq_c, a.pos_scale_c, a.rope_scale_c = ic.data_ptr(), float(gc.pos_scale), float(gc.rope_scale)
        a.sm_scale = float(sm_scale)
        a.pct = float(pct)
        a.n_global, a.n_local, a.tile, a.k_max = int(n_global), int(n_local), T, int(k_max or 0)
        a.select_score = L.SCORE[select_score]
        a.measure = int(bool(measure))
        a.block_n = int(block_n)
        a.pos_advance = L.ADV[pos_advance]
        a.use_skip = int(bool(use_skip))
        if variant == "shared":
            a.shared_size = st["shared_size"][b].data_ptr()
            a.kept_size = st["kept_size"][b].data_ptr()
            a.chosen = st["chosen"][b].data_ptr()
            a.overflow = st["overflow"][b].data_ptr()
            a.kpct_meas = st["kpct_meas"][b].data_ptr()
            a.overflow20 = st["overflow20"][b].data_ptr()
        elif variant == "pq_union":
            a.shared_size = st["usize"][b].data_ptr()
            a.kept_size = st["kept_size"][b].data_ptr()
            a.overflow = st["overflow"][b].data_ptr()
        elif variant == "chunk":
            a.shared_size = st["usize"][b].data_ptr()
            a.kept_size = st["kept_size"][b].data_ptr()
            a.chunk_size, a.n_chunk = int(chunk_size), int(n_chunk)
            a.chunk_agg = {"sum": 0, "mean": 1}[chunk_agg]
        else:
            a.span = st["span"][b].data_ptr()
            a.kept_rows = st["kept"][b].data_ptr()
            a.blocks = st["blocks"][b].data_ptr()
            a.skipped = st["skipped"][b].data_ptr()
        if sets:
            a.idx_out = sets["idx"][b].data_ptr()
            a.newpos_k_out = sets["newpos_k"][b].data_ptr()
            a.newpos_q_out = sets["newpos_q"][b].data_ptr()
            if "mask" in sets:
                a.mask_out = sets["mask"][b].data_ptr()
        a.max_workspace_bytes = int(max_workspace_bytes)
        a.same_geometry = same_geometry
        a.q_pos_base = q_pos_base
        if ga.dca is not None:
            a.dca_chunk_size, a.dca_local_window = int(ga.dca[0]), int(ga.dca[1])
        if stage_events is not None:
            arr = (ctypes.c_void_p * len(stage_events))(*[e.cuda_event for e in stage_events])
            a.stage_events = ctypes.cast(arr, ctypes.c_void_p)
        nbytes = fn_ws(ctypes.byref(a))
        if nbytes == 0:
            L.check(1, f"sta_{variant}_workspace_bytes")
        if b == 0 and stage_events is not None:
            # the stage events bracket the last group of kv heads: report the group count
            cap = a.max_workspace_bytes
            a.max_workspace_bytes = 0
            full = fn_ws(ctypes.byref(a))
            a.max_workspace_bytes = cap
            groups = max(1, round(full / nbytes))
            while Hk % groups:
                groups += 1
            st["kv_head_groups"] = groups
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        L.check(fn(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()),
                   stream), f"sta_{variant}_forward")
    return out, st, sets


# -------------------------------------------------------------------------------------------
# stage-level access (used by the parity tests to compare intermediates with the oracle)
# -------------------------------------------------------------------------------------------
def forward_host(variant: str, q, k, v, tau, ga: Geometry, gc: Geometry, *, groups=4,
                 device=None, **kw):
    """The op on HOST tensors, with the transfers overlapped with the compute.

    q (Z,H,N,D), k / v (Z,Hkv,N,D) in pinned host memory (a copy is made otherwise).  The kv
    heads (the q heads when Hkv is 1) are cut into ``groups`` equal groups (the largest divisor
    not above it), or into groups of the listed counts (small first and last groups shorten the
    transfer that nothing overlaps: the first group's input and the last group's output): group
    g+1 is copied host -> device on one stream while group g computes on the current stream,
    and each group's output is copied back on a third stream as soon as it is done.  Every
    stage is independent per kv head, so the result equals one device call on the whole input.
    Returns (out (Z,H,Nq,D) pinned host tensor, statistics on the device); the caller
    synchronises (e.g. ``torch.cuda.current_stream().synchronize()``) before reading ``out``."""
    for x in (q, k, v):
        if x.is_cuda:
            raise ValueError("forward_host takes host tensors; use forward for device tensors")
    q, k, v = (x if x.is_pinned() else x.pin_memory() for x in (q, k, v))
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    Z, H, Nq, D = q.shape
    Hk = k.shape[1]
    if H % Hk:
        raise ValueError("number of q heads must be a multiple of the number of kv heads")
    G = H // Hk
    # group units: kv heads, or q heads when there is a single kv head (its k / v go first)
    units = Hk if Hk > 1 else H
    if isinstance(groups, (list, tuple)):
        sizes = [int(x) for x in groups]
        if sum(sizes) != units or min(sizes) < 1:
            raise ValueError(f"group sizes {sizes} must be positive and sum to {units}")
    else:
        ng = max(1, min(int(groups), units))
        while units % ng:
            ng -= 1
        sizes = [units // ng] * ng
    bounds = [0]
    for x in sizes:
        bounds.append(bounds[-1] + x)
    ng = len(sizes)
    if Hk > 1:
        qsl = [slice(bounds[g] * G, bounds[g + 1] * G) for g in range(ng)]
        ksl = [slice(bounds[g], bounds[g + 1]) for g in range(ng)]
    else:
        qsl = [slice(bounds[g], bounds[g + 1]) for g in range(ng)]
        ksl = [slice(0, 1)] * ng
    qd = torch.empty(q.shape, dtype=q.dtype, device=dev)
    kd = torch.empty(k.shape, dtype=k.dtype, device=dev)
    vd = torch.empty(v.shape, dtype=v.dtype, device=dev)
    out_h = torch.empty((Z, H, Nq, D), dtype=q.dtype, pin_memory=True)
    comp = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    s_in.wait_stream(comp)   # device buffers were allocated on the current stream
    s_out.wait_stream(comp)
    ev_in = []
    with torch.cuda.stream(s_in):
        for g in range(ng):
            hs, ks = qsl[g], ksl[g]
            for b in range(Z):  # per batch element: contiguous slices, one DMA each
                if Hk > 1 or g == 0:
                    kd[b, ks].copy_(k[b, ks], non_blocking=True)
                    vd[b, ks].copy_(v[b, ks], non_blocking=True)
                qd[b, hs].copy_(q[b, hs], non_blocking=True)
            e = torch.cuda.Event()
            e.record(s_in)
            ev_in.append(e)
    tau_h = torch.as_tensor(tau, dtype=torch.float32).reshape(-1)
    stats = []
    for g in range(ng):
        hs, ks = qsl[g], ksl[g]
        comp.wait_event(ev_in[g])
        o, st, _ = forward(variant, qd[:, hs], kd[:, ks], vd[:, ks], tau_h[hs], ga, gc, **kw)
        stats.append(st)
        done = torch.cuda.Event()
        done.record(comp)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            for b in range(Z):
                out_h[b, hs].copy_(o[b], non_blocking=True)
        o.record_stream(s_out)
    for x in (qd, kd, vd):
        x.record_stream(s_in)
    comp.wait_stream(s_out)  # the caller's stream orders after the last copy back
    st = {name: torch.cat([sg[name] for sg in stats], dim=1) for name in stats[0]
          if torch.is_tensor(stats[0][name])}
    return out_h, st


_TABLES = {}


def _rope_table(inv_freq: torch.Tensor, rope_scale: float, R: float, length: int, src=None):
    """Cached (cos, sin) * rope_scale table at positions i / R, 0 <= i < length (sta_rope_table),
    keyed by the frequencies' VALUES; grown by doubling so that a decode loop builds it
    O(log n) times.  inv_freq: fp32 on the target device; src: the same values where they are
    already on the host (saves a device-to-host read for the key)."""
    vals = (src if src is not None and not src.is_cuda else inv_freq).detach().float().cpu()
    key = (inv_freq.device, vals.numpy().tobytes(), float(rope_scale), float(R))
    t = _TABLES.get(key)
    if t is None or t[1] < length:
        cap = max(length, 2 * (t[1] if t else 0), 1024)
        half = inv_freq.numel()
        buf = torch.empty((cap, half, 2), dtype=torch.float32, device=inv_freq.device)
        freq = inv_freq.detach().clone()
        L.check(L.lib().sta_rope_table(_p(freq), 2 * half, float(rope_scale), float(R), cap,
                                       _p(buf), _stream()), "sta_rope_table")
        t = (buf, cap)
        _TABLES[key] = t
    return t[0], t[1]


def _table_R(pos_scale):
    for r in (1, 2, 4):
        if float(pos_scale) * r == 1.0:
            return float(r)
    return 0.0


def decode(mode: str, q, k, v, tau, ga: Geometry, gc: Geometry, *, n_global=32, n_local=32,
           k_max=1024, pct_decode=100.0, block_n=32, sm_scale=None, keep_sets=False,
           chunk_size=16, n_chunk=0, chunk_agg="sum", select_score="expmass"):
    """One decode step: the query at position m-1 of every head against the cache.

    mode: 'pi' (shared hooks: threshold + optional top-pct + forced + tie-inclusive k_max cap by
    score + PI reposition, shared_selection_triton_exact.py:464-560), 'rank' (PQ-Union:
    exact-budget cap, dense ranks, perquery.py:652-740), 'stream' (PQ-Stream: no cap, streamed
    positions, pqstream_kernel.py:694-795) or 'chunk' (chunk_exact: forced + top n_chunk chunks,
    dense ranks, shared_selection_triton_chunked.py:412-483).  q (Z,H,D); k, v (Z,Hkv,m,D) raw cache (GQA-native).
    ga: selection geometry; gc: attend geometry (pos_scale_c repositions in 'pi').
    Returns (out (Z,H,D), stats {kept, usize} (Z,H) [+ sets idx / newpos_k / newpos_q])."""
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("q, k, v must be CUDA tensors (there is no CPU path)")
    if q.dim() != 3 or k.dim() != 4 or v.shape != k.shape:
        raise ValueError("decode expects q (Z,H,D) and k, v (Z,Hkv,m,D)")
    Z, H, D = q.shape
    Hk, M = k.shape[1], k.shape[2]
    if H % Hk or k.shape[0] != Z or k.shape[3] != D:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share one dtype")
    dev = q.device
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    md = L.DECODE[mode]
    tau_d = _dev_f32(tau, dev).reshape(-1)
    if tau_d.numel() != H:
        raise ValueError(f"tau must have one entry per q head ({H})")
    ia, ic = _dev_f32(ga.inv_freq, dev), _dev_f32(gc.inv_freq, dev)
    rs_c = float(gc.rope_scale) if mode == "pi" else 1.0
    qr = q if q.stride(-1) == 1 and q.stride(0) == H * q.stride(1) else q.contiguous()
    kr = k if k.stride(-1) == 1 else k.contiguous()
    vr = v if v.stride(-1) == 1 else v.contiguous()
    if kr.stride(0) != Hk * kr.stride(1) or vr.stride(0) != Hk * vr.stride(1):
        kr, vr = kr.contiguous(), vr.contiguous()
    out = torch.empty((Z, H, D), dtype=q.dtype, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    st = {"kept": torch.empty((Z, H), **i32), "usize": torch.empty((Z, H), **i32)}
    cap = M if mode == "stream" else int(k_max)
    sets = {}
    if keep_sets:
        sets = {"idx": torch.empty((Z, H, cap), **i32),
                "newpos_k": torch.empty((Z, H, cap), dtype=torch.float32, device=dev),
                "newpos_q": torch.empty((Z, H), dtype=torch.float32, device=dev)}
    a = L.DecodeArgs()
    a.q, a.q_stride_h = qr.data_ptr(), qr.stride(1)
    a.k, a.k_stride_h, a.k_stride_n = kr.data_ptr(), kr.stride(1), kr.stride(2)
    a.v, a.v_stride_h, a.v_stride_n = vr.data_ptr(), vr.stride(1), vr.stride(2)
    a.out = out.data_ptr()
    a.dtype = dtype_code(q.dtype)
    a.batch, a.n_heads, a.n_kv_heads, a.m, a.d = Z, H, Hk, M, D
    a.tau = tau_d.data_ptr()
    a.inv_freq_a, a.pos_scale_a, a.rope_scale_a = ia.data_ptr(), float(ga.pos_scale), float(ga.rope_scale)
    a.inv_freq_c, a.pos_scale_c, a.rope_scale_c = ic.data_ptr(), float(gc.pos_scale), rs_c
    a.sm_scale = float(sm_scale)
    a.mode = md
    a.n_global, a.n_local, a.k_max = int(n_global), int(n_local), int(k_max or 0)
    a.pct_decode, a.block_n = float(pct_decode), int(block_n)
    Ra = _table_R(ga.pos_scale)
    if Ra:
        ta, la = _rope_table(ia, float(ga.rope_scale), Ra, int(M * Ra) + 1, src=ga.inv_freq)
        a.rope_table_a, a.rope_table_a_R, a.rope_table_a_len = ta.data_ptr(), Ra, la
    a.chunk_size, a.n_chunk = int(chunk_size), int(n_chunk)
    a.chunk_agg = {"sum": 0, "mean": 1}[chunk_agg]
    a.select_score = L.SCORE[select_score]
    Rc = {"pi": _table_R(gc.pos_scale), "rank": 1.0, "stream": -1.0, "chunk": 1.0}[mode]
    if Rc:
        tc, lc = _rope_table(ic, rs_c, Rc, int(M * abs(Rc)) + 1, src=gc.inv_freq)
        a.rope_table_c, a.rope_table_c_R, a.rope_table_c_len = tc.data_ptr(), Rc, lc
    a.kept_out, a.usize_out = st["kept"].data_ptr(), st["usize"].data_ptr()
    if sets:
        a.idx_out, a.newpos_k_out = sets["idx"].data_ptr(), sets["newpos_k"].data_ptr()
        a.newpos_q_out = sets["newpos_q"].data_ptr()
    nbytes = L.lib().sta_decode_workspace_bytes(ctypes.byref(a))
    if nbytes == 0:
        L.check(1, "sta_decode_workspace_bytes")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    L.check(L.lib().sta_decode_forward(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()),
                                       ctypes.c_size_t(nbytes), _stream()), "sta_decode_forward")
    return out, st, sets


def rope_split(x: torch.Tensor, g: Geometry):
    """x (heads, n, d) -> (hi, lo) bf16 rotated at the selection geometry."""
    x = _rows(x)
    Hx, N, D = x.shape
    hi = torch.empty((Hx, N, D), dtype=torch.bfloat16, device=x.device)
    lo = torch.empty_like(hi)
    invf = _dev_f32(g.inv_freq, x.device)
    L.check(L.lib().sta_rope_split(_p(x), dtype_code(x.dtype), Hx, N, D, x.stride(0),
                                   x.stride(1), _p(invf), float(g.pos_scale),
                                   float(g.rope_scale), _p(hi), _p(lo), _stream()),
            "sta_rope_split")
    return hi, lo


def tri_head_stride(n: int, tile: int) -> int:
    return int(L.lib().sta_tri_head_stride(n, tile))


def rope_split_dca(x: torch.Tensor, g: Geometry, role: int, out_hi=None, out_lo=None):
    """x (heads, n, d) -> (hi, lo) bf16 rotated at Dual Chunk Attention position role
    (1 keys / same-chunk queries, 2 previous-chunk queries, 3 older-chunk queries)."""
    x = _rows(x)
    Hx, N, D = x.shape
    hi = out_hi if out_hi is not None else torch.empty((Hx, N, D), dtype=torch.bfloat16,
                                                       device=x.device)
    lo = out_lo if out_lo is not None else torch.empty_like(hi)
    invf = _dev_f32(g.inv_freq, x.device)
    L.check(L.lib().sta_rope_split_dca(_p(x), dtype_code(x.dtype), Hx, N, D, x.stride(0),
                                       x.stride(1), _p(invf), float(g.rope_scale),
                                       int(g.dca[0]), int(g.dca[1]), int(role), _p(hi), _p(lo),
                                       _stream()), "sta_rope_split_dca")
    return hi, lo


def select(q: torch.Tensor, k: torch.Tensor, tau, g: Geometry, *, tile, sm_scale=None,
           wmode=0, bits=False, max_only=False, wait_limit_ns=0, screen=False,
           vote_hist=False):
    """Kernel A on raw (H,N,D) q and (Hkv,N,D) k.  Returns dict of compact votes / wvotes /
    bits, row_max (H,N) and row_count (H,N).  `wait_limit_ns` bounds every device-side wait
    (0: the library default); an expired wait shows in device_error(), not here.  With
    ``g.dca`` the selection geometry is Dual Chunk Attention (three rotated query planes).
    ``screen`` (unweighted modes) scores with one fp16 product per pair and exact rescoring of
    the pairs a proven bound leaves undecided (the forward entry points do so under
    ``STA_SELECT_SCREEN=1``); the default scores every pair with three bf16 products.
    ``vote_hist`` (tile 64 / 128) also returns each tile's histogram of nonzero votes."""
    H, N, D = q.shape
    Hk = k.shape[0]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    dca_len = 0
    if g.dca is None:
        qh, ql = rope_split(q, g)
        kh, kl = rope_split(k, g)
    else:
        qh = torch.empty((3, H, N, D), dtype=torch.bfloat16, device=q.device)
        ql = torch.empty_like(qh)
        for role in (1, 2, 3):
            rope_split_dca(q, g, role, qh[role - 1], ql[role - 1])
        kh, kl = rope_split_dca(k, g, 1)
        dca_len = int(g.dca[0]) - int(g.dca[1])
    HS = tri_head_stride(N, tile)
    dev = q.device
    res = {"row_max": torch.empty((H, N), dtype=torch.float32, device=dev),
           "row_count": torch.empty((H, N), dtype=torch.int32, device=dev)}
    if not max_only:
        res["votes"] = torch.empty((H * HS,), dtype=torch.uint8, device=dev)
        if wmode:
            res["wvotes"] = torch.empty((H * HS,), dtype=torch.float32, device=dev)
        if bits:
            res["bits"] = torch.empty((H * HS,), dtype=torch.int32, device=dev)
    tau_d = _dev_f32(tau, dev)
    a = L.SelectArgs()
    a.q_hi, a.q_lo, a.k_hi, a.k_lo = qh.data_ptr(), ql.data_ptr(), kh.data_ptr(), kl.data_ptr()
    a.batch, a.n_heads, a.n_kv_heads, a.n, a.d, a.tile = 1, H, Hk, N, D, tile
    a.sm_scale = float(sm_scale)
    a.wmode = int(wmode)
    a.tau = tau_d.data_ptr()
    a.max_only = int(bool(max_only))
    a.votes = res["votes"].data_ptr() if "votes" in res else None
    a.wvotes = res["wvotes"].data_ptr() if "wvotes" in res else None
    a.bits = res["bits"].data_ptr() if "bits" in res else None
    a.row_max = res["row_max"].data_ptr()
    a.row_count = res["row_count"].data_ptr()
    a.dca_chunk_len = dca_len
    a.wait_limit_ns = int(wait_limit_ns)
    if vote_hist and not max_only and tile != 32:
        res["vote_hist"] = torch.zeros((H, (N + tile - 1) // tile, tile + 1), dtype=torch.int32,
                                       device=dev)
        a.vote_hist = res["vote_hist"].data_ptr()
    scr = None
    if screen and not wmode:
        nb = int(L.lib().sta_select_screen_bytes(ctypes.byref(a)))
        scr = torch.empty((nb,), dtype=torch.uint8, device=dev)
        a.screen_ws = scr.data_ptr()
    L.check(L.lib().sta_select(ctypes.byref(a), _stream()), "sta_select")
    del scr  # freed after the launch: torch's caching allocator keeps stream order
    return res


def expand_compact(flat: torch.Tensor, H: int, N: int, tile: int, fill=0):
    """compact (H*HS,) per-(head, tile) array -> dense (H, nt, N) (small sizes only)."""
    HS = tri_head_stride(N, tile)
    nt = (N + tile - 1) // tile
    x = flat.reshape(H, HS)
    out = torch.full((H, nt, N), fill, dtype=flat.dtype, device=flat.device)
    for t in range(nt):
        hi = min((t + 1) * tile, N)
        o = tile * t * (t + 1) // 2
        out[:, t, :hi] = x[:, o:o + hi]
    return out


def compact_from_dense(dense: torch.Tensor, tile: int):
    """dense (H, nt, N) -> compact (H*HS,) (inverse of expand_compact)."""
    H, nt, N = dense.shape
    parts = []
    for h in range(H):
        for t in range(nt):
            parts.append(dense[h, t, :min((t + 1) * tile, N)])
    return torch.cat(parts).contiguous()


def dca_dense(q, k, v, inv_freq, *, chunk_size, local_window, rope_scale=1.0, sm_scale=None,
              q_pos_base=0):
    """Dense Dual Chunk Attention prefill (sta_dca_forward): q (Z,H,Nq,D), k / v (Z,Hkv,N,D)
    raw, Nq = N - q_pos_base.  chunk_size == 0: plain causal attention with RoPE at the true
    positions.  Returns out (Z,H,Nq,D) in q's dtype."""
    q_pos_base = int(q_pos_base)
    Z, H, Hk, N, D = _check_inputs(q, k, v, q_pos_base)
    dev = q.device
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    invf = _dev_f32(inv_freq, dev)
    if invf.numel() != D // 2:
        raise ValueError("inv_freq must have head_dim/2 entries")
    out = torch.empty((Z, H, N - q_pos_base, D), dtype=q.dtype, device=dev)
    lib = L.lib()
    ws = None
    for b in range(Z):
        qb, kb, vb = _rows(q[b]), _rows(k[b]), _rows(v[b])
        a = L.DcaArgs()
        a.q, a.q_stride_h, a.q_stride_n = qb.data_ptr(), qb.stride(0), qb.stride(1)
        a.k, a.k_stride_h, a.k_stride_n = kb.data_ptr(), kb.stride(0), kb.stride(1)
        a.v, a.v_stride_h, a.v_stride_n = vb.data_ptr(), vb.stride(0), vb.stride(1)
        a.out = out[b].data_ptr()
        a.dtype = dtype_code(q.dtype)
        a.batch, a.n_heads, a.n_kv_heads, a.n, a.d = 1, H, Hk, N, D
        a.inv_freq = invf.data_ptr()
        a.rope_scale, a.sm_scale = float(rope_scale), float(sm_scale)
        a.chunk_size, a.local_window = int(chunk_size), int(local_window)
        a.q_pos_base = q_pos_base
        nbytes = lib.sta_dca_workspace_bytes(ctypes.byref(a))
        if nbytes == 0:
            L.check(1, "sta_dca_workspace_bytes")
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        L.check(lib.sta_dca_forward(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()),
                                    ctypes.c_size_t(ws.numel()), _stream()), "sta_dca_forward")
    return out


def device_error() -> int:
    """Synchronise the current stream and return (and clear) the device error word of the
    bounded waits: 0 when no wait expired since the last read."""
    code = L.c_i32(0)
    L.lib().sta_device_error(_stream(), ctypes.byref(code))
    return int(code.value)


def build_sets(votes_c, wvotes_c, H, N, *, tile, k_max, n_global=32, n_local=32, pct=30.0,
               pos_scale=1.0, select_score="freq", measure=False):
    """Stage 2 on compact votes (uint8) / wvotes (f32).  Returns the reference's 9 outputs."""
    dev = votes_c.device
    nt = (N + tile - 1) // tile
    i32 = dict(dtype=torch.int32, device=dev)
    o = dict(idx=torch.empty((H, nt, k_max), **i32),
             newpos_k=torch.empty((H, nt, k_max), dtype=torch.float32, device=dev),
             newpos_q=torch.empty((H, nt, tile), dtype=torch.float32, device=dev),
             shared_size=torch.empty((H, nt), **i32), kept_size=torch.empty((H, nt), **i32),
             chosen=torch.empty((H, nt), **i32),
             overflow=torch.empty((H, nt), dtype=torch.uint8, device=dev),
             kpct_meas=torch.empty((H, nt), **i32),
             overflow20=torch.empty((H, nt), dtype=torch.uint8, device=dev))
    a = L.BuildArgs()
    a.votes = votes_c.data_ptr()
    a.wvotes = wvotes_c.data_ptr() if wvotes_c is not None else None
    a.heads, a.n, a.tile, a.k_max = H, N, tile, k_max
    a.n_global, a.n_local, a.pct, a.pos_scale = n_global, n_local, float(pct), float(pos_scale)
    a.select_score = L.SCORE[select_score]
    a.measure = int(bool(measure))
    for name in ("idx", "newpos_k", "newpos_q", "shared_size", "kept_size", "chosen",
                 "overflow", "kpct_meas", "overflow20"):
        setattr(a, name, o[name].data_ptr())
    L.check(L.lib().sta_build_sets(ctypes.byref(a), _stream()), "sta_build_sets")
    return o


def build_sets_pq(votes_c, wvotes_c, bits_c, H, N, *, k_max, n_global=32, n_local=32,
                  select_score="expmass"):
    dev = votes_c.device
    T = 32
    nt = (N + T - 1) // T
    i32 = dict(dtype=torch.int32, device=dev)
    o = dict(idx=torch.empty((H, nt, k_max), **i32),
             newpos_k=torch.empty((H, nt, k_max), dtype=torch.float32, device=dev),
             newpos_q=torch.empty((H, nt, T), dtype=torch.float32, device=dev),
             mask=torch.empty((H, nt, k_max), **i32), usize=torch.empty((H, nt), **i32),
             kept_size=torch.empty((H, nt), **i32),
             overflow=torch.empty((H, nt), dtype=torch.uint8, device=dev))
    a = L.BuildPQArgs()
    a.votes = votes_c.data_ptr()
    a.wvotes = wvotes_c.data_ptr() if wvotes_c is not None else None
    a.bits = bits_c.data_ptr()
    a.heads, a.n, a.tile, a.k_max = H, N, T, k_max
    a.n_global, a.n_local = n_global, n_local
    a.select_score = L.SCORE[select_score]
    for name in ("idx", "newpos_k", "newpos_q", "mask", "usize", "kept_size", "overflow"):
        setattr(a, name, o[name].data_ptr())
    L.check(L.lib().sta_build_sets_pq(ctypes.byref(a), _stream()), "sta_build_sets_pq")
    return o


def gather_attend(q, k, v, idx, newpos_k, newpos_q, g: Geometry, *, tile, sm_scale=None,
                  mask=None, kept_size=None):
    """Stage 3 on raw (H,N,D) q and (Hkv,N,D) k, v with (H,nt,k_max) slot arrays."""
    q, k, v = _rows(q), _rows(k), _rows(v)
    H, N, D = q.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    out = torch.empty((H, N, D), dtype=q.dtype, device=q.device)
    invf = _dev_f32(g.inv_freq, q.device)
    a = L.AttendArgs()
    a.q, a.q_stride_h, a.q_stride_n = q.data_ptr(), q.stride(0), q.stride(1)
    a.k, a.k_stride_h, a.k_stride_n = k.data_ptr(), k.stride(0), k.stride(1)
    a.v, a.v_stride_h, a.v_stride_n = v.data_ptr(), v.stride(0), v.stride(1)
    a.out = out.data_ptr()
    a.dtype = dtype_code(q.dtype)
    a.batch, a.n_heads, a.n_kv_heads, a.n, a.d = 1, H, k.shape[0], N, D
    a.tile, a.k_max = tile, idx.shape[-1]
    idx = idx.to(torch.int32).contiguous()
    newpos_k = newpos_k.float().contiguous()
    newpos_q = newpos_q.float().contiguous()
    a.idx, a.newpos_k, a.newpos_q = idx.data_ptr(), newpos_k.data_ptr(), newpos_q.data_ptr()
    if mask is not None:
        mask = mask.to(torch.int32).contiguous()
        a.mask = mask.data_ptr()
    if kept_size is not None:
        kept_size = kept_size.to(torch.int32).contiguous()
        a.kept_size = kept_size.data_ptr()
    a.inv_freq = invf.data_ptr()
    a.rope_scale = float(g.rope_scale)
    a.sm_scale = float(sm_scale)
    L.check(L.lib().sta_gather_attend(ctypes.byref(a), _stream()), "sta_gather_attend")
    return out


def build_sets_chunk(votes_c, wvotes_c, H, N, *, k_max, chunk_size=16, n_chunk, tile=32,
                     n_global=32, n_local=32, select_score="expmass", chunk_agg="sum"):
    dev = votes_c.device
    T = tile
    nt = (N + T - 1) // T
    i32 = dict(dtype=torch.int32, device=dev)
    o = dict(idx=torch.empty((H, nt, k_max), **i32),
             newpos_k=torch.empty((H, nt, k_max), dtype=torch.float32, device=dev),
             newpos_q=torch.empty((H, nt, T), dtype=torch.float32, device=dev),
             mask=torch.empty((H, nt, k_max), **i32), usize=torch.empty((H, nt), **i32),
             kept_size=torch.empty((H, nt), **i32))
    a = L.BuildChunkArgs()
    a.votes = votes_c.data_ptr()
    a.wvotes = wvotes_c.data_ptr() if wvotes_c is not None else None
    a.heads, a.n, a.tile, a.k_max = H, N, T, k_max
    a.n_global, a.n_local, a.chunk_size, a.n_chunk = n_global, n_local, chunk_size, n_chunk
    a.select_score = L.SCORE[select_score]
    a.chunk_agg = {"sum": 0, "mean": 1}[chunk_agg]
    for name in ("idx", "newpos_k", "newpos_q", "mask", "usize", "kept_size"):
        setattr(a, name, o[name].data_ptr())
    L.check(L.lib().sta_build_sets_chunk(ctypes.byref(a), _stream()), "sta_build_sets_chunk")
    return o
