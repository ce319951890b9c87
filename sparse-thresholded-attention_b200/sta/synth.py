"""Seeded synthetic prefill inputs for the thresholded-attention benchmark configs.

The reference was evaluated on RULER / LongBench / PG-19 with real Llama weights and a
calibrated per-head tau table (run_ruler.py:25, :128-133); none of that exists here.  These
generators stand in for it with the shapes and value structure the benchmark configs name:

* q, k, v ~ N(0, 1);
* a shared rank-16 component U @ V (per kv head, element std 2.0) added to q and k, which
  makes scores structured (many keys pass a tau=5 threshold for some queries);
* ``n_planted`` planted keys per kv head at distinct uniform positions.  Each planted key is
  set to ``mean_key_norm * u`` for a random unit direction u, and for 64 random *later*
  queries of every q head in the group the query is replaced by
  ``|q| * (0.8 u + 0.6 u_perp)`` (cosine 0.8 with the key before RoPE).

All randomness comes from one ``torch.Generator`` seeded with ``seed`` and runs on the CPU in
fp32; the result is cast to ``dtype`` at the end, so the same seed gives the same tensors on
every machine.  Nothing here reproduces any item of the reference's evaluation suites.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class SynthSpec:
    batch: int = 1
    n_heads: int = 4          # q heads
    n_kv_heads: int = 4       # k / v heads (GQA when < n_heads)
    seq_len: int = 1024
    head_dim: int = 64
    n_planted: int = 32       # planted keys per kv head
    n_planted_queries: int = 64
    rank: int = 16
    rank_std: float = 2.0
    cosine: float = 0.8
    seed: int = 0
    dtype: torch.dtype = torch.float32
    # optional "dense clusters": scale the queries of these ranges towards zero so that they keep
    # many causal keys (drives the 30->25->20% fallback).  Entries are (batch, start, length)
    # -- every row scaled by ``flat_scale``, so all rows keep nearly every causal key and the
    # votes tie -- or (batch, start, length, lo, hi): row r scaled by the geometric ramp
    # lo * (hi/lo)^(r/(length-1)), which grades the votes so a 25% or 20% pick can fit k_max
    flat_query_ranges: list = field(default_factory=list)
    flat_scale: float = 0.02


def make_inputs(spec: SynthSpec):
    """Return (q, k, v) of shapes (B, H, S, D), (B, Hkv, S, D), (B, Hkv, S, D)."""
    g = torch.Generator().manual_seed(int(spec.seed))
    B, H, Hk, S, D = spec.batch, spec.n_heads, spec.n_kv_heads, spec.seq_len, spec.head_dim
    assert H % Hk == 0, "q heads must be a multiple of kv heads"
    G = H // Hk
    q = torch.randn((B, H, S, D), generator=g)
    k = torch.randn((B, Hk, S, D), generator=g)
    v = torch.randn((B, Hk, S, D), generator=g)
    sv = spec.rank_std / math.sqrt(spec.rank)
    for b in range(B):
        for kh in range(Hk):
            U = torch.randn((S, spec.rank), generator=g)
            V = torch.randn((spec.rank, D), generator=g) * sv
            comp = U @ V
            k[b, kh] += comp
            q[b, kh * G:(kh + 1) * G] += comp[None]
    mean_knorm = float(k.norm(dim=-1).mean())
    P = min(spec.n_planted, max(S - 1, 0))
    for b in range(B):
        for kh in range(Hk):
            if P == 0:
                continue
            # planted positions: distinct, and not the very last position (they need later queries)
            pos = torch.randperm(S - 1, generator=g)[:P]
            for p in pos.tolist():
                u = torch.randn((D,), generator=g)
                u = u / u.norm()
                k[b, kh, p] = mean_knorm * u
                n_later = S - 1 - p
                nq = min(spec.n_planted_queries, n_later)
                for h in range(kh * G, (kh + 1) * G):
                    # random later queries (drawn with replacement, then de-duplicated so the
                    # scatter below is deterministic)
                    later = torch.unique(torch.randint(p + 1, S, (nq,), generator=g))
                    w = torch.randn((nq, D), generator=g)[:later.numel()]
                    w = w - (w @ u)[:, None] * u[None, :]
                    w = w / w.norm(dim=-1, keepdim=True).clamp_min(1e-12)
                    qn = q[b, h, later].norm(dim=-1, keepdim=True)
                    q[b, h, later] = qn * (spec.cosine * u[None, :]
                                           + math.sqrt(1.0 - spec.cosine ** 2) * w)
    for rng in spec.flat_query_ranges:
        b, start, length = rng[:3]
        if len(rng) == 3:
            q[b, :, start:start + length] *= spec.flat_scale
        else:
            lo, hi = float(rng[3]), float(rng[4])
            r = torch.arange(length, dtype=torch.float32) / max(length - 1, 1)
            ramp = lo * (hi / lo) ** r
            q[b, :, start:start + length] *= ramp[None, :, None]
    return q.to(spec.dtype), k.to(spec.dtype), v.to(spec.dtype)


def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """Base RoPE frequencies theta^(-2i/D), fp32, as the reference hooks compute them
    (shared_selection_triton_hybrid_exact.py:716, shared_selection_triton_perquery.py:813)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))


def yarn_inv_freq(head_dim: int, theta: float, factor: float, original_max: int,
                  beta_fast: float = 32.0, beta_slow: float = 1.0):
    """YaRN NTK-by-parts frequencies and attention factor (mscale), computed by the installed
    transformers ``ROPE_INIT_FUNCTIONS['yarn']`` -- the same third-party routine the reference
    hooks read through ``model.model.rotary_emb`` (shared_selection_triton_YaRN_exact.py:681-690).
    Returns (inv_freq fp32 (D/2,), attention_factor float)."""
    from transformers import LlamaConfig
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
    cfg = LlamaConfig(hidden_size=head_dim * 2, num_attention_heads=2, head_dim=head_dim,
                      max_position_embeddings=int(original_max * factor),
                      rope_parameters={"rope_type": "yarn", "rope_theta": float(theta),
                                       "factor": float(factor),
                                       "original_max_position_embeddings": int(original_max),
                                       "beta_fast": float(beta_fast),
                                       "beta_slow": float(beta_slow)})
    inv, att = ROPE_INIT_FUNCTIONS["yarn"](cfg, "cpu")
    return inv.float(), float(att)


# ---------------------------------------------------------------------------------------------
# The benchmark configurations (shapes, seeds, geometry) as plain dictionaries.
# ---------------------------------------------------------------------------------------------
def config(idx: int) -> dict:
    """Shapes and geometry of benchmark config ``idx`` (0..4)."""
    if idx == 0:
        return dict(name="cfg0-cpu-plumbing", B=1, H=4, Hkv=4, S=1024, D=64, dtype="f32", T=64,
                    planted=32, seed=0, theta=1e4, geom="pi", pos_scale=1.0, rope_scale=1.0,
                    tau=5.0, pct=30.0, k_max=2048)
    if idx == 1:
        return dict(name="cfg1-llama2-7b-pi-8k", B=1, H=32, Hkv=32, S=8192, D=128, dtype="bf16",
                    T=64, planted=256, seed=1, theta=1e4, geom="pi", pos_scale=0.5,
                    rope_scale=1.0, tau=5.0, pct=30.0, k_max=2048)
    if idx == 2:
        return dict(name="cfg2-llama3-8b-gqa-yarn-32k", B=1, H=32, Hkv=8, S=32768, D=128,
                    dtype="bf16", T=64, planted=1024, seed=2, theta=5e5, geom="yarn",
                    yarn_factor=4.0, yarn_orig=8192, pos_scale=1.0, tau=5.0, pct=30.0,
                    k_max=2048)
    if idx == 3:
        return dict(name="cfg3-hybrid-dca-64k", B=2, H=32, Hkv=8, S=65536, D=128, dtype="bf16",
                    T=64, planted=1024, seed=3, theta=5e5, geom="hybrid", pos_scale_c=0.5,
                    dca_chunk_size=6144, dca_local_window=1024, dca_pretrain=8192,
                    tau=5.0, pct=30.0, k_max=2048)
    if idx == 4:
        return dict(name="cfg4-pq-128k", B=1, H=32, Hkv=8, S=131072, D=128, dtype="bf16", T=32,
                    planted=4096, seed=4, theta=5e5, geom="yarn", yarn_factor=16.0,
                    yarn_orig=8192, pos_scale=1.0, tau=5.0, k_max=2048)
    raise ValueError(idx)


def make_config_inputs(idx: int, seq_len: int | None = None, n_heads: int | None = None,
                       n_kv_heads: int | None = None, batch: int | None = None):
    """Inputs of config ``idx``, optionally shrunk (for parity tests at sizes the oracle
    finishes in seconds).  Returns (q, k, v, cfg)."""
    c = config(idx)
    S = seq_len or c["S"]
    H = n_heads or c["H"]
    Hk = n_kv_heads or (c["Hkv"] if n_heads is None else max(1, H * c["Hkv"] // c["H"]))
    B = batch or c["B"]
    planted = max(1, c["planted"] * S // c["S"])
    flat = []
    if idx == 2 and S >= 8192:
        # dense clusters that exercise the 30->25->20% fallback: two graded tiles (query tiles
        # 80 and 100: the 25% and 20% picks fit k_max on some heads, unresolved on others) and
        # one flat tile half-way (every pick overflows: unresolved, keeps the 20% set)
        T = c["T"]
        flat = [(0, 80 * T, T, 0.02, 1.0), (0, 100 * T, T, 0.02, 1.0),
                (0, (S // 2 // T) * T, T)]
    spec = SynthSpec(batch=B, n_heads=H, n_kv_heads=Hk, seq_len=S, head_dim=c["D"],
                     n_planted=planted, seed=c["seed"],
                     dtype=torch.float32 if c["dtype"] == "f32" else torch.bfloat16,
                     flat_query_ranges=flat)
    q, k, v = make_inputs(spec)
    c = dict(c, S=S, H=H, Hkv=Hk, B=B, planted=planted)
    return q, k, v, c


def config_geometry(c: dict, variant: str = "shared"):
    """Selection and attend geometries of a benchmark config: (ga, gc) dicts with inv_freq,
    pos_scale, rope_scale (and dca for the hybrid config's selection).

    * yarn: YaRN frequencies and attention factor, raw positions, for both;
    * hybrid: selection in the Dual Chunk Attention geometry (ChunkLlama rule with s < c as the
      reference asserts, dca_kernel.py:553: s = 6144, w = 1024 for c = 8192, so chunk_len 5120)
      with its mscale 0.05 ln(S / c) + 1; attend with base RoPE at PI scale pos_scale_c;
    * pi: base RoPE at pos_scale for both.
    The per-query variants attend with base RoPE at raw positions (rope_scale 1)."""
    import math
    D = c["D"]
    if c["geom"] == "yarn":
        invf, ms = yarn_inv_freq(D, c["theta"], c["yarn_factor"], c["yarn_orig"])
        ga = dict(inv_freq=invf, pos_scale=1.0, rope_scale=ms)
        gc = dict(ga)
    elif c["geom"] == "hybrid":
        invf = rope_inv_freq(D, c["theta"])
        ms = 0.05 * math.log(c["S"] / c["dca_pretrain"]) + 1.0 if c["S"] > c["dca_pretrain"] else 1.0
        ga = dict(inv_freq=invf, pos_scale=1.0, rope_scale=ms,
                  dca=(c["dca_chunk_size"], c["dca_local_window"]))
        gc = dict(inv_freq=invf, pos_scale=c["pos_scale_c"], rope_scale=1.0)
    else:
        invf = rope_inv_freq(D, c["theta"])
        ga = dict(inv_freq=invf, pos_scale=c.get("pos_scale", 1.0), rope_scale=1.0)
        gc = dict(ga)
    if variant != "shared":
        gc = dict(inv_freq=rope_inv_freq(D, c["theta"]), pos_scale=1.0, rope_scale=1.0)
    return ga, gc
