"""CPU-side checks of the C ABI library and the host layer (no GPU compute)."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from sta import _lib as L
from sta import core

HERE = os.path.dirname(os.path.abspath(__file__))
HEADER = os.path.join(os.path.dirname(HERE), "include", "sta.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sta_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    decl = declared_functions()
    assert len(decl) >= 15
    for name in decl:
        assert hasattr(lib, name), name
    assert sorted(L.EXPORTED) == decl


def test_struct_layouts_match_header_order():
    """ctypes mirrors list the header's fields in order (names compared)."""
    src = open(HEADER).read()
    for cname, cls in (("sta_select_args", L.SelectArgs), ("sta_build_args", L.BuildArgs),
                       ("sta_build_pq_args", L.BuildPQArgs), ("sta_attend_args", L.AttendArgs),
                       ("sta_pqstream_args", L.PQStreamArgs), ("sta_forward_args", L.ForwardArgs),
                       ("sta_build_chunk_args", L.BuildChunkArgs),
                       ("sta_decode_args", L.DecodeArgs), ("sta_dca_args", L.DcaArgs)):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (cname, cname), src, re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        fields = re.findall(r"\**\s*([A-Za-z_0-9]+)\s*;", body)
        assert [f for f, _ in cls._fields_] == fields, cname


def test_tri_head_stride():
    lib = L.lib()
    for n, t in ((300, 64), (1024, 32), (1, 32), (131072, 32), (65536, 64)):
        nt = (n + t - 1) // t
        assert lib.sta_tri_head_stride(n, t) == t * (nt - 1) * nt // 2 + n


def test_tri_head_stride_of_query_slabs():
    """Compact layout of a query slab [base, n): local tile t holds keys j < base + (t+1)*T."""
    lib = L.lib()
    for n, t, base in ((1000, 64, 384), (131072, 32, 43904), (300, 32, 0), (1100, 64, 1024)):
        nt = (n - base + t - 1) // t
        his = [min(base + (i + 1) * t, n) for i in range(nt)]
        assert lib.sta_tri_head_stride_q(n, t, base) == sum(his)
    assert lib.sta_tri_head_stride_q(32768, 64, 0) == lib.sta_tri_head_stride(32768, 64)


def test_slab_partition_balanced_and_exact_cover():
    from sta.partition import plan, slab_edges
    for n, parts in ((131072, 8), (32768, 2), (65536, 4), (1000, 3)):
        e = slab_edges(n, parts, attend_weight=4096.0 if n > 4096 else 128.0)
        assert e[0] == 0 and e[-1] == n and all(a < b for a, b in zip(e, e[1:]))
        assert all(x % 128 == 0 for x in e[:-1])
        if n >= 32768:
            cost = [(b * b - a * a) / 2 + 4096.0 * (b - a) for a, b in zip(e, e[1:])]
            assert max(cost) / min(cost) < 1.05, cost
    for world, mode in ((8, "heads"), (8, "slabs"), (16, "grid"), (4, "grid"), (6, "auto")):
        cover = {}
        for r in range(world):
            u = plan(8 if world != 6 else 6, 4096, world, r, mode)
            for h in range(*u["kv"]):
                for pos in range(*u["slab"]):
                    cover[(h, pos)] = cover.get((h, pos), 0) + 1
        hk = 8 if world != 6 else 6
        assert len(cover) == hk * 4096 and set(cover.values()) == {1}, (world, mode)


def test_null_arguments_rejected_without_gpu():
    lib = L.lib()
    assert lib.sta_select(None, None) == 1
    assert lib.sta_build_sets(None, None) == 1
    assert lib.sta_gather_attend(None, None) == 1
    assert lib.sta_shared_workspace_bytes(None) == 0
    assert b"null" in lib.sta_last_error()


def test_workspace_query_and_grouping():
    lib = L.lib()
    a = L.ForwardArgs()
    for f in ("q", "k", "v", "out", "tau", "inv_freq_a", "inv_freq_c", "shared_size",
              "kept_size", "chosen", "overflow", "kpct_meas", "overflow20"):
        setattr(a, f, 256)  # non-null placeholders: the size query reads no memory
    a.dtype, a.batch, a.n_heads, a.n_kv_heads, a.n, a.d = 1, 1, 32, 8, 32768, 128
    a.tile, a.k_max, a.select_score = 64, 2048, 0
    full = lib.sta_shared_workspace_bytes(ctypes.byref(a))
    assert full > 0
    a.max_workspace_bytes = full // 4
    part = lib.sta_shared_workspace_bytes(ctypes.byref(a))
    assert 0 < part <= full // 4 + 4096


def test_cpu_tensors_rejected():
    from sta import shared_selection_exact_2 as ex2
    x = torch.zeros((1, 2, 64, 64))
    with pytest.raises(ValueError):
        ex2.shared_pi_attention(x, x, x, torch.ones(2), torch.ones(32))


def test_compact_layout_roundtrip():
    H, N, T = 2, 300, 64
    rng = np.random.default_rng(0)
    dense = torch.from_numpy(rng.integers(0, 65, size=(H, (N + T - 1) // T, N)).astype(np.int32))
    nt = dense.shape[1]
    for t in range(nt):
        dense[:, t, min((t + 1) * T, N):] = 0
    flat = core.compact_from_dense(dense, T)
    assert flat.numel() == H * core.tri_head_stride(N, T)
    assert torch.equal(core.expand_compact(flat, H, N, T), dense)


def test_synth_is_deterministic():
    from sta.synth import SynthSpec, make_inputs
    a = make_inputs(SynthSpec(n_heads=2, n_kv_heads=1, seq_len=128, head_dim=64, seed=3))
    b = make_inputs(SynthSpec(n_heads=2, n_kv_heads=1, seq_len=128, head_dim=64, seed=3))
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    assert a[0].shape == (1, 2, 128, 64) and a[1].shape == (1, 1, 128, 64)


def test_abi_version():
    assert L.lib().sta_version() == 5


def _static_args():
    a = L.ForwardArgs()
    for f in ("q", "k", "v", "out", "tau", "inv_freq_a", "inv_freq_c", "shared_size",
              "kept_size", "chosen", "overflow", "kpct_meas", "overflow20"):
        setattr(a, f, 256)  # non-null placeholders: these calls return before any device work
    a.dtype, a.batch, a.n_heads, a.n_kv_heads, a.d = 1, 1, 4, 2, 128
    a.tile, a.k_max, a.pct = 64, 512, 30.0
    a.pos_scale_a = a.pos_scale_c = a.rope_scale_a = a.rope_scale_c = 1.0
    return a


def test_static_entry_passes_through_argument_codes_without_gpu():
    """The allocation-free entry reports the argument check's own code (head_dim 96 is
    unsupported, not an argument error) and accepts an empty problem like sta_shared_forward,
    whatever its position scales."""
    lib = L.lib()
    a = _static_args()
    a.n, a.d = 256, 96
    assert lib.sta_shared_forward_static(ctypes.byref(a), None) == 2
    assert b"head_dim" in lib.sta_last_error()
    a = _static_args()
    a.n = 0
    a.pos_scale_a = a.pos_scale_c = 0.125
    assert lib.sta_shared_forward_static(ctypes.byref(a), None) == 0


def test_dca_arguments_checked_without_gpu():
    """The dense DCA entry validates before touching the device: chunk_len must be a multiple
    of 128; an empty problem is a no-op."""
    lib = L.lib()
    a = L.DcaArgs()
    for f in ("q", "k", "v", "out", "inv_freq"):
        setattr(a, f, 256)
    a.dtype, a.batch, a.n_heads, a.n_kv_heads, a.n, a.d = 1, 1, 4, 2, 1000, 128
    a.chunk_size, a.local_window, a.rope_scale, a.sm_scale = 320, 100, 1.0, 0.088
    assert lib.sta_dca_workspace_bytes(ctypes.byref(a)) == 0
    assert b"multiple of 128" in lib.sta_last_error()
    a.local_window = 64
    assert lib.sta_dca_workspace_bytes(ctypes.byref(a)) > 0
    a.n = 0
    assert lib.sta_dca_forward(ctypes.byref(a), None, 0, None) == 0
