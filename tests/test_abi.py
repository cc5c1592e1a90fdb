"""CPU checks of the C-ABI boundary: the library loads, exports every function the
header declares, the ctypes mirrors have the C layouts, and argument validation
fails loudly without touching a GPU."""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

from oasis_b200 import _lib
from tests.helpers import ROOT

HEADER = os.path.join(ROOT, "include", "oasis_b200.h")


def declared_functions() -> list[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(oasis_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), f"{n} declared in oasis_b200.h but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures and header disagree"


STRUCTS = ["OasisDitSubBlock", "OasisDitWeights", "OasisVaeBlock", "OasisVaeWeights", "OasisDitArgs",
           "OasisDdimCoeffs", "OasisStepArgs", "OasisFrameArgs", "OasisVaeArgs", "OasisGemmArgs", "OasisLayerNormArgs",
           "OasisTpArgs", "OasisVaeEncoderWeights", "OasisVaeEncodeArgs", "OasisCondWeights", "OasisTpSpArgs"]


def test_ctypes_layouts_match_c():
    prog = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for s in STRUCTS:
        prog.append(f'  printf("{s} %zu\\n", sizeof({s}));')
        for f, _ in getattr(_lib, s)._fields_:
            prog.append(f'  printf("{s}.{f} %zu\\n", offsetof({s}, {f}));')
    prog.append("  return 0; }")
    with tempfile.TemporaryDirectory() as d:
        c, exe = os.path.join(d, "l.c"), os.path.join(d, "l")
        open(c, "w").write("\n".join(prog))
        subprocess.run(["gcc", "-std=c99", c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    sizes = dict(line.rsplit(" ", 1) for line in out.strip().splitlines())
    for s in STRUCTS:
        cls = getattr(_lib, s)
        assert int(sizes[s]) == C.sizeof(cls), s
        for f, _ in cls._fields_:
            assert int(sizes[f"{s}.{f}"]) == getattr(cls, f).offset, f"{s}.{f}"


def test_invalid_arguments_are_rejected_without_a_gpu():
    lib = _lib.load()
    rc = lib.oasis_gemm(None, None)
    assert rc == -1 and b"null" in lib.oasis_last_error()
    args = _lib.OasisGemmArgs()
    args.a, args.w, args.m, args.n, args.k, args.out = 16, 16, 128, 100, 1024, 16
    assert lib.oasis_gemm(C.byref(args), None) == -1
    assert b"multiple of 16" in lib.oasis_last_error()
    args.n, args.k = 128, 100
    assert lib.oasis_gemm(C.byref(args), None) == -1
    assert b"multiple of 64" in lib.oasis_last_error()
    assert lib.oasis_attention_temporal(16, 16, 1, 33, 16, None) == -1
    assert b"frames" in lib.oasis_last_error()
    d = _lib.OasisDitArgs(1, 40, 16, 16, 16, 1, 16, 1 << 30)
    w = _lib.OasisDitWeights()
    assert lib.oasis_dit_forward(C.byref(w), C.byref(d), None) == -1
    d = _lib.OasisDitArgs(1, 2, 16, 16, 16, 1, 0, 0)
    assert lib.oasis_dit_forward(C.byref(w), C.byref(d), None) == -3  # no workspace
    assert b"workspace" in lib.oasis_last_error()
    v = _lib.OasisVaeArgs(0, 16, 16, 16, 1)
    assert lib.oasis_vae_decode(C.byref(_lib.OasisVaeWeights()), C.byref(v), None) == -1


def test_call_raises_with_status_and_message():
    with pytest.raises(_lib.OasisError) as ei:
        _lib.call("oasis_attention_temporal", 16, 16, 1, 0, 16, None)
    assert ei.value.code == -1 and "frames" in str(ei.value)


def test_workspace_sizes_scale_with_batch():
    lib = _lib.load()
    a = lib.oasis_dit_workspace_size(1, 2)
    b = lib.oasis_dit_workspace_size(4, 2)
    assert 0 < a < b
    assert lib.oasis_step_workspace_size(1, 2) > a
    assert lib.oasis_vae_workspace_size(2) > lib.oasis_vae_workspace_size(1) > 0


def test_new_entry_points_validate_without_a_gpu():
    """Context caching, the tcgen05 attention and the LN-fused GEMM epilogue reject
    bad arguments with a status and a message before touching the device."""
    lib = _lib.load()
    w = _lib.OasisDitWeights()
    assert lib.oasis_kv_cache_size(0, 3) == 0 and lib.oasis_kv_cache_size(2, 0) == 0
    assert lib.oasis_kv_cache_size(2, 3) == 16 * 2 * 3 * 144 * 3072 * 2
    d = _lib.OasisDitArgs(1, 0, 16, 16, 16, 0, 16, 1 << 20)  # zero context frames
    assert lib.oasis_dit_precompute_past(C.byref(w), C.byref(d), 16, 1 << 30, None) == -1
    assert b"frames" in lib.oasis_last_error()
    d = _lib.OasisDitArgs(1, 2, 16, 16, 16, 1, 16, 1 << 20)  # the current frame must be one frame
    assert lib.oasis_dit_forward_current(C.byref(w), C.byref(d), 16, 1 << 30, 1, None) == -1
    assert b"frames must be 1" in lib.oasis_last_error()
    d = _lib.OasisDitArgs(1, 1, 16, 16, 16, 1, 16, 1 << 20)
    assert lib.oasis_dit_forward_current(C.byref(w), C.byref(d), 16, 16, 3, None) == -3  # cache too small
    assert b"kv cache" in lib.oasis_last_error()
    assert lib.oasis_attention_tc(16, 16, 2, 100, 16, None) == -1
    assert b"seq=100" in lib.oasis_last_error()
    assert lib.oasis_attention_temporal_cached(16, 16, 16, 1, 40, 16, None) == -1
    g = _lib.OasisGemmArgs()
    g.a, g.w, g.out, g.resid, g.gate = 16, 16, 16, 16, 16
    g.m, g.n, g.k, g.mode, g.rows_per_frame = 256, 512, 1024, 8, 144
    assert lib.oasis_gemm(C.byref(g), None) == -1  # the LN epilogue needs N = 1024
    assert b"N = 1024" in lib.oasis_last_error()
    g.n, g.ldo, g.ldr = 1024, 1024, 1024
    assert lib.oasis_gemm(C.byref(g), None) == -1  # ... and an output and a modulation table
    assert b"modulation" in lib.oasis_last_error()
    g.mode = 9
    assert lib.oasis_gemm(C.byref(g), None) == -1
    assert lib.oasis_get_last_error() == lib.oasis_last_error()


def test_tensor_parallel_entry_validates_without_a_gpu():
    """oasis_dit_forward_tp rejects a head count that does not divide 16, a missing
    collective and a short workspace before touching the device."""
    lib = _lib.load()
    assert lib.oasis_tp_workspace_size(0, 2, 8) == 0
    assert lib.oasis_tp_workspace_size(2, 2, 8) > lib.oasis_tp_workspace_size(1, 2, 8) > 0
    w = _lib.OasisDitWeights()
    cb = _lib.ALLREDUCE_FN(lambda buf, n, user, st: 0)
    a = _lib.OasisTpArgs(1, 2, 3, 16, 16, 16, 16, cb, None, 16, 1 << 30)
    assert lib.oasis_dit_forward_tp(C.byref(w), C.byref(a), None) == -1
    assert b"heads=3" in lib.oasis_last_error()
    a = _lib.OasisTpArgs(1, 2, 8, 16, 16, 16, 16, _lib.ALLREDUCE_FN(), None, 16, 1 << 30)
    assert lib.oasis_dit_forward_tp(C.byref(w), C.byref(a), None) == -1
    assert b"collective" in lib.oasis_last_error()
    a = _lib.OasisTpArgs(1, 2, 8, 16, 16, 16, 16, cb, None, 16, 16)
    assert lib.oasis_dit_forward_tp(C.byref(w), C.byref(a), None) == -3
    assert b"workspace" in lib.oasis_last_error()


def test_vae_encoder_entry_validates_without_a_gpu():
    lib = _lib.load()
    assert lib.oasis_vae_encoder_workspace_size(0) == 0
    assert lib.oasis_vae_encoder_workspace_size(2) > lib.oasis_vae_encoder_workspace_size(1) > 0
    w = _lib.OasisVaeEncoderWeights()
    a = _lib.OasisVaeEncodeArgs(1, 16, None, None, 16, 1 << 30)  # no output
    assert lib.oasis_vae_encode(C.byref(w), C.byref(a), None) == -1
    assert b"neither latent nor chunk" in lib.oasis_last_error()
    w.num_blocks = 13
    a = _lib.OasisVaeEncodeArgs(1, 16, 16, None, 16, 1 << 30)
    assert lib.oasis_vae_encode(C.byref(w), C.byref(a), None) == -1
    assert b"num_blocks=13" in lib.oasis_last_error()
    w.num_blocks = 0
    w.patch_w = w.quant_w = w.norm_w = w.norm_b = 16
    a = _lib.OasisVaeEncodeArgs(1, 16, 16, None, 16, 16)
    assert lib.oasis_vae_encode(C.byref(w), C.byref(a), None) == -3
    assert b"workspace" in lib.oasis_last_error()


def test_frame_count_bounds():
    """T is bounded by the temporal RoPE table (OASIS_MAX_FRAMES = 32 positions)."""
    lib = _lib.load()
    w = _lib.OasisDitWeights()
    for T in (0, 33):
        d = _lib.OasisDitArgs(1, T, 16, 16, 16, 1, 16, 1 << 40)
        assert lib.oasis_dit_forward(C.byref(w), C.byref(d), None) == -1
        assert b"frames" in lib.oasis_last_error() or b"T=" in lib.oasis_last_error(), lib.oasis_last_error()


def _plan(lib, m, n, k, mode=0, block_n=0, splits=0):
    bn, sp, pair, by = C.c_int(), C.c_int(), C.c_int(), C.c_size_t()
    rc = lib.oasis_gemm_plan(m, n, k, mode, block_n, splits, C.byref(bn), C.byref(sp), C.byref(pair), C.byref(by))
    return rc, bn.value, sp.value, pair.value, by.value


def test_gemm_plan_and_workspace_queries_agree():
    """oasis_gemm_plan is the launch's own planning rule; the workspace queries
    (the caller-workspace one and the fixed-scratch entry point's size check)
    size from the same plan."""
    lib = _lib.load()
    # bench shapes (M = 73728): every DiT projection on CTA pairs, no split-K
    for n, k, mode in ((3072, 1024, 6), (1024, 1024, 4), (4096, 1024, 2), (1024, 4096, 4)):
        rc, bn, sp, pair, by = _plan(lib, 73728, n, k, mode)
        assert (rc, bn, sp, pair, by) == (0, 512, 1, 1, 0), (n, k, mode)
    # B = 1 FC2 (M = 288, K = 4096): 128-wide tiles x 4 K splits in clusters
    rc, bn, sp, pair, by = _plan(lib, 288, 1024, 4096, 4)
    assert (rc, bn, sp, pair) == (0, 128, 4, 0)
    assert by == 3 * 8 * 4 * 128 * 128 * 4
    assert lib.oasis_gemm_workspace_size(288, 1024, 4096) == by
    # B = 1 O projection: fp32 epilogue narrows to 32-wide tiles, no split
    rc, bn, sp, pair, by = _plan(lib, 288, 1024, 1024, 4)
    assert (rc, bn, sp, by) == (0, 32, 1, 0)
    # explicit overrides are what the launch uses
    rc, bn, sp, pair, by = _plan(lib, 300, 1024, 4096, 4, block_n=64, splits=4)
    assert (rc, bn, sp) == (0, 64, 4) and by == 3 * 16 * 4 * 128 * 64 * 4
    rc, bn, sp, pair, by = _plan(lib, 4096, 4096, 4096, 0, block_n=64, splits=8)
    assert by == 32 * 64 * 8 * 128 * 64 * 4 and by > lib.oasis_gemm_static_scratch_capacity()
    # rejected overrides: bf16 output on 32-wide tiles, splits that do not divide K
    assert _plan(lib, 288, 1024, 1024, 1, block_n=32)[0] == -1
    assert _plan(lib, 288, 1024, 1024, 0, block_n=64, splits=3)[0] == -1
    assert _plan(lib, 288, 1024, 1000, 0)[0] == -1
