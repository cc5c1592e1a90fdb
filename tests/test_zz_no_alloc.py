"""The allocation-free GEMM entry point, for callers that cannot allocate device
memory themselves (their allocator belongs to a host framework, or allocating is
not allowed where they run). It must give the same result as oasis_gemm with a
caller workspace, call after call, and refuse problems whose split-K scratch
does not fit its fixed array.

This file is named to be collected last, so a run that stops at the first
failure has run every other test before this one."""
from __future__ import annotations

import ctypes as C

import pytest
import torch

from oasis_b200 import _lib
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _args(a, w, out, *, resid=None, gate=None, bias=None, block_n=64, splits=4, ws=None):
    M, K = a.shape
    N = w.shape[0]
    g = _lib.OasisGemmArgs()
    g.a, g.lda, g.w, g.m, g.n, g.k = a.data_ptr(), K, w.data_ptr(), M, N, K
    g.mode = 4 if gate is not None else 0
    g.out, g.ldo, g.bias = out.data_ptr(), N, _lib.ptr(bias)
    g.resid, g.ldr = _lib.ptr(resid), N
    g.gate, g.ldg, g.rows_per_frame = _lib.ptr(gate), N, 144
    g.block_n, g.splits = block_n, splits
    if ws is not None:
        g.workspace, g.workspace_bytes = ws.data_ptr(), ws.numel()
    return g


def _call(name, g):
    _lib.call(name, C.byref(g), torch.cuda.current_stream().cuda_stream)


def test_static_scratch_matches_workspace_gemm_twice():
    gen = torch.Generator().manual_seed(7)
    M, N, K = 300, 1024, 4096  # B=1-like shape that takes the split-K path
    a = (torch.randn(M, K, generator=gen)).to(DEV, torch.bfloat16)
    w = (torch.randn(N, K, generator=gen) * 0.02).to(DEV, torch.bfloat16)
    bias = torch.randn(N, generator=gen).to(DEV)
    gate = torch.randn((M + 143) // 144, N, generator=gen).to(DEV)
    z0 = torch.randn(M, N, generator=gen).to(DEV)
    ws = torch.empty(_lib.load().oasis_gemm_workspace_size(M, N, K) + (64 << 20), dtype=torch.uint8, device=DEV)

    ref = z0.clone()
    _call("oasis_gemm", _args(a, w, ref, resid=ref, gate=gate, bias=bias, ws=ws))
    for _ in range(2):  # the shared array keeps the last call's contents; both calls must agree
        got = z0.clone()
        _call("oasis_gemm_static_scratch", _args(a, w, got, resid=got, gate=gate, bias=bias))
        torch.cuda.synchronize()
        assert rel_l2(got, ref) < 1e-5
        assert torch.equal(got, ref)  # split-K sums in split order: deterministic

    # a plain (non-gated) split-K problem as well
    out_ref = torch.empty(M, N, device=DEV)
    out = torch.empty(M, N, device=DEV)
    _call("oasis_gemm", _args(a, w, out_ref, bias=bias, splits=2, ws=ws))
    _call("oasis_gemm_static_scratch", _args(a, w, out, bias=bias, splits=2))
    torch.cuda.synchronize()
    assert rel_l2(out, out_ref) < 1e-5


def test_static_scratch_rejects_oversized_problems():
    lib = _lib.load()
    cap = lib.oasis_gemm_static_scratch_capacity()
    assert cap == 8 << 20
    M, N, K = 4096, 4096, 4096  # 32 x 64 tiles x 8 splits x 32 KB >> 8 MiB
    a = torch.zeros(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(N, K, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=DEV)
    g = _args(a, w, out, block_n=64, splits=8)
    rc = lib.oasis_gemm_static_scratch(C.byref(g), torch.cuda.current_stream().cuda_stream)
    assert rc == -3
    assert b"more than the fixed" in lib.oasis_last_error()
