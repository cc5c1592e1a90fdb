"""Small, self-contained launch cases for ncu captures of single kernels.

    python profile_cases.py gemm --m 16384 --n 4096 --k 1024 --mode 2 [--reps 3]
    python profile_cases.py attn_spatial --groups 512
    python profile_cases.py attn_temporal --batch 64 --frames 8
    python profile_cases.py layernorm --rows 73728
    python profile_cases.py attn_temporal_cached --batch 64 --frames 8
    python profile_cases.py frame --batch 64 --frames 8 [--kv] --reps 1

Each case allocates only what the one kernel needs (a few GB at most), runs it
`reps` times and exits, so an ncu capture with -k/-c ends by itself quickly.
"""
from __future__ import annotations

import argparse
import ctypes as C
import os
import sys

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from oasis_b200 import _lib  # noqa: E402


def _st():
    return torch.cuda.current_stream().cuda_stream


def gemm(a):
    M, N, K = a.m, a.n, a.k
    A = (torch.randn(M, K, device="cuda") * 0.5).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    bias = torch.zeros(N, device="cuda")
    gate = torch.randn((M + 143) // 144, N, device="cuda")
    rope = torch.zeros(16, 144, 4, device="cuda")  # identity rotation, the kernel's table layout
    rope[..., 0] = 1
    rope[..., 2] = 1
    args = _lib.OasisGemmArgs()
    args.a, args.lda, args.w, args.m, args.n, args.k, args.mode = A.data_ptr(), K, W.data_ptr(), M, N, K, a.mode
    args.out, args.ldo, args.bias = out.data_ptr(), N, bias.data_ptr()
    args.resid, args.ldr, args.gate, args.ldg, args.rows_per_frame = out.data_ptr(), N, gate.data_ptr(), N, 144
    args.rope, args.rope_div, args.rope_mod = rope.data_ptr(), 1, 144
    args.block_n, args.splits = a.block_n, a.splits
    need = C.c_size_t(0)
    _lib.call("oasis_gemm_plan", M, N, K, a.mode, a.block_n, a.splits, None, None, None, C.byref(need))
    ws = torch.empty(max(need.value, 256), dtype=torch.uint8, device="cuda")
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    a._keep = (A, W, out, bias, gate, rope, ws, args)
    return lambda: _lib.call("oasis_gemm", C.byref(args), _st())


def attn_spatial(a):
    qkv = torch.randn(a.groups * a.seq, 3072, device="cuda").to(torch.bfloat16)
    out = torch.empty(a.groups * a.seq, 1024, device="cuda", dtype=torch.bfloat16)
    a._keep = (qkv, out)
    return lambda: _lib.call("oasis_attention_spatial", qkv.data_ptr(), out.data_ptr(), a.groups, a.seq, 16, _st())


def attn_temporal(a):
    rows = a.batch * a.frames * 144
    qkv = torch.randn(rows, 3072, device="cuda").to(torch.bfloat16)
    out = torch.empty(rows, 1024, device="cuda", dtype=torch.bfloat16)
    a._keep = (qkv, out)
    return lambda: _lib.call("oasis_attention_temporal", qkv.data_ptr(), out.data_ptr(), a.batch, a.frames, 16, _st())


def attn_temporal_cached(a):
    P = 144
    past = torch.randn(a.batch * (a.frames - 1) * P, 3072, device="cuda").to(torch.bfloat16)
    cur = torch.randn(a.batch * P, 3072, device="cuda").to(torch.bfloat16)
    out = torch.empty(a.batch * P, 1024, device="cuda", dtype=torch.bfloat16)
    a._keep = (past, cur, out)
    return lambda: _lib.call("oasis_attention_temporal_cached", past.data_ptr(), cur.data_ptr(), out.data_ptr(),
                             a.batch, a.frames - 1, 16, _st())


def frame(a):
    """One whole frame (conditioning, 4 DDIM steps + VAE) for --batch sessions x
    --frames T, full-T (default) or with the context rows cached (--kv)."""
    from oasis_b200 import engine as E
    from oasis_b200.weights import DitDeviceWeights, VaeDeviceWeights, init_dit_weights, init_vae_weights

    dev = torch.device("cuda")
    dw = DitDeviceWeights(init_dit_weights(seed=0), dev)
    vw = VaeDeviceWeights(init_vae_weights(seed=0), dev)
    fe = E.FrameEngine(dw, vw, a.batch, a.frames, kv=a.kv, device_cond=True)  # as bench.py
    fe.chunk.normal_()
    fe.context_z.normal_()
    fe.actions[..., 0] = 1.0
    a._keep = (dw, vw, fe)
    return fe.run


def layernorm(a):
    x = torch.randn(a.rows, 1024, device="cuda")
    y = torch.empty(a.rows, 1024, device="cuda", dtype=torch.bfloat16)
    frames = (a.rows + 143) // 144
    mod = torch.randn(frames, 2048, device="cuda")
    args = _lib.OasisLayerNormArgs()
    args.x, args.y, args.rows_out, args.P, args.in_group = x.data_ptr(), y.data_ptr(), a.rows, 144, 144
    args.frame_mul, args.eps, args.mod, args.ld_mod, args.shift_off, args.scale_off = 1, 1e-6, mod.data_ptr(), 2048, 0, 1024
    a._keep = (x, y, mod, args)
    return lambda: _lib.call("oasis_layernorm", C.byref(args), _st())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "attn_spatial", "attn_temporal", "attn_temporal_cached", "layernorm",
                                     "frame"])
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--mode", type=int, default=2)
    ap.add_argument("--block-n", type=int, default=0)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--groups", type=int, default=512)
    ap.add_argument("--seq", type=int, default=144)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--frames", type=int, default=8)
    ap.add_argument("--rows", type=int, default=73728)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--kv", action="store_true", help="frame case: context rows cached")
    ap.add_argument("--time", action="store_true", help="print the mean time per launch (CUDA events)")
    a = ap.parse_args()
    launch = globals()[a.case](a)
    if a.time:
        # the reps launches recorded as one CUDA graph, so the time is the
        # device's (host launch cost would dominate a few-microsecond kernel)
        for _ in range(3):
            launch()
        torch.cuda.synchronize()
        s_ = torch.cuda.Stream()
        with torch.cuda.stream(s_):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s_):
                for _ in range(a.reps):
                    launch()
        g.replay()
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        g.replay()
        ev[1].record()
        ev[1].synchronize()
        print(f"{a.case}: {ev[0].elapsed_time(ev[1]) * 1000 / a.reps:.2f} us per launch (graph)")
    else:
        for _ in range(a.reps):
            launch()
    torch.cuda.synchronize()
    err = _lib.load().oasis_device_error(0)
    if err:
        raise SystemExit(f"device error word {err}")


if __name__ == "__main__":
    main()
