"""n-way tensor parallelism of the DiT forward (the reference's multi-chip
strategy, oasis_inference.py:289-305, 569-626, 1153-1201, re-expressed for
B200 ranks over NCCL).

Rank r of n holds heads [16 r / n, 16 (r + 1) / n):
  QKV   column-parallel: the q, k and v rows of those heads  -> local qkv [M, 3 x 1024 / n]
  attention on the local heads (spatial and temporal attention stay rank-local)
  O     row-parallel: to_out columns of those heads -> fp32 partial [M, 1024]
  FC1   column-parallel (4096 / n hidden units), FC2 row-parallel -> fp32 partial
After each row-parallel projection the partials are summed with an NCCL
all-reduce, then one kernel adds bias, applies the adaLN gate and the residual.
LayerNorm, adaLN, the final layer and the residual stream are replicated.

Every kernel is a C-ABI call of liboasis_b200.so on the current stream; the
all-reduce is torch.distributed (NCCL over NVLink) on the same stream.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib
from . import host as H
from .weights import DitDeviceWeights, count_blocks

D = H.D_MODEL


def shard_rows(w: torch.Tensor, n: int, r: int) -> torch.Tensor:
    k = w.shape[0] // n
    return w[r * k:(r + 1) * k]


def shard_cols(w: torch.Tensor, n: int, r: int) -> torch.Tensor:
    k = w.shape[1] // n
    return w[:, r * k:(r + 1) * k]


def shard_qkv(w: torch.Tensor, n: int, r: int) -> torch.Tensor:
    """to_qkv.weight [3 x 1024, 1024] -> the q, k, v rows of rank r's heads."""
    return torch.cat([shard_rows(part, n, r) for part in w.split(D, dim=0)], dim=0)


class TPDitWeights:
    """Replicated parts (adaLN, final layer, embed, RoPE) + rank r's shards."""

    def __init__(self, sd: dict, n: int, r: int, device):
        if 16 % n:
            raise ValueError(f"{n}-way tensor parallelism needs n | 16")
        self.n, self.r, self.heads = n, r, 16 // n
        self.full = DitDeviceWeights(sd, device)  # replicated pieces are read from here
        dev = torch.device(device)
        self.n_blocks = count_blocks(sd)

        def bf(t):
            return t.to(dev, torch.bfloat16).contiguous()

        def f32(t):
            return t.to(dev, torch.float32).contiguous()

        self.sub = []
        for i in range(self.n_blocks):
            for s in ("s", "t"):
                p = f"blocks.{i}.{s}"
                self.sub.append(dict(
                    qkv_w=bf(shard_qkv(sd[f"{p}_attn.to_qkv.weight"], n, r)),
                    out_w=bf(shard_cols(sd[f"{p}_attn.to_out.weight"], n, r)),
                    out_b=f32(sd[f"{p}_attn.to_out.bias"]),
                    fc1_w=bf(shard_rows(sd[f"{p}_mlp.fc1.weight"], n, r)),
                    fc1_b=f32(shard_rows(sd[f"{p}_mlp.fc1.bias"], n, r)),
                    fc2_w=bf(shard_cols(sd[f"{p}_mlp.fc2.weight"], n, r)),
                    fc2_b=f32(sd[f"{p}_mlp.fc2.bias"])))


def _st() -> int:
    return torch.cuda.current_stream().cuda_stream


def _gemm(a, w, m, n, k, mode, out, *, bias=None, rope=None, rope_div=1, rope_mod=1, rope_dim=0, rope_stride=0):
    g = _lib.OasisGemmArgs()
    g.a, g.lda, g.w, g.m, g.n, g.k, g.mode = a.data_ptr(), k, w.data_ptr(), m, n, k, mode
    g.out, g.ldo, g.bias = out.data_ptr(), n, _lib.ptr(bias)
    g.rope, g.rope_div, g.rope_mod, g.rope_dim = _lib.ptr(rope), rope_div, rope_mod, rope_dim
    g.rope_stride = rope_stride
    _lib.call("oasis_gemm", C.byref(g), _st())


def _ln(x, y, rows, mod, ld, shift_off, scale_off, *, in_group=144, in_off=0, frame_mul=1, frame_add=0):
    a = _lib.OasisLayerNormArgs()
    a.x, a.y, a.rows_out, a.P, a.in_group, a.in_off = x.data_ptr(), y.data_ptr(), rows, 144, in_group, in_off
    a.frame_mul, a.frame_add, a.eps = frame_mul, frame_add, 1e-6
    a.mod, a.ld_mod, a.shift_off, a.scale_off = mod.data_ptr(), ld, shift_off, scale_off
    _lib.call("oasis_layernorm", C.byref(a), _st())


class TPScratch:
    """Per-rank buffers of one TP forward for B sessions x T frames."""

    def __init__(self, tpw: TPDitWeights, batch: int, frames: int, device):
        F, M = batch * frames, batch * frames * 144
        self.ldm = 2 * tpw.n_blocks * 6144 + 2048
        dev = torch.device(device)
        self.silu = torch.empty(F, D, dtype=torch.bfloat16, device=dev)
        self.adaln = torch.empty(F, self.ldm, device=dev)
        self.xn = torch.empty(M, D, dtype=torch.bfloat16, device=dev)
        self.qkv = torch.empty(M, 3 * D // tpw.n, dtype=torch.bfloat16, device=dev)
        self.attn = torch.empty(M, D // tpw.n, dtype=torch.bfloat16, device=dev)
        self.h = torch.empty(M, 4 * D // tpw.n, dtype=torch.bfloat16, device=dev)
        self.part = torch.empty(M, D, device=dev)


def dit_forward_tp(tpw: TPDitWeights, z: torch.Tensor, cond: torch.Tensor, v_out: torch.Tensor, sc: TPScratch,
                   group=None) -> torch.Tensor:
    """TP DiT forward: z [B, T, 144, 1024] fp32 (replicated, overwritten), cond
    [B, T, 1024] -> v_out [B, 144, 64] for the last frame (replicated)."""
    B, T = z.shape[0], z.shape[1]
    F, M = B * T, B * T * 144
    full, n, ldm = tpw.full, tpw.n, sc.ldm
    _lib.call("oasis_silu_bf16", cond.data_ptr(), sc.silu.data_ptr(), cond.numel(), _st())
    _gemm(sc.silu, full.adaln_w, F, ldm, D, 0, sc.adaln, bias=full.adaln_b)
    zf = z.view(M, D)
    dl = D // n
    for i, w in enumerate(tpw.sub):
        spatial = i % 2 == 0
        off = i * 6144
        _ln(zf, sc.xn, M, sc.adaln, ldm, off, off + D)
        _gemm(sc.xn, w["qkv_w"], M, 3 * dl, D, 6, sc.qkv, rope=full.rope_spatial if spatial else full.rope_temporal,
              rope_div=1 if spatial else 144, rope_mod=144 if spatial else T, rope_dim=dl,
              rope_stride=144 if spatial else H.MAX_T)
        if spatial:
            _lib.call("oasis_attention_spatial", sc.qkv.data_ptr(), sc.attn.data_ptr(), F, 144, tpw.heads, _st())
        else:
            _lib.call("oasis_attention_temporal", sc.qkv.data_ptr(), sc.attn.data_ptr(), B, T, tpw.heads, _st())
        _gemm(sc.attn, w["out_w"], M, D, dl, 0, sc.part)
        dist.all_reduce(sc.part, group=group)
        _lib.call("oasis_gated_residual", zf.data_ptr(), sc.part.data_ptr(), w["out_b"].data_ptr(),
                  sc.adaln[:, off + 2 * D:].data_ptr(), ldm, 144, M, _st())
        _ln(zf, sc.xn, M, sc.adaln, ldm, off + 3 * D, off + 4 * D)
        _gemm(sc.xn, w["fc1_w"], M, 4 * dl, D, 2, sc.h, bias=w["fc1_b"])
        _gemm(sc.h, w["fc2_w"], M, D, 4 * dl, 0, sc.part)
        dist.all_reduce(sc.part, group=group)
        _lib.call("oasis_gated_residual", zf.data_ptr(), sc.part.data_ptr(), w["fc2_b"].data_ptr(),
                  sc.adaln[:, off + 5 * D:].data_ptr(), ldm, 144, M, _st())
    foff = len(tpw.sub) * 6144
    _ln(zf, sc.xn, B * 144, sc.adaln, ldm, foff, foff + D, in_group=T * 144, in_off=(T - 1) * 144,
        frame_mul=T, frame_add=T - 1)
    _gemm(sc.xn, full.final_w, B * 144, H.OUT_DIM, D, 0, v_out, bias=full.final_b)
    return v_out
