"""Per-kernel parity through the C ABI against plain PyTorch fp32 references of
the same op on the same (bf16-rounded) inputs."""
from __future__ import annotations

import ctypes as C
import math

import pytest
import torch
import torch.nn.functional as F

from oasis_b200 import _lib
from oasis_b200 import host as H
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _s():
    return torch.cuda.current_stream().cuda_stream


def gemm(a, w, mode, out, *, bias=None, resid=None, gate=None, ldg=0, rows_per_frame=1, rope=None,
         rope_div=1, rope_mod=1, rope_dim=0, rope_stride=0, block_n=0, splits=0, ws=None):
    M, K = a.shape
    N = w.shape[0]
    args = _lib.OasisGemmArgs()
    args.a, args.lda, args.w = a.data_ptr(), K, w.data_ptr()
    args.m, args.n, args.k, args.mode = M, N, K, mode
    args.out, args.ldo = out.data_ptr(), (N if mode != 7 else 0)
    args.bias = _lib.ptr(bias)
    args.resid, args.ldr = _lib.ptr(resid), N
    args.gate, args.ldg, args.rows_per_frame = _lib.ptr(gate), ldg, rows_per_frame
    args.rope, args.rope_div, args.rope_mod, args.rope_dim = _lib.ptr(rope), rope_div, rope_mod, rope_dim
    args.rope_stride = rope_stride
    args.block_n, args.splits = block_n, splits
    if ws is not None:
        args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.call("oasis_gemm", C.byref(args), _s())
    torch.cuda.synchronize()
    return out


def rand_bf16(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(DEV, torch.bfloat16)


@pytest.mark.parametrize("M,N,K,block_n,splits", [
    (128, 256, 64, 256, 1), (288, 3072, 1024, 0, 0), (300, 1024, 1024, 64, 4), (1000, 4096, 1024, 256, 1),
    (577, 1024, 4096, 128, 1), (2, 2048, 1024, 64, 2), (1152, 64, 1024, 64, 1), (4608, 1024, 4096, 0, 0),
    (73, 1200, 1024, 128, 1), (512, 1024, 1024, 64, 8), (300, 1024, 4096, 32, 2), (300, 1024, 1024, 32, 1),
    (300, 1216, 192, 64, 1), (130, 1024, 4096, 64, 1),
    # block_n 512: 256 x 256 tiles on CTA pairs (one stage; ragged M and N; several tiles per pair)
    (256, 256, 64, 512, 1), (1000, 4096, 1024, 512, 1), (300, 1200, 320, 512, 1), (20000, 4096, 1024, 512, 1),
    (577, 1024, 4096, 512, 1),
])
def test_gemm_f32(M, N, K, block_n, splits):
    a = rand_bf16(M, K, seed=1)
    w = rand_bf16(N, K, scale=0.05, seed=2)
    bias = torch.randn(N, device=DEV)
    out = torch.full((M, N), float("nan"), device=DEV)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=DEV)
    gemm(a, w, 0, out, bias=bias, block_n=block_n, splits=splits, ws=ws)
    ref = a.float() @ w.float().T + bias
    assert rel_l2(out, ref) < 1e-5, rel_l2(out, ref)


def test_gemm_splitk_deterministic():
    a, w = rand_bf16(300, 4096, seed=3), rand_bf16(1024, 4096, scale=0.05, seed=4)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=DEV)
    o1 = torch.empty(300, 1024, device=DEV)
    o2 = torch.empty(300, 1024, device=DEV)
    gemm(a, w, 0, o1, block_n=64, splits=8, ws=ws)
    gemm(a, w, 0, o2, block_n=64, splits=8, ws=ws)
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("block_n", [0, 512])
def test_gemm_bf16_epilogues(mode, block_n):
    M, N, K = 700, 4096, 1024
    a, w = rand_bf16(M, K, seed=5), rand_bf16(N, K, scale=0.05, seed=6)
    bias = torch.randn(N, device=DEV) * 0.1
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    gemm(a, w, mode, out, bias=bias, block_n=block_n)
    ref = a.float() @ w.float().T + bias
    if mode == 2:
        ref = F.gelu(ref, approximate="tanh")
    elif mode == 3:
        ref = F.gelu(ref)
    assert rel_l2(out.float(), ref) < 5e-3


@pytest.mark.parametrize("M,block_n,splits", [(288, 0, 0), (1152, 256, 1), (300, 64, 4), (1152, 512, 1),
                                                (40000, 512, 1)])
def test_gemm_gated_residual(M, block_n, splits):
    N, K, P = 1024, 1024, 144
    frames = (M + P - 1) // P
    a, w = rand_bf16(M, K, seed=7), rand_bf16(N, K, scale=0.05, seed=8)
    bias = torch.randn(N, device=DEV) * 0.1
    ld = 6144 * 2 + 2048
    table = torch.randn(frames, ld, device=DEV)
    off = 6144 + 2 * 1024
    resid = torch.randn(M, N, device=DEV)
    z = resid.clone()
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=DEV)
    gemm(a, w, 4, z, bias=bias, resid=z, gate=table[:, off:], ldg=ld, rows_per_frame=P, block_n=block_n,
         splits=splits, ws=ws)
    gate = table[torch.arange(M, device=DEV) // P, off:off + N]
    ref = resid + gate * (a.float() @ w.float().T + bias)
    assert rel_l2(z, ref) < 1e-5


def test_gemm_pair_matches_single_cta_tiles():
    """The heuristic sends a C4-sized FC1 to CTA pairs; the result matches 128 x 256 tiles."""
    M, N, K = 73728, 4096, 1024
    a, w = rand_bf16(M, K, seed=11), rand_bf16(N, K, scale=0.05, seed=12)
    bias = torch.randn(N, device=DEV) * 0.1
    o_pair = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    o_one = torch.empty_like(o_pair)
    gemm(a, w, 2, o_pair, bias=bias)
    gemm(a, w, 2, o_one, bias=bias, block_n=256)
    assert rel_l2(o_pair.float(), o_one.float()) < 1e-3


def test_gemm_residual():
    M, N, K = 576 * 2, 1024, 4096
    a, w = rand_bf16(M, K, seed=9), rand_bf16(N, K, scale=0.02, seed=10)
    bias = torch.randn(N, device=DEV)
    z = torch.randn(M, N, device=DEV)
    ref = z + a.float() @ w.float().T + bias
    gemm(a, w, 5, z, bias=bias, resid=z)
    assert rel_l2(z, ref) < 1e-5


def _rope_ref(x, tab, pos, hd=1024):
    """x [M, 3 hd] fp32; rotate q/k column pairs with tab[pos[r], pair]."""
    out = x.clone()
    c = tab[pos][:, :, 0].repeat(1, hd // 64)  # one entry per pair across the heads
    s = tab[pos][:, :, 1].repeat(1, hd // 64)
    for sec in range(2):
        seg = x[:, sec * hd:(sec + 1) * hd]
        x0, x1 = seg[:, 0::2], seg[:, 1::2]
        out[:, sec * hd:(sec + 1) * hd][:, 0::2] = x0 * c - x1 * s
        out[:, sec * hd:(sec + 1) * hd][:, 1::2] = x1 * c + x0 * s
    return out


@pytest.mark.parametrize("kind", ["spatial", "temporal", "vae"])
@pytest.mark.parametrize("block_n", [0, 512])
def test_gemm_rope(kind, block_n):
    if kind == "spatial":
        M, tab, div, mod = 2 * 144 * 3, H.rope_pair_table(H.spatial_rope_angles(H.default_spatial_freqs())), 1, 144
    elif kind == "temporal":
        T = 8
        M, tab, div, mod = 2 * T * 144, H.rope_pair_table(H.temporal_rope_angles(H.default_temporal_freqs())), 144, T
    else:
        M, tab, div, mod = 2 * 576, H.rope_pair_table(H.vae_rope_angles(H.default_vae_freqs())), 1, 576
    K, N = 1024, 3072
    a, w = rand_bf16(M, K, seed=11), rand_bf16(N, K, scale=0.05, seed=12)
    bias = torch.randn(N, device=DEV) * 0.1 if kind == "vae" else None
    tab_d = tab.to(DEV)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    quad = tab.reshape(tab.shape[0], 16, 4).permute(1, 0, 2).contiguous().to(DEV)  # [16, positions, 4]
    gemm(a, w, 6, out, bias=bias, rope=quad, rope_div=div, rope_mod=mod, rope_stride=tab.shape[0], block_n=block_n)
    x = a.float() @ w.float().T + (bias if bias is not None else 0)
    pos = (torch.arange(M, device=DEV) // div) % mod
    ref = _rope_ref(x, tab_d, pos)
    assert rel_l2(out.float(), ref) < 5e-3


@pytest.mark.parametrize("n", [2, 4, 8])
def test_tensor_parallel_shard_shapes(n):
    """The GEMM shapes one rank runs under n-way tensor parallelism (QKV + RoPE on
    its 16 / n heads, O and FC2 row shards with K = 1024 / n and 4096 / n, FC1
    column shard) against PyTorch, at the C5 row count of one DiT step slice."""
    M, D, HD = 2 * 144 * 3, 1024, 1024 // n
    a = rand_bf16(M, D, seed=21)
    tab = H.rope_pair_table(H.temporal_rope_angles(H.default_temporal_freqs())).to(DEV)
    w = rand_bf16(3 * HD, D, scale=0.05, seed=22)
    qkv = torch.empty(M, 3 * HD, device=DEV, dtype=torch.bfloat16)
    quad = tab.reshape(tab.shape[0], 16, 4).permute(1, 0, 2).contiguous()
    gemm(a, w, 6, qkv, rope=quad, rope_div=144, rope_mod=3, rope_dim=HD, rope_stride=tab.shape[0])
    pos = (torch.arange(M, device=DEV) // 144) % 3
    ref = _rope_ref(a.float() @ w.float().T, tab, pos, hd=HD)
    assert rel_l2(qkv.float(), ref) < 5e-3
    for K in (HD, 4 * HD):  # O and FC2 row shards: fp32 partials
        x, wo = rand_bf16(M, K, seed=23 + K), rand_bf16(D, K, scale=0.05, seed=24 + K)
        part = torch.empty(M, D, device=DEV)
        gemm(x, wo, 0, part)
        assert rel_l2(part, x.float() @ wo.float().T) < 1e-5
    w1, b1 = rand_bf16(4 * HD, D, scale=0.05, seed=25), torch.randn(4 * HD, device=DEV) * 0.1
    h = torch.empty(M, 4 * HD, device=DEV, dtype=torch.bfloat16)
    gemm(a, w1, 2, h, bias=b1)
    assert rel_l2(h.float(), F.gelu(a.float() @ w1.float().T + b1, approximate="tanh")) < 5e-3


@pytest.mark.parametrize("M,K", [(1152, 4096), (300, 1024), (4608, 1024), (2 * 148 * 128 + 200, 1024)])
def test_gemm_gated_residual_layernorm(M, K):
    """Mode 8: the gated residual update of z plus the next sub-block's LayerNorm +
    adaLN modulate of the updated rows, written as bf16 (whole 1024-wide rows per
    CTA, row statistics combined across the row's four tiles; the last case gives
    every CTA three row blocks)."""
    N, P = 1024, 144
    frames = (M + P - 1) // P
    a, w = rand_bf16(M, K, seed=41), rand_bf16(N, K, scale=0.05, seed=42)
    bias = torch.randn(N, device=DEV) * 0.1
    ldm = 4096
    mod = torch.randn(frames, ldm, device=DEV) * 0.5
    mod[:, 1024:2048] += 1.0  # (1 + scale) as the adaLN table holds it
    gate_off, shift_off, scale_off = 2048, 0, 1024
    z0 = torch.randn(M, N, device=DEV) * 2 + 0.3
    z = z0.clone()
    xn = torch.full((M, N), float("nan"), device=DEV, dtype=torch.bfloat16)
    g = _lib.OasisGemmArgs()
    g.a, g.lda, g.w, g.m, g.n, g.k, g.mode = a.data_ptr(), K, w.data_ptr(), M, N, K, 8
    g.out, g.ldo, g.bias, g.resid, g.ldr = z.data_ptr(), N, bias.data_ptr(), z.data_ptr(), N
    g.gate, g.ldg, g.rows_per_frame = mod[:, gate_off:].data_ptr(), ldm, P
    g.ln_out, g.ln_mod, g.ln_ld_mod, g.ln_shift_off, g.ln_scale_off = xn.data_ptr(), mod.data_ptr(), ldm, shift_off, scale_off
    _lib.call("oasis_gemm", C.byref(g), _s())
    torch.cuda.synchronize()
    assert _lib.load().oasis_device_error(1) == 0
    fr = torch.arange(M, device=DEV) // P
    z_ref = z0 + mod[fr, gate_off:gate_off + N] * (a.float() @ w.float().T + bias)
    assert rel_l2(z, z_ref) < 1e-5
    ln = F.layer_norm(z_ref, (N,), eps=1e-6)
    xn_ref = ln * mod[fr, scale_off:scale_off + N] + mod[fr, shift_off:shift_off + N]
    assert not torch.isnan(xn.float()).any()
    assert rel_l2(xn.float(), xn_ref) < 5e-3, rel_l2(xn.float(), xn_ref)


def test_gemm_image():
    B = 2
    M, N, K = B * 576, 1200, 1024
    a, w = rand_bf16(M, K, seed=13), rand_bf16(N, K, scale=0.05, seed=14)
    bias = torch.randn(N, device=DEV) * 0.1
    img = torch.full((B, 3, 360, 640), float("nan"), device=DEV)
    gemm(a, w, 7, img, bias=bias)
    pred = (a.float() @ w.float().T + bias).reshape(B, 18, 32, 1200).permute(0, 3, 1, 2)
    pred = pred.reshape(B, 3, 20, 20, 18, 32).permute(0, 1, 4, 2, 5, 3).reshape(B, 3, 360, 640)
    ref = pred.clamp(-1, 1)
    assert not torch.isnan(img).any()
    assert rel_l2(img, ref) < 1e-5


def _ln(args):
    _lib.call("oasis_layernorm", C.byref(args), _s())
    torch.cuda.synchronize()


def test_layernorm_modulate():
    B, T, P = 2, 3, 144
    M = B * T * P
    x = torch.randn(M, 1024, device=DEV) * 3 + 1
    ld = 6144 + 2048
    mod = torch.randn(B * T, ld, device=DEV)
    y = torch.empty(M, 1024, device=DEV, dtype=torch.bfloat16)
    a = _lib.OasisLayerNormArgs()
    a.x, a.y, a.rows_out, a.P, a.in_group = x.data_ptr(), y.data_ptr(), M, P, P
    a.frame_mul, a.eps, a.mod, a.ld_mod, a.shift_off, a.scale_off = 1, 1e-6, mod.data_ptr(), ld, 3072, 4096
    _ln(a)
    fr = torch.arange(M, device=DEV) // P
    ref = F.layer_norm(x, (1024,), eps=1e-6) * mod[fr, 4096:5120] + mod[fr, 3072:4096]
    assert rel_l2(y.float(), ref) < 4e-3


def test_layernorm_final_gather():
    B, T, P = 3, 4, 144
    x = torch.randn(B * T * P, 1024, device=DEV)
    ld = 2048
    mod = torch.randn(B * T, ld, device=DEV)
    y = torch.empty(B * P, 1024, device=DEV, dtype=torch.bfloat16)
    a = _lib.OasisLayerNormArgs()
    a.x, a.y, a.rows_out, a.P = x.data_ptr(), y.data_ptr(), B * P, P
    a.in_group, a.in_off, a.frame_mul, a.frame_add = T * P, (T - 1) * P, T, T - 1
    a.eps, a.mod, a.ld_mod, a.shift_off, a.scale_off = 1e-6, mod.data_ptr(), ld, 0, 1024
    _ln(a)
    xl = x.reshape(B, T, P, 1024)[:, -1].reshape(B * P, 1024)
    fr = (torch.arange(B * P, device=DEV) // P) * T + T - 1
    ref = F.layer_norm(xl, (1024,), eps=1e-6) * mod[fr, 1024:] + mod[fr, :1024]
    assert rel_l2(y.float(), ref) < 4e-3


def test_layernorm_affine():
    M = 576 * 2
    x = torch.randn(M, 1024, device=DEV) * 2
    w, b = torch.randn(1024, device=DEV), torch.randn(1024, device=DEV)
    y = torch.empty(M, 1024, device=DEV, dtype=torch.bfloat16)
    a = _lib.OasisLayerNormArgs()
    a.x, a.y, a.rows_out, a.P, a.eps = x.data_ptr(), y.data_ptr(), M, M, 1e-6
    a.affine_w, a.affine_b = w.data_ptr(), b.data_ptr()
    _ln(a)
    ref = F.layer_norm(x, (1024,), w, b, eps=1e-6)
    assert rel_l2(y.float(), ref) < 4e-3


def _attn_ref(q, k, v, mask=None):
    s = q @ k.transpose(-1, -2) / 8.0
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf"))
    return torch.softmax(s, -1) @ v


ATTN_CASES = [(1, 144, 16), (5, 144, 16), (37, 144, 16), (9, 144, 8), (3, 144, 2), (2, 576, 16), (3, 576, 16),
              (1, 576, 4), (1, 50, 16), (3, 200, 16)]


@pytest.mark.parametrize("groups,seq,H", ATTN_CASES)
def test_attention_full(groups, seq, H):
    """Full attention within groups: seq 144 (DiT spatial) and 576 (VAE) run the
    tcgen05 kernel (128-row query tiles that straddle groups), other lengths the
    mma.sync kernel; H = 16 / n under n-way tensor parallelism."""
    HD = H * 64
    qkv = rand_bf16(groups * seq, 3 * HD, seed=groups * 1000 + seq + H)
    out = torch.full((groups * seq, HD), float("nan"), device=DEV, dtype=torch.bfloat16)
    _lib.call("oasis_attention_spatial", qkv.data_ptr(), out.data_ptr(), groups, seq, H, _s())
    torch.cuda.synchronize()
    assert _lib.load().oasis_device_error(1) == 0
    x = qkv.float().reshape(groups, seq, 3, H, 64).permute(2, 0, 3, 1, 4)  # 3 G H S D
    ref = _attn_ref(x[0], x[1], x[2]).permute(0, 2, 1, 3).reshape(groups * seq, HD)
    assert not torch.isnan(out.float()).any()
    assert rel_l2(out.float(), ref) < 1e-2, rel_l2(out.float(), ref)


@pytest.mark.parametrize("groups,seq,H", [c for c in ATTN_CASES if c[1] in (144, 576)])
def test_attention_tc(groups, seq, H):
    """The tcgen05 attention kernel (OASIS_ATTN_TC=1 selects it on the model path)
    against the PyTorch fp32 reference."""
    from oasis_b200 import _lib as L

    HD = H * 64
    qkv = rand_bf16(groups * seq, 3 * HD, seed=groups * 7 + seq + H)
    out = torch.full((groups * seq, HD), float("nan"), device=DEV, dtype=torch.bfloat16)
    L.call("oasis_attention_tc", qkv.data_ptr(), out.data_ptr(), groups, seq, H, _s())
    torch.cuda.synchronize()
    assert L.load().oasis_device_error(1) == 0
    x = qkv.float().reshape(groups, seq, 3, H, 64).permute(2, 0, 3, 1, 4)
    ref = _attn_ref(x[0], x[1], x[2]).permute(0, 2, 1, 3).reshape(groups * seq, HD)
    assert rel_l2(out.float(), ref) < 1e-2, rel_l2(out.float(), ref)


@pytest.mark.parametrize("B,T,H", [(1, 1, 16), (1, 2, 16), (2, 8, 16), (1, 32, 16), (3, 5, 16), (2, 8, 8), (1, 16, 4),
                                   (2, 8, 2), (1, 32, 2)])
def test_attention_temporal(B, T, H):
    """Causal temporal attention (H = 16, or 16 / n heads per rank under n-way
    tensor parallelism: a warp's 256 columns then cover fewer than four heads)."""
    P, HD = 144, H * 64
    qkv = rand_bf16(B * T * P, 3 * HD, seed=B * 100 + T + H)
    out = torch.full((B * T * P, HD), float("nan"), device=DEV, dtype=torch.bfloat16)
    _lib.call("oasis_attention_temporal", qkv.data_ptr(), out.data_ptr(), B, T, H, _s())
    torch.cuda.synchronize()
    x = qkv.float().reshape(B, T, P, 3, H, 64).permute(3, 0, 2, 4, 1, 5)  # 3 B P H T D
    mask = torch.tril(torch.ones(T, T, dtype=torch.bool, device=DEV))
    ref = _attn_ref(x[0], x[1], x[2], mask).permute(0, 3, 1, 2, 4).reshape(B * T * P, HD)
    assert not torch.isnan(out.float()).any()
    assert rel_l2(out.float(), ref) < 1e-2


@pytest.mark.parametrize("B,T,H", [(1, 1, 16), (1, 2, 16), (2, 8, 16), (1, 32, 16), (3, 5, 16), (2, 8, 8), (2, 3, 2),
                                   (1, 4, 1)])
def test_attention_temporal_cached(B, T, H):
    """The generated frame's query against cached context K/V equals the last
    frame's rows of full causal temporal attention (H heads: 16, or 16 / n under
    n-way tensor parallelism)."""
    P, Tp, HD = 144, T - 1, H * 64
    qkv = rand_bf16(B * T * P, 3 * HD, seed=B * 10 + T).reshape(B, T, P, 3 * HD)
    past = qkv[:, :Tp].contiguous()
    cur = qkv[:, Tp].contiguous()
    out = torch.empty(B * P, HD, device=DEV, dtype=torch.bfloat16)
    _lib.call("oasis_attention_temporal_cached", past.data_ptr() if Tp else 0, cur.data_ptr(), out.data_ptr(), B, Tp,
              H, _s())
    full = torch.empty(B * T * P, HD, device=DEV, dtype=torch.bfloat16)
    _lib.call("oasis_attention_temporal", qkv.data_ptr(), full.data_ptr(), B, T, H, _s())
    torch.cuda.synchronize()
    assert rel_l2(out.reshape(B, P, HD).float(), full.reshape(B, T, P, HD)[:, Tp].float()) < 1e-2
    x = qkv.float().reshape(B, T, P, 3, H, 64).permute(3, 0, 2, 4, 1, 5)
    ref = _attn_ref(x[0][..., Tp:, :], x[1], x[2], None).permute(0, 3, 1, 2, 4).reshape(B * P, HD)
    assert rel_l2(out.float(), ref) < 1e-2


def test_silu_patch_embed_ddim_bridge_postquant():
    F_ = 6
    c = torch.randn(F_, 1024, device=DEV)
    y = torch.empty(F_, 1024, device=DEV, dtype=torch.bfloat16)
    _lib.call("oasis_silu_bf16", c.data_ptr(), y.data_ptr(), c.numel(), _s())
    torch.cuda.synchronize()
    assert rel_l2(y.float(), F.silu(c)) < 4e-3

    # DDIM update
    chunk = torch.randn(2, 144, 64, device=DEV)
    v = torch.randn(2, 144, 64, device=DEV)
    st = H.ddim_schedule()[1]
    ref = chunk.clone()
    at, an = st.at_sqrt ** 2, st.an_sqrt ** 2
    x0 = math.sqrt(at) * ref - math.sqrt(1 - at) * v
    eps = (math.sqrt(1 / at) * ref - x0) / math.sqrt(1 / at - 1)
    ref = math.sqrt(an) * x0 + math.sqrt(1 - an) * eps
    co = _lib.OasisDdimCoeffs(*st.as_tuple())
    _lib.call("oasis_ddim_update", chunk.data_ptr(), v.data_ptr(), C.byref(co), chunk.numel(), _s())
    torch.cuda.synchronize()
    assert rel_l2(chunk, ref) < 1e-6

    # bridge
    ch = torch.randn(3, 144, 64, device=DEV)
    lat = torch.empty(3, 576, 16, device=DEV)
    _lib.call("oasis_bridge_unpatchify", ch.data_ptr(), lat.data_ptr(), 3, _s())
    torch.cuda.synchronize()
    ref = H.unpatchify(ch.cpu()).permute(0, 2, 3, 1).reshape(3, 576, 16) / H.SCALING_FACTOR
    assert rel_l2(lat, ref) < 1e-6

    # post quant
    w = torch.randn(16, 1024, device=DEV)
    b = torch.randn(1024, device=DEV)
    z = torch.empty(3 * 576, 1024, device=DEV)
    _lib.call("oasis_post_quant", lat.data_ptr(), w.data_ptr(), b.data_ptr(), z.data_ptr(), 3 * 576, _s())
    torch.cuda.synchronize()
    assert rel_l2(z, lat.reshape(-1, 16) @ w + b) < 1e-6
