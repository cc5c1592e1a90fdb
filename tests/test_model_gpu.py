"""End-to-end parity of the frame path (DiT forward, DDIM step, bridge, VAE decode,
full frame) through the C ABI against the CPU fp32 oracle on seeded random-init
weights. Bar (benchmark spec): relative L2 <= 1e-2 and cosine >= 0.999 on every
step's v-prediction and on the decoded frame."""
from __future__ import annotations

import pytest
import torch

from oracle import oasis_oracle as O
from oasis_b200 import engine as E
from oasis_b200 import host as H
from oasis_b200.weights import DitDeviceWeights, VaeDeviceWeights, init_dit_weights, init_vae_weights
from tests.helpers import COS_TOL, REL_L2_TOL, cosine, rel_l2

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.fixture(scope="module")
def dit_small():
    sd = init_dit_weights(seed=1, n_blocks=2, bias_std=0.02)
    return sd, DitDeviceWeights(sd, DEV)


@pytest.fixture(scope="module")
def dit_full():
    sd = init_dit_weights(seed=1)
    return sd, DitDeviceWeights(sd, DEV)


@pytest.fixture(scope="module")
def vae_full():
    sd = init_vae_weights(seed=2, bias_std=0.02, norm_std=0.1)
    return sd, VaeDeviceWeights(sd, DEV)


def _inputs(B, T, seed=0):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(B, T, H.N_PATCHES, H.D_MODEL, generator=g)
    cond = torch.randn(B, T, H.D_MODEL, generator=g)
    return z, cond


@pytest.mark.parametrize("B,T", [(1, 1), (1, 2), (2, 3), (1, 8), (1, 32)])  # T = 32: the RoPE table's last position
def test_dit_forward_small(dit_small, B, T):
    sd, dw = dit_small
    z, cond = _inputs(B, T)
    ref = O.dit_forward(z, cond, sd)
    zg = z.to(DEV)
    v = torch.empty(B, T, H.N_PATCHES, H.OUT_DIM, device=DEV)
    ws = E.workspace(E.dit_workspace_bytes(B, T), DEV)
    E.dit_forward(dw, zg, cond.to(DEV), v, ws, last_frame_only=False)
    assert rel_l2(v, ref) < REL_L2_TOL and cosine(v, ref) > COS_TOL, (rel_l2(v, ref), cosine(v, ref))
    # last-frame-only output is the same rows
    z2 = z.to(DEV)
    v2 = torch.empty(B, H.N_PATCHES, H.OUT_DIM, device=DEV)
    E.dit_forward(dw, z2, cond.to(DEV), v2, ws, last_frame_only=True)
    assert torch.equal(v2, v[:, -1])


def test_dit_forward_full_depth(dit_full):
    """C2: one 16-block step, B=1, T=2."""
    sd, dw = dit_full
    z, cond = _inputs(1, 2, seed=1)
    ref = O.dit_forward(z, cond, sd)[:, -1]
    v = torch.empty(1, H.N_PATCHES, H.OUT_DIM, device=DEV)
    E.dit_forward(dw, z.to(DEV), cond.to(DEV), v, E.workspace(E.dit_workspace_bytes(1, 2), DEV))
    assert rel_l2(v, ref) < REL_L2_TOL and cosine(v, ref) > COS_TOL, (rel_l2(v, ref), cosine(v, ref))


def test_vae_decode_full(vae_full):
    sd, vw = vae_full
    g = torch.Generator().manual_seed(5)
    lat = torch.randn(2, H.VAE_TOKENS, H.VAE_LATENT, generator=g)
    ref = O.vae_decode(lat, sd)
    img = torch.empty(2, 3, 360, 640, device=DEV)
    E.vae_decode(vw, lat.to(DEV), img, E.workspace(E.vae_workspace_bytes(2), DEV))
    assert rel_l2(img, ref) < REL_L2_TOL and cosine(img, ref) > COS_TOL, (rel_l2(img, ref), cosine(img, ref))


def _frame_inputs(sd, B, T, seed):
    g = torch.Generator().manual_seed(seed)
    chunk = H.patchify(torch.randn(B, 16, 18, 32, generator=g).clamp(-H.NOISE_ABS_MAX, H.NOISE_ABS_MAX))
    ctx_lat = torch.randn(B * (T - 1), 16, 18, 32, generator=g)
    ctx_z = O.patch_embed(ctx_lat, sd).reshape(B, T - 1, H.N_PATCHES, H.D_MODEL).contiguous()
    actions = torch.zeros(B, 25)
    actions[torch.arange(B), torch.randint(0, 25, (B,), generator=g)] = 1
    steps = H.ddim_schedule()
    conds = []
    for st in steps:
        c_ctx = O.cond_vector(torch.full((B * (T - 1),), H.STABILIZATION_LEVEL - 1), None, sd).reshape(B, T - 1, -1)
        c_gen = O.cond_vector(torch.full((B,), st.noise_level), actions, sd).reshape(B, 1, -1)
        conds.append(torch.cat([c_ctx, c_gen], 1))
    return chunk, ctx_z, conds, steps


def test_frame_c3(dit_full, vae_full):
    """C3: one frame, B=1, T=2: 4 DDIM steps + VAE decode. Each step's
    v-prediction (the DiT forward on the step's own input) meets rel-L2 <= 1e-2
    and cosine >= 0.999 against the oracle's; the step itself goes through
    oasis_ddim_step and must equal ddim_update(chunk, that v)."""
    dsd, dw = dit_full
    vsd, vw = vae_full
    B, T = 1, 2
    chunk, ctx_z, conds, steps = _frame_inputs(dsd, B, T, seed=2)
    fe = E.FrameEngine(dw, vw, B, T, steps)
    fe.chunk.copy_(chunk)
    fe.context_z.copy_(ctx_z)
    for i, c in enumerate(conds):
        fe.cond[i].copy_(c)
    c_ref = chunk.clone()
    step_ws = E.workspace(E.step_workspace_bytes(B, T), DEV)
    dit_ws = E.workspace(E.dit_workspace_bytes(B, T), DEV)
    z = torch.empty(B, T, H.N_PATCHES, H.D_MODEL, device=DEV)
    v = torch.empty(B, H.N_PATCHES, H.OUT_DIM, device=DEV)
    for i, st in enumerate(steps):
        c_ref, v_ref = O.ddim_step(c_ref, ctx_z, conds[i], st.at_sqrt ** 2, st.an_sqrt ** 2, dsd)
        z[:, :T - 1].copy_(fe.context_z)
        E.patch_embed(dw, fe.chunk.reshape(-1, H.OUT_DIM), z, T * H.N_PATCHES, (T - 1) * H.N_PATCHES)
        E.dit_forward(dw, z, fe.cond[i], v, dit_ws, last_frame_only=True)
        expect = fe.chunk.clone()
        E.ddim_update(expect, v, st)
        E.ddim_step(dw, fe.chunk, fe.context_z, fe.cond[i], st, step_ws)
        torch.cuda.synchronize()
        assert rel_l2(v, v_ref) < REL_L2_TOL and cosine(v, v_ref) > COS_TOL, (i, rel_l2(v, v_ref), cosine(v, v_ref))
        assert rel_l2(fe.chunk, expect) < 1e-5, (i, rel_l2(fe.chunk, expect))
        assert rel_l2(fe.chunk, c_ref) < REL_L2_TOL, (i, rel_l2(fe.chunk, c_ref))
    img_ref = O.vae_decode(O.bridge(c_ref), vsd)
    fe.run_decode()
    torch.cuda.synchronize()
    assert rel_l2(fe.image, img_ref) < REL_L2_TOL and cosine(fe.image, img_ref) > COS_TOL


def test_frame_graph_replay_matches_eager(dit_full, vae_full):
    """The CUDA-graph frame equals the eagerly launched frame bit for bit."""
    dsd, dw = dit_full
    vsd, vw = vae_full
    B, T = 2, 3
    chunk, ctx_z, conds, steps = _frame_inputs(dsd, B, T, seed=3)
    fe = E.FrameEngine(dw, vw, B, T, steps)
    fe.context_z.copy_(ctx_z)
    for i, c in enumerate(conds):
        fe.cond[i].copy_(c)
    fe.chunk.copy_(chunk)
    fe.run()
    torch.cuda.synchronize()
    eager_img, eager_chunk = fe.image.clone(), fe.chunk.clone()
    fe.chunk.copy_(chunk)
    fe.capture()  # runs once eagerly as warm-up, then captures
    fe.chunk.copy_(chunk)
    fe.replay()
    torch.cuda.synchronize()
    assert torch.equal(fe.chunk, eager_chunk)
    assert torch.equal(fe.image, eager_img)


def test_device_error_word_clear():
    from oasis_b200 import _lib

    assert _lib.load().oasis_device_error(1) == 0


def test_graft_smoke():
    """The driver's smoke check (one small DDIM step + VAE decode vs the oracle)."""
    import __graft_entry__

    __graft_entry__.smoke()


def test_generate_frame_matches_per_step_path(dit_full, vae_full):
    """oasis_generate_frame (all adaLN tables from one GEMM) equals the frame built
    from oasis_ddim_step calls + bridge + decode, and the oracle."""
    dsd, dw = dit_full
    vsd, vw = vae_full
    B, T = 2, 3
    chunk, ctx_z, conds, steps = _frame_inputs(dsd, B, T, seed=4)
    fe = E.FrameEngine(dw, vw, B, T, steps)
    fe.context_z.copy_(ctx_z)
    for i, c in enumerate(conds):
        fe.cond[i].copy_(c)
    fe.chunk.copy_(chunk)
    fe.run()
    torch.cuda.synchronize()
    frame_chunk, frame_img = fe.chunk.clone(), fe.image.clone()
    fe.chunk.copy_(chunk)
    fe.run_steps_separately()
    fe.run_decode()
    torch.cuda.synchronize()
    assert rel_l2(frame_chunk, fe.chunk) < 1e-5
    assert rel_l2(frame_img, fe.image) < 1e-5
    c_ref = chunk.clone()
    for i, st in enumerate(steps):
        c_ref, _ = O.ddim_step(c_ref, ctx_z, conds[i], st.at_sqrt ** 2, st.an_sqrt ** 2, dsd)
    img_ref = O.vae_decode(O.bridge(c_ref), vsd)
    assert rel_l2(frame_chunk, c_ref) < REL_L2_TOL
    assert rel_l2(frame_img, img_ref) < REL_L2_TOL and cosine(frame_img, img_ref) > COS_TOL


@pytest.mark.parametrize("B,T", [(2, 3), (1, 2), (1, 1)])
def test_kv_cached_forward_matches_full_T(dit_small, B, T):
    """precompute_past + forward_current (context rows once) equals the full-T
    forward's last frame, and the oracle."""
    sd, dw = dit_small
    z, cond = _inputs(B, T, seed=7)
    ref = O.dit_forward(z, cond, sd)[:, -1]
    v_full = torch.empty(B, H.N_PATCHES, H.OUT_DIM, device=DEV)
    E.dit_forward(dw, z.to(DEV), cond.to(DEV), v_full, E.workspace(E.dit_workspace_bytes(B, T), DEV))
    Tp = T - 1
    ws = E.workspace(E.dit_workspace_bytes(B, max(Tp, 1)), DEV)
    cache = E.kv_cache(B, Tp, DEV) if Tp else None
    if Tp:
        E.dit_precompute_past(dw, z[:, :Tp].contiguous().to(DEV), cond[:, :Tp].contiguous().to(DEV), cache, ws)
    v = torch.empty(B, H.N_PATCHES, H.OUT_DIM, device=DEV)
    E.dit_forward_current(dw, z[:, Tp].contiguous().to(DEV), cond[:, Tp].contiguous().to(DEV), cache, Tp, v, ws)
    torch.cuda.synchronize()
    assert rel_l2(v, v_full) < 5e-3, rel_l2(v, v_full)  # different softmax orders (bf16 outputs)
    assert rel_l2(v, ref) < REL_L2_TOL and cosine(v, ref) > COS_TOL


@pytest.mark.parametrize("B,T", [(2, 3), (1, 2)])
def test_generate_frame_kv_matches_full_T(dit_full, vae_full, B, T):
    """C3-style frame through oasis_generate_frame_kv equals oasis_generate_frame
    and the oracle (every step's chunk and the decoded frame)."""
    dsd, dw = dit_full
    vsd, vw = vae_full
    chunk, ctx_z, conds, steps = _frame_inputs(dsd, B, T, seed=8)
    out = {}
    for kv in (False, True):
        fe = E.FrameEngine(dw, vw, B, T, steps, kv=kv)
        fe.context_z.copy_(ctx_z)
        for i, c in enumerate(conds):
            fe.cond[i].copy_(c)
        fe.chunk.copy_(chunk)
        fe.run()
        torch.cuda.synchronize()
        out[kv] = (fe.chunk.clone(), fe.image.clone())
    # the two paths differ only in the temporal softmax order (bf16 outputs)
    assert rel_l2(out[True][0], out[False][0]) < 5e-3, rel_l2(out[True][0], out[False][0])
    assert rel_l2(out[True][1], out[False][1]) < 5e-3, rel_l2(out[True][1], out[False][1])
    c_ref = chunk.clone()
    for i, st in enumerate(steps):
        c_ref, _ = O.ddim_step(c_ref, ctx_z, conds[i], st.at_sqrt ** 2, st.an_sqrt ** 2, dsd)
    img_ref = O.vae_decode(O.bridge(c_ref), vsd)
    assert rel_l2(out[True][0], c_ref) < REL_L2_TOL
    assert rel_l2(out[True][1], img_ref) < REL_L2_TOL and cosine(out[True][1], img_ref) > COS_TOL


def test_dropin_kv_functions(dit_small):
    """oasis_inference.precompute_past_state / dit_forward_currentonly under the
    reference's names give dit_forward_device's last-frame rows."""
    from oasis_b200 import oasis_inference as OI

    sd, dw = dit_small
    T = 2
    z, cond = _inputs(1, T, seed=9)
    scr = OI.prealloc_scratch(DEV, n_frames=T)
    full = OI.dit_forward_device(z.reshape(-1, H.D_MODEL).to(DEV), [c for c in cond[0].to(DEV)], dw, scr)
    OI.precompute_past_state(z[0, 0].to(DEV), cond[0, 0].to(DEV), dw, scr)
    v = OI.dit_forward_currentonly(z[0, 1].to(DEV), cond[0, 1].to(DEV), dw, scr)
    torch.cuda.synchronize()
    assert rel_l2(v, full[H.N_PATCHES:]) < 5e-3


@pytest.fixture(scope="module")
def video_case(dit_full, vae_full):
    """Inputs of a 3-frame loop (B=1, T=3) and the oracle's frames and final windows."""
    dsd, _ = dit_full
    vsd, _ = vae_full
    B, T, F_ = 1, 3, 3
    g = torch.Generator().manual_seed(11)
    steps = H.ddim_schedule()
    ctx_lat = torch.randn(B * (T - 1), 16, 18, 32, generator=g)
    ctx_z = O.patch_embed(ctx_lat, dsd).reshape(B, T - 1, H.N_PATCHES, H.D_MODEL).contiguous()
    noise = H.patchify(torch.randn(F_ * B, 16, 18, 32, generator=g).clamp(-H.NOISE_ABS_MAX, H.NOISE_ABS_MAX))
    noise = noise.reshape(F_, B, H.N_PATCHES, H.OUT_DIM)
    acts = torch.zeros(F_, B, 25)
    acts[..., 3] = 1
    ctx_cond = O.cond_vector(torch.full((B * (T - 1),), H.STABILIZATION_LEVEL - 1), None, dsd).reshape(B, T - 1, -1)
    gen_conds = torch.stack([torch.stack([O.cond_vector(torch.full((B,), st.noise_level), acts[f], dsd)
                                          for st in steps]) for f in range(F_)])  # [F, S, B, D]
    new_ctx = torch.stack([O.cond_vector(torch.full((B,), H.STABILIZATION_LEVEL - 1), acts[f], dsd)
                           for f in range(F_)])  # [F, B, D]
    coeffs = [{"at": st.at_sqrt ** 2, "an": st.an_sqrt ** 2} for st in steps]
    ref = O.generate_video(noise, ctx_z, ctx_cond, gen_conds, new_ctx, coeffs, dsd, vsd)
    return dict(B=B, T=T, F=F_, steps=steps, ctx_z=ctx_z, ctx_cond=ctx_cond, noise=noise, gen_conds=gen_conds,
                new_ctx=new_ctx, ref=ref)


@pytest.mark.parametrize("kv", [False, True])
def test_video_loop_matches_oracle(dit_full, vae_full, video_case, kv):
    """Three frames of the autoregressive loop (context window rolled on the
    device, graph-replayed; full-T and context-cached frames) against the
    oracle's loop: every decoded frame and the final windows."""
    _, dw = dit_full
    _, vw = vae_full
    c = video_case
    ref_imgs, cz, cc = c["ref"]
    ve = E.VideoEngine(dw, vw, c["B"], c["T"], c["steps"], kv=kv)
    ve.capture()
    ve.set_context(c["ctx_z"].to(DEV), c["ctx_cond"].to(DEV))
    for f in range(c["F"]):
        img = ve.step(c["noise"][f].to(DEV), c["gen_conds"][f].to(DEV), c["new_ctx"][f].to(DEV))
        torch.cuda.synchronize()
        assert rel_l2(img, ref_imgs[f]) < REL_L2_TOL and cosine(img, ref_imgs[f]) > COS_TOL, (f, rel_l2(img, ref_imgs[f]))
    assert rel_l2(ve.context_z, cz) < REL_L2_TOL
    assert torch.allclose(ve.ctx_cond.cpu(), cc, atol=1e-5)
