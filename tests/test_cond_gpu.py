"""Frame conditioning on the GPU (oasis_compute_cond) and the video loop that
computes it inside its frame graph.

compute_cond_for_frame (oasis_inference.py:1406-1427) runs on the host in fp32 in
the reference; here it is two fp32 CUDA-core kernels. Pinned against the
reference's own function (golden fixture from make_golden.py) and against the
host restatement on random levels and actions; the video loop with on-device
conditioning is checked against the oracle's loop frame by frame."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oasis_oracle as O
from oasis_b200 import engine as E
from oasis_b200 import host as H
from oasis_b200.weights import CondDeviceWeights, DitDeviceWeights, VaeDeviceWeights, init_dit_weights, init_vae_weights
from tests.golden.make_golden import cond_weights
from tests.helpers import COS_TOL, GOLDEN, REL_L2_TOL, cosine, rel_l2

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _golden_sd():
    dev = cond_weights()
    return {"t_embedder.mlp.0.weight": dev["t_emb_w0_host"].T, "t_embedder.mlp.0.bias": dev["t_emb_b0_host"],
            "t_embedder.mlp.2.weight": dev["t_emb_w2_host"].T, "t_embedder.mlp.2.bias": dev["t_emb_b2_host"],
            "external_cond.weight": dev["ext_cond_w_host"].T, "external_cond.bias": dev["ext_cond_b_host"]}


def _cond(cw, levels, actions=None):
    lv = torch.as_tensor(levels, dtype=torch.float32).to(DEV)
    out = torch.empty(lv.numel(), H.D_MODEL, device=DEV)
    ws = E.workspace(E.cond_workspace_bytes(lv.numel()), DEV)
    E.compute_cond(cw, lv, out, ws, None if actions is None else actions.to(DEV))
    torch.cuda.synchronize()
    return out.cpu()


def test_compute_cond_matches_reference_fixture():
    g = np.load(GOLDEN)
    cw = CondDeviceWeights(_golden_sd(), DEV)
    np.testing.assert_allclose(_cond(cw, [14.0])[0].numpy(), g["cond_t14_noaction"], atol=1e-5)
    act = torch.zeros(1, 25)
    act[0, 11] = 1
    np.testing.assert_allclose(_cond(cw, [999.0], act)[0].numpy(), g["cond_t999_walk"], atol=1e-5)


@pytest.mark.parametrize("n,a_rows", [(1, 1), (7, 7), (2048, 512), (100, 25)])
def test_compute_cond_matches_host(n, a_rows):
    sd = init_dit_weights(seed=5, n_blocks=1)
    cw = CondDeviceWeights(sd, DEV)
    gen = torch.Generator().manual_seed(n)
    levels = torch.randint(0, 1000, (n,), generator=gen).float()
    acts = torch.zeros(a_rows, 25)
    acts[torch.arange(a_rows), torch.randint(0, 25, (a_rows,), generator=gen)] = 1
    acts[0] = torch.rand(25, generator=gen)  # dense rows work too
    got = _cond(cw, levels, acts)
    ref = H.compute_cond(levels, acts[torch.arange(n) % a_rows], sd)
    assert rel_l2(got, ref) < 1e-5, rel_l2(got, ref)
    got0 = _cond(cw, levels)  # no action term
    ref0 = H.compute_cond(levels, None, sd)
    assert rel_l2(got0, ref0) < 1e-5


def test_frame_engine_device_cond_fills_the_frame_table():
    sd = init_dit_weights(seed=6, n_blocks=1)
    dw = DitDeviceWeights(sd, DEV)
    vw = VaeDeviceWeights(init_vae_weights(seed=6, n_blocks=1), DEV)
    B, T = 3, 4
    fe = E.FrameEngine(dw, vw, B, T, device_cond=True)
    gen = torch.Generator().manual_seed(0)
    acts = torch.zeros(B, T, 25)
    acts.view(-1, 25)[torch.arange(B * T), torch.randint(0, 25, (B * T,), generator=gen)] = 1
    fe.actions.copy_(acts)
    fe.run_cond()
    torch.cuda.synchronize()
    for i, st in enumerate(fe.steps):
        lv = torch.full((B, T), float(H.STABILIZATION_LEVEL - 1))
        lv[:, -1] = st.noise_level
        ref = H.compute_cond(lv.reshape(-1), acts.reshape(-1, 25), sd).reshape(B, T, -1)
        assert rel_l2(fe.cond[i], ref) < 1e-5, (i, rel_l2(fe.cond[i], ref))


@pytest.mark.parametrize("kv", [False, True])
def test_video_loop_with_device_cond_matches_oracle(kv):
    """Three frames (B=2, T=3) of the loop with the conditioning computed in the
    frame graph from actions, against the oracle's loop with host conditioning."""
    dsd = init_dit_weights(seed=1)
    vsd = init_vae_weights(seed=2, bias_std=0.02, norm_std=0.1)
    dw, vw = DitDeviceWeights(dsd, DEV), VaeDeviceWeights(vsd, DEV)
    B, T, F_ = 2, 3, 3
    steps = H.ddim_schedule()
    g = torch.Generator().manual_seed(12)
    ctx_lat = torch.randn(B * (T - 1), 16, 18, 32, generator=g)
    ctx_z = O.patch_embed(ctx_lat, dsd).reshape(B, T - 1, H.N_PATCHES, H.D_MODEL).contiguous()
    noise = H.patchify(torch.randn(F_ * B, 16, 18, 32, generator=g).clamp(-H.NOISE_ABS_MAX, H.NOISE_ABS_MAX))
    noise = noise.reshape(F_, B, H.N_PATCHES, H.OUT_DIM)
    ctx_acts = torch.zeros(B, T - 1, 25)
    ctx_acts[:, :, 7] = 1
    acts = torch.zeros(F_, B, 25)
    acts.view(-1, 25)[torch.arange(F_ * B), torch.randint(0, 25, (F_ * B,), generator=g)] = 1
    stab = H.STABILIZATION_LEVEL - 1
    ctx_cond = O.cond_vector(torch.full((B * (T - 1),), stab), ctx_acts.reshape(-1, 25), dsd).reshape(B, T - 1, -1)
    gen_conds = torch.stack([torch.stack([O.cond_vector(torch.full((B,), st.noise_level), acts[f], dsd)
                                          for st in steps]) for f in range(F_)])
    new_ctx = torch.stack([O.cond_vector(torch.full((B,), stab), acts[f], dsd) for f in range(F_)])
    coeffs = [{"at": st.at_sqrt ** 2, "an": st.an_sqrt ** 2} for st in steps]
    ref_imgs, cz, _ = O.generate_video(noise, ctx_z, ctx_cond, gen_conds, new_ctx, coeffs, dsd, vsd)

    ve = E.VideoEngine(dw, vw, B, T, steps, kv=kv, device_cond=True)
    ve.capture()
    ve.set_context(ctx_z.to(DEV), ctx_acts.to(DEV))
    for f in range(F_):
        img = ve.step_actions(noise[f], acts[f])
        torch.cuda.synchronize()
        assert rel_l2(img, ref_imgs[f]) < REL_L2_TOL and cosine(img, ref_imgs[f]) > COS_TOL, (f, rel_l2(img, ref_imgs[f]))
    assert rel_l2(ve.context_z, cz) < REL_L2_TOL
    # the action window rolled with the frames: the last T-1 actions
    assert torch.equal(ve.ctx_actions.cpu(), acts[F_ - (T - 1):].transpose(0, 1))
