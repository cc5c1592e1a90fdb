"""Parity at the configurations the benchmark times, against the CPU fp32 oracle.

C4 (bench.py's workload): 64 sessions x T = 8, full 16-block DiT + 12-block VAE,
M = 73 728 token rows, so every projection runs on the CTA-pair GEMM and the
temporal attention on its T = 8 kernel. Sessions 0, 31 and 63 are checked
against the oracle run at B = 1 on the same per-session seeds:
  - each DDIM step's v-prediction (the GPU and the oracle each follow their own
    trajectory), rel-L2 <= 1e-2 and cosine >= 0.999;
  - the decoded frame after the 4 steps;
  - the whole frame as the benchmark runs it (FrameEngine, one CUDA graph with
    the conditioning computed on the GPU from the action window).
C5: 16 sessions x T = 32 (M = 73 728, the long-T temporal kernel), one full-depth
DiT forward, sessions 0 and 15 against the oracle.

Reference: ddim_step_fn / dit_forward_device / vae_decode_forward
(oasis_inference.py:1909-1932, 1438-1526, 1546-1618)."""
from __future__ import annotations

import pytest
import torch

import bench
from oracle import oasis_oracle as O
from oasis_b200 import engine as E
from oasis_b200 import host as H
from oasis_b200.weights import DitDeviceWeights, VaeDeviceWeights, init_dit_weights, init_vae_weights
from tests.helpers import COS_TOL, REL_L2_TOL, cosine, rel_l2

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
C4_SESSIONS = (0, 31, 63)


def _ok(a, b):
    return rel_l2(a, b) < REL_L2_TOL and cosine(a, b) > COS_TOL


@pytest.fixture(scope="module")
def c4_weights():
    dsd, vsd = init_dit_weights(seed=0), init_vae_weights(seed=0)  # bench.py's weights
    return dsd, vsd, DitDeviceWeights(dsd, DEV), VaeDeviceWeights(vsd, DEV)


def _session_context(T, s):
    """The context latents bench.make_inputs draws for session seed s."""
    g = torch.Generator().manual_seed(s)
    torch.randn(16, 18, 32, generator=g)  # the noise chunk comes first
    return torch.randn(T - 1, 16, 18, 32, generator=g)


def test_c4_bench_frame_matches_oracle(c4_weights):
    dsd, vsd, dw, vw = c4_weights
    B, T = 64, 8
    fe = E.FrameEngine(dw, vw, B, T, device_cond=True)  # as bench.py: conditioning inside the frame graph
    chunk0, ctx_z, conds, _ = bench.make_inputs(fe, dw, 0, B, T)
    steps = fe.steps
    idx = list(C4_SESSIONS)

    # oracle inputs of the checked sessions, from the same seeds
    ctx_ref = torch.stack([O.patch_embed(_session_context(T, s), dsd) for s in idx])
    assert rel_l2(ctx_z[idx], ctx_ref) < 1e-5  # the GPU patch embed of the context frames
    c_ref = chunk0[idx].clone()
    cond_ref = conds[:, idx]

    # GPU: each step through dit_forward (the bench's M = 73728 kernels) + ddim_update
    z = torch.empty(B, T, H.N_PATCHES, H.D_MODEL, device=DEV)
    v = torch.empty(B, H.N_PATCHES, H.OUT_DIM, device=DEV)
    chunk = chunk0.to(DEV)
    ctx_dev = ctx_z.to(DEV)
    ws = E.workspace(E.dit_workspace_bytes(B, T), DEV)
    for i, st in enumerate(steps):
        z[:, :T - 1].copy_(ctx_dev)
        E.patch_embed(dw, chunk.reshape(-1, H.OUT_DIM), z, T * H.N_PATCHES, (T - 1) * H.N_PATCHES)
        E.dit_forward(dw, z, conds[i].to(DEV), v, ws, last_frame_only=True)
        E.ddim_update(chunk, v, st)
        torch.cuda.synchronize()
        c_ref, v_ref = O.ddim_step(c_ref, ctx_ref, cond_ref[i], st.at_sqrt ** 2, st.an_sqrt ** 2, dsd)
        for j, s in enumerate(idx):
            assert _ok(v[s], v_ref[j]), (i, s, rel_l2(v[s], v_ref[j]), cosine(v[s], v_ref[j]))
    for j, s in enumerate(idx):
        assert rel_l2(chunk[s], c_ref[j]) < REL_L2_TOL, (s, rel_l2(chunk[s], c_ref[j]))
    del z, ws
    img_ref = O.vae_decode(O.bridge(c_ref), vsd)

    # the benchmark's frame: one CUDA graph over all 64 sessions
    fe.chunk.copy_(chunk0)
    fe.capture()
    fe.chunk.copy_(chunk0)
    fe.replay()
    torch.cuda.synchronize()
    for j, s in enumerate(idx):
        assert rel_l2(fe.chunk[s], chunk[s]) < 5e-3, (s, rel_l2(fe.chunk[s], chunk[s]))
        assert rel_l2(fe.chunk[s], c_ref[j]) < REL_L2_TOL
        assert _ok(fe.image[s], img_ref[j]), (s, rel_l2(fe.image[s], img_ref[j]), cosine(fe.image[s], img_ref[j]))


def test_c5_long_context_forward_matches_oracle():
    S, T = 16, 32
    sd = init_dit_weights(seed=3)
    dw = DitDeviceWeights(sd, DEV)
    g = torch.Generator().manual_seed(3)
    z0 = torch.randn(S, T, H.N_PATCHES, H.D_MODEL, generator=g)
    cond = torch.randn(S, T, H.D_MODEL, generator=g)
    v = torch.empty(S, T, H.N_PATCHES, H.OUT_DIM, device=DEV)
    E.dit_forward(dw, z0.to(DEV), cond.to(DEV), v, E.workspace(E.dit_workspace_bytes(S, T), DEV),
                  last_frame_only=False)
    torch.cuda.synchronize()
    for s in (0, S - 1):
        ref = O.dit_forward(z0[s:s + 1], cond[s:s + 1], sd)[0]
        assert _ok(v[s], ref), (s, rel_l2(v[s], ref), cosine(v[s], ref))
        assert _ok(v[s, -1], ref[-1]), s  # the generated frame's rows alone
