"""Host-side pieces of the frame path that stay Python (fp32, CPU), as in the
reference: model constants, timestep conditioning, the beta schedule and DDIM
coefficients, RoPE frequency tables, and patchify helpers.

Reference anchors (zoecarver/open-oasis, oasis_inference.py):
  constants            :90-150
  timestep_embedding   :307-311
  sigmoid_beta_schedule:313-321
  RoPE freqs           :344-373 (spatial axial, temporal)
  compute_cond_for_frame :1406-1427
  DDIM coefficients    :1843-1860, schedule :1763-1771
  patchify / unpatchify:958-969
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

# --- model constants (oasis_inference.py:90-150) ---------------------------
D_MODEL = 1024
N_HEADS = 16
D_HEAD = 64
D_MLP = 4096
N_BLOCKS = 16
PATCH_SIZE = 2
IN_CHANNELS = 16
INPUT_H, INPUT_W = 18, 32
FRAME_H, FRAME_W = INPUT_H // PATCH_SIZE, INPUT_W // PATCH_SIZE  # 9, 16
N_PATCHES = FRAME_H * FRAME_W  # 144 (the reference pads to 160; this build does not)
FREQ_DIM = 256
EXT_COND_DIM = 25
OUT_DIM = PATCH_SIZE * PATCH_SIZE * IN_CHANNELS  # 64
SCALING_FACTOR = 0.07843137255
MAX_T = 32

VAE_DEPTH = 12
VAE_ENC_DEPTH = 6  # encoder depth for random init; a checkpoint's encoder.* keys set the real one
VAE_ENC_K = 1216  # patch_embed GEMM depth: 1200 pixels zero-padded to a multiple of 64
VAE_DIM = 1024
VAE_HEADS = 16
VAE_LATENT = 16
VAE_PATCH = 20
VAE_PATCH_DIM = 3 * VAE_PATCH ** 2  # 1200
VAE_H, VAE_W = 18, 32
VAE_TOKENS = VAE_H * VAE_W  # 576
VAE_ROT_DIM = 32  # first 32 of each head's 64 dims are rotated

MAX_NOISE_LEVEL = 1000
DDIM_STEPS = 4
NOISE_ABS_MAX = 20.0
STABILIZATION_LEVEL = 15  # context frames are conditioned at t = 14


# --- conditioning -----------------------------------------------------------
def timestep_freqs(dim: int = FREQ_DIM, max_period: float = 10000.0) -> torch.Tensor:
    """The embedding's frequencies exp(-ln(max_period) i / (dim/2)), i < dim/2 (fp32)."""
    half = dim // 2
    return torch.exp(-math.log(max_period) * torch.arange(0, half, dtype=torch.float32) / half)


def timestep_embedding(t: torch.Tensor, dim: int = FREQ_DIM, max_period: float = 10000.0) -> torch.Tensor:
    """[cos | sin] sinusoidal embedding, freqs exp(-ln(max_period) i / (dim/2))."""
    freqs = timestep_freqs(dim, max_period)
    args = t[:, None].float() * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


def compute_cond(t_levels: torch.Tensor, actions: torch.Tensor | None, w: dict) -> torch.Tensor:
    """cond = t_mlp(timestep_embedding(t)) + external_cond(action), fp32 on the host.

    t_levels: (N,) integer noise levels; actions: (N, 25) or None; w: reference-keyed
    fp32 state dict. Returns (N, 1024).
    """
    e = timestep_embedding(t_levels.reshape(-1))
    h = e @ w["t_embedder.mlp.0.weight"].T + w["t_embedder.mlp.0.bias"]
    h = h * torch.sigmoid(h)
    cond = h @ w["t_embedder.mlp.2.weight"].T + w["t_embedder.mlp.2.bias"]
    if actions is not None:
        cond = cond + actions.float() @ w["external_cond.weight"].T + w["external_cond.bias"]
    return cond.float()


# --- schedule ---------------------------------------------------------------
def linear_beta_schedule(timesteps: int = MAX_NOISE_LEVEL, start: float = 1e-4, end: float = 2e-2) -> torch.Tensor:
    """Linear betas (the schedule BASELINE names; endpoints are the DDPM defaults)."""
    return torch.linspace(start, end, timesteps, dtype=torch.float64)


def sigmoid_beta_schedule(timesteps: int = MAX_NOISE_LEVEL, start: float = -3, end: float = 3, tau: float = 1,
                          clamp_min: float = 1e-5) -> torch.Tensor:
    """The reference's own schedule (oasis_inference.py:313-321), kept as an option."""
    steps = timesteps + 1
    t = torch.linspace(0, timesteps, steps, dtype=torch.float64) / timesteps
    v_start = torch.tensor(start / tau).sigmoid()
    v_end = torch.tensor(end / tau).sigmoid()
    ac = (-((t * (end - start) + start) / tau).sigmoid() + v_end) / (v_end - v_start)
    ac = ac / ac[0]
    betas = 1 - (ac[1:] / ac[:-1])
    return torch.clip(betas, 0, 0.999)


@dataclass
class DdimStep:
    noise_level: int
    at_sqrt: float
    one_minus_at_sqrt: float
    inv_at_sqrt: float
    inv_sigma: float
    an_sqrt: float
    one_minus_an_sqrt: float

    def as_tuple(self):
        return (self.at_sqrt, self.one_minus_at_sqrt, self.inv_at_sqrt, self.inv_sigma, self.an_sqrt,
                self.one_minus_an_sqrt)


def ddim_schedule(steps: int = DDIM_STEPS, schedule: str = "linear") -> list[DdimStep]:
    """Per-step DDIM coefficients, highest noise first (oasis_inference.py:1843-1860).

    noise_range = linspace(-1, 999, steps + 1); step i uses t = noise_range[steps - i]
    and t_next = noise_range[steps - i - 1]; the last step decodes to alpha_next = 1.
    """
    betas = linear_beta_schedule() if schedule == "linear" else sigmoid_beta_schedule()
    alphas_cumprod = torch.cumprod(1.0 - betas.float(), dim=0)
    noise_range = torch.linspace(-1, MAX_NOISE_LEVEL - 1, steps + 1)
    out = []
    for noise_idx in reversed(range(1, steps + 1)):
        t = int(noise_range[noise_idx].item())
        t_next = int(noise_range[noise_idx - 1].item())
        at = float(alphas_cumprod[t].item())
        an = float(alphas_cumprod[max(t_next, 0)].item())
        if noise_idx == 1:
            an = 1.0
        out.append(DdimStep(t, at ** 0.5, (1 - at) ** 0.5, (1.0 / at) ** 0.5, 1.0 / ((1.0 / at - 1) ** 0.5),
                            an ** 0.5, (1 - an) ** 0.5))
    return out


# --- RoPE -------------------------------------------------------------------
def default_spatial_freqs() -> torch.Tensor:
    """16 'pixel' frequencies, linspace(1, max_freq/2, 16) * pi with max_freq 256
    (rotary-embedding-torch's pixel init). Stands in for the learned
    blocks.0.s_attn.rotary_emb.freqs, which the random-init model does not have."""
    return torch.linspace(1.0, 128.0, 16) * math.pi


def default_temporal_freqs() -> torch.Tensor:
    """32 'lang' frequencies 1 / 10000^(2i/64) (stands in for t_attn.rotary_emb.freqs)."""
    return 1.0 / (10000.0 ** (torch.arange(0, 64, 2).float() / 64))


def default_vae_freqs() -> torch.Tensor:
    """8 pixel frequencies per axis for the VAE's 2D RoPE (linspace(1, 32, 8) * pi)."""
    return torch.linspace(1.0, 32.0, 8) * math.pi


def _repeat2(x: torch.Tensor) -> torch.Tensor:
    return x.repeat_interleave(2, dim=-1)


def spatial_rope_angles(freqs: torch.Tensor) -> torch.Tensor:
    """(144, 64) axial angles: dims 0..31 from h in linspace(-1,1,9), 32..63 from w
    in linspace(-1,1,16); each frequency repeated for its (even, odd) pair."""
    h = _repeat2(torch.einsum("i,f->if", torch.linspace(-1, 1, FRAME_H), freqs))  # (9, 32)
    w = _repeat2(torch.einsum("i,f->if", torch.linspace(-1, 1, FRAME_W), freqs))  # (16, 32)
    ang = torch.cat([h[:, None, :].expand(FRAME_H, FRAME_W, -1), w[None, :, :].expand(FRAME_H, FRAME_W, -1)], -1)
    return ang.reshape(N_PATCHES, 64)


def temporal_rope_angles(freqs: torch.Tensor, max_t: int = MAX_T) -> torch.Tensor:
    """(max_t, 64) angles for frame positions 0..max_t-1."""
    return _repeat2(torch.einsum("i,f->if", torch.arange(max_t, dtype=torch.float32), freqs))


def vae_rope_angles(freqs: torch.Tensor) -> torch.Tensor:
    """(576, 32) axial pixel angles over the 18 x 32 token grid (16 dims per axis)."""
    h = _repeat2(torch.einsum("i,f->if", torch.linspace(-1, 1, VAE_H), freqs))  # (18, 16)
    w = _repeat2(torch.einsum("i,f->if", torch.linspace(-1, 1, VAE_W), freqs))  # (32, 16)
    ang = torch.cat([h[:, None, :].expand(VAE_H, VAE_W, -1), w[None, :, :].expand(VAE_H, VAE_W, -1)], -1)
    return ang.reshape(VAE_TOKENS, VAE_ROT_DIM)


def rope_quad_table(angles: torch.Tensor, pairs: int = 32) -> torch.Tensor:
    """The layout the GEMM's RoPE epilogue reads: (pairs / 2, positions, 4) with
    (cos, sin) of pairs 2q and 2q + 1 at [q, pos]. Threads of a warp hold
    consecutive rows, i.e. consecutive (or equal) positions, so each table load
    of a warp is one contiguous run."""
    tab = rope_pair_table(angles, pairs)  # (pos, pairs, 2)
    pos = tab.shape[0]
    return tab.reshape(pos, pairs // 2, 4).permute(1, 0, 2).contiguous()


def rope_pair_table(angles: torch.Tensor, pairs: int = 32) -> torch.Tensor:
    """(positions, pairs, 2) (cos, sin) per head-dim pair as the kernels read it.
    Pairs beyond the rotated dims get (1, 0)."""
    pos = angles.shape[0]
    a = angles[:, 0::2].double()  # one angle per (even, odd) pair
    tab = torch.zeros(pos, pairs, 2, dtype=torch.float64)
    tab[:, :, 0] = 1.0
    tab[:, : a.shape[1], 0] = torch.cos(a)
    tab[:, : a.shape[1], 1] = torch.sin(a)
    return tab.float().contiguous()


# --- patch layouts (oasis_inference.py:958-969, 1636-1645) ------------------
def patchify(latent: torch.Tensor) -> torch.Tensor:
    """(..., 16, 18, 32) latent -> (..., 144, 64) patches in (p, q, c) order."""
    lead = latent.shape[:-3]
    x = latent.reshape(*lead, IN_CHANNELS, FRAME_H, PATCH_SIZE, FRAME_W, PATCH_SIZE)
    x = x.movedim(-5, -1)  # (..., h, p, w, q, c)
    x = x.transpose(-4, -3)  # (..., h, w, p, q, c)
    return x.reshape(*lead, N_PATCHES, OUT_DIM)


def unpatchify(patches: torch.Tensor) -> torch.Tensor:
    """(..., 144, 64) -> (..., 16, 18, 32); inverse of patchify."""
    lead = patches.shape[:-2]
    x = patches.reshape(*lead, FRAME_H, FRAME_W, PATCH_SIZE, PATCH_SIZE, IN_CHANNELS)
    x = x.transpose(-4, -3)  # (..., h, p, w, q, c)
    x = x.movedim(-1, -5)  # (..., c, h, p, w, q)
    return x.reshape(*lead, IN_CHANNELS, INPUT_H, INPUT_W)


def patch_embed_matrix(conv_w: torch.Tensor) -> torch.Tensor:
    """x_embedder conv weight (1024, 16, 2, 2) -> (64, 1024) map over (p, q, c)
    patch vectors (W_rt, oasis_inference.py:1821-1826)."""
    return conv_w.float().permute(0, 2, 3, 1).reshape(D_MODEL, OUT_DIM).T.contiguous()
