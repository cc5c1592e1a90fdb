"""Drop-in replacements for the device-side functions of zoecarver/open-oasis
`oasis_inference.py`, with the same names and argument order, backed by the
sm_100a kernels (no ttnn, no CPU fallback).

Mapping (reference file:line -> here):
  preload_dit_weights      :505   -> preload_dit_weights(state_dict, device, n_frames)
  prealloc_scratch         :790   -> prealloc_scratch(device, n_frames, batch=1)
  dit_forward_device       :1438  -> dit_forward_device(z_cur, cond_list, dev, scr, ...)
  precompute_past_state    :1354  -> precompute_past_state(past_z, past_cond, dev, scr, ...)
  dit_forward_currentonly  :1372  -> dit_forward_currentonly(curr_z, curr_cond, dev, scr, ...)
  ddim_step_fn (closure)   :1909  -> make_ddim_step_fn(dev, scr, context_z)(chunk, step_coeffs, cond_list)
  compute_cond_for_frame   :1406  -> compute_cond_for_frame(t_scalar, action_vec, dev, scr, tt_device)
  preload_vae_decoder_weights :679 -> preload_vae_decoder_weights(vae_state_dict, device)
  prealloc_vae_scratch     :763   -> prealloc_vae_scratch(device, batch=1)
  vae_decode_forward       :1546  -> vae_decode_forward(vae_dev, vae_scr, ...)
  bridge_unpatchify        :1697  -> bridge_unpatchify(dit_output, bridge, bridge_tmp, vae_input)
  vae.encode(x).mean * SCALING_FACTOR  :1748-1751
                                  -> vae_encode(enc_dev, x) with enc_dev = preload_vae_encoder_weights(...)

Differences a caller sees (all deliberate, B200-first):
  * token rows are exactly 144 per frame (the reference pads to 160); SEQ = 144 T;
  * vae_input is (576, 16) fp32 (no padding to 32 columns);
  * vae_decode_forward fuses vae_unpatchify and the clamp into the predictor GEMM:
    vae_scr["pred_out"] is the (1, 3, 360, 640) frame in [-1, 1], not (576, 1216) patches;
  * precompute_past_state / dit_forward_currentonly take the conditioning before
    SiLU (the SiLU runs in the library) and any number n_frames - 1 of context
    frames (the reference caches exactly one);
  * tt_device / scaler / mean_scale arguments are accepted and ignored;
  * errors raise OasisError (the C status and message) instead of ttnn exceptions.
"""
from __future__ import annotations

import torch

from . import checkpoint as CK
from . import engine as E
from . import host as H
from .host import sigmoid_beta_schedule, timestep_embedding  # noqa: F401  (reference names)
from .weights import DitDeviceWeights, VaeDeviceWeights, VaeEncoderDeviceWeights

TILE = 32
D_MODEL = H.D_MODEL
N_PATCHES = H.N_PATCHES
OUT_DIM = H.OUT_DIM


def preload_dit_weights(state_dict, device="cuda", n_frames: int = 2) -> DitDeviceWeights:
    """Packs a reference-keyed DiT state dict (or the path of the released
    safetensors file) onto the GPU (bf16 GEMM weights)."""
    if isinstance(state_dict, str):
        state_dict = CK.load_dit_checkpoint(state_dict)
    return DitDeviceWeights(state_dict, device)


def prealloc_scratch(device="cuda", n_frames: int = 2, batch: int = 1) -> dict:
    """Scratch of one DiT forward / DDIM step, sized for `batch` sessions of n_frames."""
    dev = torch.device(device)
    return {
        "n_frames": n_frames,
        "batch": batch,
        "dit_ws": E.workspace(E.dit_workspace_bytes(batch, n_frames), dev),
        "step_ws": E.workspace(E.step_workspace_bytes(batch, n_frames), dev),
        "z_cur": torch.zeros(batch, n_frames, N_PATCHES, D_MODEL, device=dev),
        "final_out_f32": torch.zeros(batch, n_frames, N_PATCHES, OUT_DIM, device=dev),
        "cond": torch.zeros(batch, n_frames, D_MODEL, device=dev),
        # context caching (precompute_past_state / dit_forward_currentonly)
        "kv_cache": E.kv_cache(batch, n_frames - 1, dev) if n_frames > 1 else None,
        "kv_ws": E.workspace(E.dit_workspace_bytes(batch, max(n_frames - 1, 1)), dev),
        "z_past": torch.zeros(batch, max(n_frames - 1, 1), N_PATCHES, D_MODEL, device=dev),
        "cond_past": torch.zeros(batch, max(n_frames - 1, 1), D_MODEL, device=dev),
        "z_curr": torch.zeros(batch, N_PATCHES, D_MODEL, device=dev),
        "cond_curr": torch.zeros(batch, D_MODEL, device=dev),
        "t1_final_out_f32": torch.zeros(batch, N_PATCHES, OUT_DIM, device=dev),
    }


def _cond_rows(cond_list) -> torch.Tensor:
    rows = [c.reshape(-1, D_MODEL)[0] for c in cond_list]  # reference conds are (TILE, D) row-broadcast
    return torch.stack(rows, 0)


def dit_forward_device(z_cur, cond_list, dev: DitDeviceWeights, scr: dict, tt_device=None, scaler=None,
                       mean_scale=None, profile_step=False) -> torch.Tensor:
    """z_cur (144 T, 1024) fp32, cond_list: T conditioning vectors (pre-SiLU).
    Returns final_out (144 T, 64) fp32 v-prediction for every frame."""
    T = len(cond_list)
    if T != scr["n_frames"] or scr["batch"] != 1:
        raise ValueError(f"scratch was allocated for batch={scr['batch']} n_frames={scr['n_frames']}")
    z = scr["z_cur"]
    z.view(-1, D_MODEL).copy_(z_cur.reshape(-1, D_MODEL))
    scr["cond"][0].copy_(_cond_rows(cond_list))
    out = scr["final_out_f32"]
    E.dit_forward(dev, z, scr["cond"], out, scr["dit_ws"], last_frame_only=False)
    return out.view(T * N_PATCHES, OUT_DIM)


def precompute_past_state(past_z, past_cond, dev: DitDeviceWeights, scr: dict, tt_device=None, scaler=None,
                          mean_scale=None) -> None:
    """Runs the n_frames - 1 context frames once and fills scr["kv_cache"] with
    their RoPE'd QKV at every temporal sub-block.
    past_z: ((n_frames - 1) 144, 1024) fp32 embedded context frames;
    past_cond: one (1024,) pre-SiLU conditioning vector (shared by the context
    frames, as in the reference) or a list of n_frames - 1 of them."""
    Tp = scr["n_frames"] - 1
    if Tp < 1 or scr["batch"] != 1:
        raise ValueError("precompute_past_state needs a batch=1 scratch with n_frames >= 2")
    conds = past_cond if isinstance(past_cond, (list, tuple)) else [past_cond] * Tp
    scr["z_past"].view(-1, D_MODEL).copy_(past_z.reshape(-1, D_MODEL))
    scr["cond_past"][0].copy_(_cond_rows(conds))
    E.dit_precompute_past(dev, scr["z_past"], scr["cond_past"], scr["kv_cache"], scr["kv_ws"])


def dit_forward_currentonly(curr_z, curr_cond, dev: DitDeviceWeights, scr: dict, tt_device=None, scaler=None,
                            mean_scale=None) -> torch.Tensor:
    """The generated frame alone (at temporal position n_frames - 1) against the
    cache from precompute_past_state. curr_z (144, 1024) fp32; curr_cond (1024,)
    pre-SiLU. Returns the (144, 64) v-prediction."""
    if scr["batch"] != 1:
        raise ValueError("dit_forward_currentonly needs a batch=1 scratch")
    Tp = scr["n_frames"] - 1
    scr["z_curr"].view(-1, D_MODEL).copy_(curr_z.reshape(-1, D_MODEL))
    scr["cond_curr"].copy_(_cond_rows([curr_cond]))
    out = scr["t1_final_out_f32"]
    E.dit_forward_current(dev, scr["z_curr"], scr["cond_curr"], scr["kv_cache"], Tp, out, scr["kv_ws"])
    return out.view(N_PATCHES, OUT_DIM)


def make_ddim_step_fn(dev: DitDeviceWeights, scr: dict, context_z: torch.Tensor | None):
    """Builds the reference's `ddim_step_fn(chunk, step_coeffs, cond_list)` closure.

    context_z: ((T-1) 144, 1024) fp32 embedded context frames (None when T == 1).
    step_coeffs: dict with the reference keys at_sqrt, 1mat_sqrt, inv_at_sqrt,
    inv_sigma, an_sqrt, 1man_sqrt (scalars or constant tensors).
    """
    T = scr["n_frames"]
    ctx = None if context_z is None else context_z.reshape(1, T - 1, N_PATCHES, D_MODEL).contiguous()

    def _s(x):
        return float(x.reshape(-1)[0]) if torch.is_tensor(x) else float(x)

    def ddim_step_fn(chunk, step_coeffs, cond_list, profile=False):
        step = H.DdimStep(-1, _s(step_coeffs["at_sqrt"]), _s(step_coeffs["1mat_sqrt"]),
                          _s(step_coeffs["inv_at_sqrt"]), _s(step_coeffs["inv_sigma"]),
                          _s(step_coeffs["an_sqrt"]), _s(step_coeffs["1man_sqrt"]))
        scr["cond"][0].copy_(_cond_rows(cond_list))
        c = chunk.view(1, N_PATCHES, OUT_DIM)
        E.ddim_step(dev, c, ctx, scr["cond"], step, scr["step_ws"])
        return chunk

    return ddim_step_fn


def compute_cond_for_frame(t_scalar, action_vec, dev: DitDeviceWeights, scr=None, tt_device=None) -> torch.Tensor:
    """Host fp32 conditioning (t-MLP + action linear), returned as a (1024,) device tensor."""
    act = None if action_vec is None else action_vec.reshape(1, -1)
    c = H.compute_cond(torch.tensor([int(t_scalar)]), act, dev.host)[0]
    return c.to(dev.device)


def preload_vae_decoder_weights(vae_state_dict, device="cuda", rotary_table=None) -> VaeDeviceWeights:
    """Packs the VAE decoder (state dict, or the path of the released safetensors
    file plus optionally the (18, 32, 32) pixel RoPE table of the VAE module)."""
    if isinstance(vae_state_dict, str):
        vae_state_dict = CK.load_vae_checkpoint(vae_state_dict, rotary_table)
    return VaeDeviceWeights(vae_state_dict, device)


def prealloc_vae_scratch(device="cuda", batch: int = 1) -> dict:
    dev = torch.device(device)
    return {
        "batch": batch,
        "vae_input": torch.zeros(batch, H.VAE_TOKENS, H.VAE_LATENT, device=dev),
        "pred_out": torch.zeros(batch, 3, H.VAE_H * H.VAE_PATCH, H.VAE_W * H.VAE_PATCH, device=dev),
        "ws": E.workspace(E.vae_workspace_bytes(batch), dev),
    }


def vae_decode_forward(vae_dev: VaeDeviceWeights, vae_scr: dict, scaler=None, mean_scale=None) -> torch.Tensor:
    """Decodes vae_scr["vae_input"] into vae_scr["pred_out"] (frames in [-1, 1])."""
    return E.vae_decode(vae_dev, vae_scr["vae_input"], vae_scr["pred_out"], vae_scr["ws"])


def bridge_unpatchify(dit_output, bridge=None, bridge_tmp=None, vae_input=None) -> torch.Tensor:
    """DiT chunk (144 B, 64) -> VAE latent tokens (B, 576, 16) / SCALING_FACTOR."""
    B = dit_output.numel() // (N_PATCHES * OUT_DIM)
    if vae_input is None:
        vae_input = torch.empty(B, H.VAE_TOKENS, H.VAE_LATENT, device=dit_output.device)
    return E.bridge_unpatchify(dit_output.contiguous(), vae_input)


def preload_vae_encoder_weights(vae_state_dict, device="cuda", rotary_table=None) -> VaeEncoderDeviceWeights:
    """Packs the VAE encoder (state dict, or the path of the VAE safetensors file).
    The reference runs the encoder on the CPU (load_vae_cpu, oasis_inference.py:1738)."""
    if isinstance(vae_state_dict, str):
        vae_state_dict = CK.load_vae_encoder_checkpoint(vae_state_dict, rotary_table)
    return VaeEncoderDeviceWeights(vae_state_dict, device)


def vae_encode(enc_dev: VaeEncoderDeviceWeights, x: torch.Tensor, ws: torch.Tensor | None = None,
               chunk: torch.Tensor | None = None) -> torch.Tensor:
    """`vae.encode(x).mean * SCALING_FACTOR` (oasis_inference.py:1748-1751):
    x (B, 3, 360, 640) in [-1, 1] -> prompt latent (B, 576, 16). If `chunk`
    (B, 144, 64) is given, the same latent is also written there in the DiT's
    patch layout (the reference's rearrange + patchify before the context
    patch embed, :1752-1754, 1806-1809)."""
    x = x.to(enc_dev.device, torch.float32).contiguous()
    B = x.shape[0]
    if ws is None:
        ws = E.workspace(E.vae_encoder_workspace_bytes(B), enc_dev.device)
    latent = torch.empty(B, H.VAE_TOKENS, H.VAE_LATENT, device=enc_dev.device)
    E.vae_encode(enc_dev, x, ws, latent=latent, chunk=chunk)
    return latent
