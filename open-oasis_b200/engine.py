"""Native frame-generation API over the C ABI.

Functions here take torch tensors only as device-memory handles; all compute is
in liboasis_b200.so, launched on the current torch CUDA stream. `FrameEngine`
preallocates every buffer of one frame (B sessions x T frames) and can capture
the whole frame (4 DDIM steps + bridge + VAE decode) into a CUDA graph, the
B200 equivalent of the reference's trace capture/replay
(oasis_inference.py:2125-2148, 2224).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from . import host as H
from .weights import CondDeviceWeights, DitDeviceWeights, VaeDeviceWeights, VaeEncoderDeviceWeights


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _check_cuda(t: torch.Tensor, name: str, dtype=torch.float32):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def dit_workspace_bytes(batch: int, frames: int) -> int:
    return int(_lib.load().oasis_dit_workspace_size(batch, frames))


def step_workspace_bytes(batch: int, frames: int) -> int:
    return int(_lib.load().oasis_step_workspace_size(batch, frames))


def vae_workspace_bytes(batch: int) -> int:
    return int(_lib.load().oasis_vae_workspace_size(batch))


def dit_forward(dw: DitDeviceWeights, z: torch.Tensor, cond: torch.Tensor, v_out: torch.Tensor,
                ws: torch.Tensor, last_frame_only: bool = True, stream=None) -> torch.Tensor:
    """z [B, T, 144, 1024] fp32 (overwritten), cond [B, T, 1024] -> v_out."""
    _check_cuda(z, "z")
    _check_cuda(cond, "cond")
    _check_cuda(v_out, "v_out")
    B, T = z.shape[0], z.shape[1]
    if tuple(z.shape[2:]) != (H.N_PATCHES, H.D_MODEL) or tuple(cond.shape) != (B, T, H.D_MODEL):
        raise ValueError(f"bad shapes z={tuple(z.shape)} cond={tuple(cond.shape)}")
    want = (B, H.N_PATCHES, H.OUT_DIM) if last_frame_only else (B, T, H.N_PATCHES, H.OUT_DIM)
    if tuple(v_out.shape) != want:
        raise ValueError(f"v_out must be {want}")
    a = _lib.OasisDitArgs(B, T, z.data_ptr(), cond.data_ptr(), v_out.data_ptr(), int(last_frame_only),
                          ws.data_ptr(), ws.numel())
    _lib.call("oasis_dit_forward", dw.ref(), C.byref(a), _stream(stream))
    return v_out


def kv_cache_bytes(batch: int, past_frames: int) -> int:
    return int(_lib.load().oasis_kv_cache_size(batch, past_frames))


def kv_cache(batch: int, past_frames: int, device) -> torch.Tensor:
    """Device buffer for the context frames' cached QKV of every temporal sub-block."""
    return workspace(kv_cache_bytes(batch, past_frames), device)


def dit_precompute_past(dw: DitDeviceWeights, z_past: torch.Tensor, cond_past: torch.Tensor, cache: torch.Tensor,
                        ws: torch.Tensor, stream=None) -> torch.Tensor:
    """Context frames z_past [B, Tp, 144, 1024] fp32 (overwritten), cond_past
    [B, Tp, 1024] -> cache (precompute_past_state, oasis_inference.py:1354)."""
    _check_cuda(z_past, "z_past")
    _check_cuda(cond_past, "cond_past")
    B, Tp = z_past.shape[0], z_past.shape[1]
    if tuple(z_past.shape[2:]) != (H.N_PATCHES, H.D_MODEL) or tuple(cond_past.shape) != (B, Tp, H.D_MODEL):
        raise ValueError(f"bad shapes z_past={tuple(z_past.shape)} cond_past={tuple(cond_past.shape)}")
    a = _lib.OasisDitArgs(B, Tp, z_past.data_ptr(), cond_past.data_ptr(), 0, 0, ws.data_ptr(), ws.numel())
    _lib.call("oasis_dit_precompute_past", dw.ref(), C.byref(a), cache.data_ptr(), cache.numel(), _stream(stream))
    return cache


def dit_forward_current(dw: DitDeviceWeights, z_cur: torch.Tensor, cond_cur: torch.Tensor, cache: torch.Tensor | None,
                        past_frames: int, v_out: torch.Tensor, ws: torch.Tensor, stream=None) -> torch.Tensor:
    """Generated frame z_cur [B, 144, 1024] fp32 (overwritten), cond_cur [B, 1024],
    with `past_frames` cached context frames -> v_out [B, 144, 64]
    (dit_forward_currentonly, oasis_inference.py:1372)."""
    _check_cuda(z_cur, "z_cur")
    _check_cuda(cond_cur, "cond_cur")
    _check_cuda(v_out, "v_out")
    B = z_cur.shape[0]
    if tuple(z_cur.shape) != (B, H.N_PATCHES, H.D_MODEL) or tuple(cond_cur.shape) != (B, H.D_MODEL):
        raise ValueError(f"bad shapes z_cur={tuple(z_cur.shape)} cond_cur={tuple(cond_cur.shape)}")
    if tuple(v_out.shape) != (B, H.N_PATCHES, H.OUT_DIM):
        raise ValueError("v_out must be [B, 144, 64]")
    a = _lib.OasisDitArgs(B, 1, z_cur.data_ptr(), cond_cur.data_ptr(), v_out.data_ptr(), 1, ws.data_ptr(), ws.numel())
    _lib.call("oasis_dit_forward_current", dw.ref(), C.byref(a), 0 if cache is None else cache.data_ptr(),
              0 if cache is None else cache.numel(), past_frames, _stream(stream))
    return v_out


def ddim_update(chunk: torch.Tensor, v: torch.Tensor, step: H.DdimStep, stream=None) -> torch.Tensor:
    _check_cuda(chunk, "chunk")
    _check_cuda(v, "v")
    if chunk.numel() != v.numel():
        raise ValueError("chunk and v differ in size")
    c = _lib.OasisDdimCoeffs(*step.as_tuple())
    _lib.call("oasis_ddim_update", chunk.data_ptr(), v.data_ptr(), C.byref(c), chunk.numel(), _stream(stream))
    return chunk


def ddim_step(dw: DitDeviceWeights, chunk: torch.Tensor, context_z: torch.Tensor | None, cond: torch.Tensor,
              step: H.DdimStep, ws: torch.Tensor, stream=None) -> torch.Tensor:
    """One DDIM step in place on chunk [B, 144, 64] with T-1 context frames."""
    _check_cuda(chunk, "chunk")
    _check_cuda(cond, "cond")
    B, T = cond.shape[0], cond.shape[1]
    if context_z is not None:
        _check_cuda(context_z, "context_z")
        if tuple(context_z.shape) != (B, T - 1, H.N_PATCHES, H.D_MODEL):
            raise ValueError(f"context_z must be {(B, T - 1, H.N_PATCHES, H.D_MODEL)}")
    a = _lib.OasisStepArgs(B, T, chunk.data_ptr(), 0 if context_z is None else context_z.data_ptr(),
                           cond.data_ptr(), _lib.OasisDdimCoeffs(*step.as_tuple()), ws.data_ptr(), ws.numel())
    _lib.call("oasis_ddim_step", dw.ref(), C.byref(a), _stream(stream))
    return chunk


def patch_embed(dw: DitDeviceWeights, patches: torch.Tensor, z: torch.Tensor, out_group: int, out_off: int,
                stream=None) -> torch.Tensor:
    """patches [R, 64] -> rows (r // 144) * out_group + out_off + r % 144 of z."""
    _check_cuda(patches, "patches")
    _check_cuda(z, "z")
    rows = patches.numel() // H.OUT_DIM
    _lib.call("oasis_patch_embed", dw.ref(), patches.data_ptr(), rows, z.data_ptr(), out_group, out_off,
              _stream(stream))
    return z


def bridge_unpatchify(chunk: torch.Tensor, latent: torch.Tensor, stream=None) -> torch.Tensor:
    """chunk [B, 144, 64] -> latent [B, 576, 16] / SCALING_FACTOR."""
    _check_cuda(chunk, "chunk")
    _check_cuda(latent, "latent")
    B = chunk.numel() // (H.N_PATCHES * H.OUT_DIM)
    if latent.numel() != B * H.VAE_TOKENS * H.VAE_LATENT:
        raise ValueError("latent must hold B x 576 x 16 values")
    _lib.call("oasis_bridge_unpatchify", chunk.data_ptr(), latent.data_ptr(), B, _stream(stream))
    return latent


def vae_decode(vw: VaeDeviceWeights, latent: torch.Tensor, image: torch.Tensor, ws: torch.Tensor,
               stream=None) -> torch.Tensor:
    """latent [B, 576, 16] -> image [B, 3, 360, 640] in [-1, 1]."""
    _check_cuda(latent, "latent")
    _check_cuda(image, "image")
    B = latent.shape[0]
    if tuple(image.shape) != (B, 3, H.VAE_H * H.VAE_PATCH, H.VAE_W * H.VAE_PATCH):
        raise ValueError("image must be [B, 3, 360, 640]")
    a = _lib.OasisVaeArgs(B, latent.data_ptr(), image.data_ptr(), ws.data_ptr(), ws.numel())
    _lib.call("oasis_vae_decode", vw.ref(), C.byref(a), _stream(stream))
    return image


def vae_encoder_workspace_bytes(batch: int) -> int:
    return int(_lib.load().oasis_vae_encoder_workspace_size(batch))


def vae_encode(ew: VaeEncoderDeviceWeights, image: torch.Tensor, ws: torch.Tensor, latent: torch.Tensor | None = None,
               chunk: torch.Tensor | None = None, stream=None) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """image [B, 3, 360, 640] in [-1, 1] -> latent [B, 576, 16] (posterior mean x
    scaling factor) and/or chunk [B, 144, 64] (the same latent in the DiT's patch
    layout, ready for patch_embed as a context frame)."""
    _check_cuda(image, "image")
    B = image.shape[0]
    if tuple(image.shape) != (B, 3, H.VAE_H * H.VAE_PATCH, H.VAE_W * H.VAE_PATCH):
        raise ValueError("image must be [B, 3, 360, 640]")
    if latent is None and chunk is None:
        raise ValueError("vae_encode needs a latent or a chunk output")
    if latent is not None:
        _check_cuda(latent, "latent")
        if tuple(latent.shape) != (B, H.VAE_TOKENS, H.VAE_LATENT):
            raise ValueError("latent must be [B, 576, 16]")
    if chunk is not None:
        _check_cuda(chunk, "chunk")
        if tuple(chunk.shape) != (B, H.N_PATCHES, H.OUT_DIM):
            raise ValueError("chunk must be [B, 144, 64]")
    a = _lib.OasisVaeEncodeArgs(B, image.data_ptr(), _lib.ptr(latent), _lib.ptr(chunk), ws.data_ptr(), ws.numel())
    _lib.call("oasis_vae_encode", ew.ref(), C.byref(a), _stream(stream))
    return latent, chunk


def frame_workspace_bytes(batch: int, frames: int, steps: int) -> int:
    return int(_lib.load().oasis_frame_workspace_size(batch, frames, steps))


def frame_kv_workspace_bytes(batch: int, frames: int, steps: int) -> int:
    return int(_lib.load().oasis_frame_kv_workspace_size(batch, frames, steps))


def cond_workspace_bytes(rows: int) -> int:
    return int(_lib.load().oasis_cond_workspace_size(rows))


def compute_cond(dw: DitDeviceWeights | CondDeviceWeights, levels: torch.Tensor, cond: torch.Tensor, ws: torch.Tensor,
                 actions: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Frame conditioning on the GPU (compute_cond_for_frame, oasis_inference.py:1406-1427):
    cond[r] = t_mlp(timestep_embedding(levels[r])) + external_cond(actions[r % A]).
    levels: fp32 [n] (any shape, flattened); cond: fp32 [n, 1024] (any shape with
    n * 1024 elements); actions: fp32 [..., 25] with A rows, or None (no action term)."""
    _check_cuda(levels, "levels")
    _check_cuda(cond, "cond")
    n = levels.numel()
    if cond.numel() != n * H.D_MODEL:
        raise ValueError(f"cond must hold {n} x {H.D_MODEL} values")
    a_rows = 0
    if actions is not None:
        _check_cuda(actions, "actions")
        if actions.shape[-1] != H.EXT_COND_DIM:
            raise ValueError(f"actions must end in {H.EXT_COND_DIM}")
        a_rows = actions.numel() // H.EXT_COND_DIM
    cw = dw.cond if isinstance(dw, DitDeviceWeights) else dw
    _lib.call("oasis_compute_cond", cw.ref(), levels.data_ptr(), n, _lib.ptr(actions), a_rows,
              cond.data_ptr(), ws.data_ptr(), ws.numel(), _stream(stream))
    return cond


def generate_frame(dw: DitDeviceWeights, vw: VaeDeviceWeights | None, chunk: torch.Tensor,
                   context_z: torch.Tensor | None, cond: torch.Tensor, steps: list[H.DdimStep],
                   image: torch.Tensor | None, ws: torch.Tensor, skip_decode: bool = False, stream=None,
                   kv: bool = False):
    """One frame for B sessions: len(steps) DDIM steps (chunk updated in place),
    then bridge + VAE decode into image [B, 3, 360, 640] unless skip_decode.
    kv=True runs the context frames once and only the generated frame per step
    (oasis_generate_frame_kv; workspace from frame_kv_workspace_bytes)."""
    _check_cuda(chunk, "chunk")
    _check_cuda(cond, "cond")
    S, B, T = cond.shape[0], cond.shape[1], cond.shape[2]
    if S != len(steps) or tuple(chunk.shape) != (B, H.N_PATCHES, H.OUT_DIM):
        raise ValueError("cond must be [steps, B, T, 1024] and chunk [B, 144, 64]")
    if context_z is not None:
        _check_cuda(context_z, "context_z")
        if tuple(context_z.shape) != (B, T - 1, H.N_PATCHES, H.D_MODEL):
            raise ValueError(f"context_z must be {(B, T - 1, H.N_PATCHES, H.D_MODEL)}")
    if not skip_decode:
        _check_cuda(image, "image")
    coeffs = (_lib.OasisDdimCoeffs * S)(*[_lib.OasisDdimCoeffs(*st.as_tuple()) for st in steps])
    a = _lib.OasisFrameArgs(B, T, S, chunk.data_ptr(), 0 if context_z is None else context_z.data_ptr(),
                            cond.data_ptr(), coeffs, 0 if image is None else image.data_ptr(), int(skip_decode),
                            ws.data_ptr(), ws.numel())
    _lib.call("oasis_generate_frame_kv" if kv else "oasis_generate_frame", dw.ref(), None if vw is None else vw.ref(), C.byref(a), _stream(stream))
    return chunk


class FrameEngine:
    """All device buffers of one generated frame for B sessions with T-frame
    context windows (kv=True: context rows run once per frame). `run()` issues the whole frame through oasis_generate_frame
    (4 DDIM steps with all adaLN tables from one GEMM, bridge, VAE decode);
    `capture()` records it (and, for timing breakdowns, the steps alone and the
    decode alone) as CUDA graphs.

    device_cond=True computes `cond` inside the frame (and its graph) from the
    per-frame action window `actions` [B, T, 25]: context frames at the
    stabilisation level, the generated frame at each step's noise level
    (oasis_compute_cond); otherwise the caller fills `cond`."""

    def __init__(self, dw: DitDeviceWeights, vw: VaeDeviceWeights, batch: int, frames: int,
                 steps: list[H.DdimStep] | None = None, kv: bool = False, device_cond: bool = False):
        self.dw, self.vw, self.kv = dw, vw, kv
        self.B, self.T = batch, frames
        self.steps = steps if steps is not None else H.ddim_schedule()
        dev = dw.device
        B, T = batch, frames
        self.chunk = torch.zeros(B, H.N_PATCHES, H.OUT_DIM, device=dev)
        self.context_z = torch.zeros(B, max(T - 1, 1), H.N_PATCHES, H.D_MODEL, device=dev)
        self.cond = torch.zeros(len(self.steps), B, T, H.D_MODEL, device=dev)
        self.latent = torch.zeros(B, H.VAE_TOKENS, H.VAE_LATENT, device=dev)
        self.image = torch.zeros(B, 3, H.VAE_H * H.VAE_PATCH, H.VAE_W * H.VAE_PATCH, device=dev)
        nbytes = (frame_kv_workspace_bytes if kv else frame_workspace_bytes)(B, T, len(self.steps))
        self.frame_ws = workspace(nbytes, dev)
        self.device_cond = device_cond
        if device_cond:
            S = len(self.steps)
            lv = torch.full((S, B, T), float(H.STABILIZATION_LEVEL - 1))
            for i, st in enumerate(self.steps):
                lv[i, :, T - 1] = float(st.noise_level)
            self.levels = lv.to(dev)
            self.actions = torch.zeros(B, T, H.EXT_COND_DIM, device=dev)
            self.cond_ws = workspace(cond_workspace_bytes(S * B * T), dev)
        self.step_ws = None
        self.vae_ws = None
        self.graph = None

    def _ctx(self):
        return self.context_z if self.T > 1 else None

    def run_cond(self, stream=None):
        if self.device_cond:
            compute_cond(self.dw, self.levels, self.cond, self.cond_ws, self.actions, stream)

    def run(self, stream=None):
        self.run_cond(stream)
        generate_frame(self.dw, self.vw, self.chunk, self._ctx(), self.cond, self.steps, self.image, self.frame_ws,
                       stream=stream, kv=self.kv)

    def run_steps(self, stream=None):
        self.run_cond(stream)
        generate_frame(self.dw, None, self.chunk, self._ctx(), self.cond, self.steps, None, self.frame_ws,
                       skip_decode=True, stream=stream, kv=self.kv)

    def run_decode(self, stream=None):
        if self.vae_ws is None:
            self.vae_ws = workspace(vae_workspace_bytes(self.B), self.dw.device)
        bridge_unpatchify(self.chunk, self.latent, stream)
        vae_decode(self.vw, self.latent, self.image, self.vae_ws, stream)

    def run_steps_separately(self, stream=None):
        """The same steps through oasis_ddim_step (adaLN per step)."""
        if self.step_ws is None:
            self.step_ws = workspace(step_workspace_bytes(self.B, self.T), self.dw.device)
        self.run_cond(stream)
        for i, st in enumerate(self.steps):
            ddim_step(self.dw, self.chunk, self._ctx(), self.cond[i], st, self.step_ws, stream)

    def capture(self, breakdown: bool = False):
        """Captures the frame as a CUDA graph (launch sequence and pointers fixed);
        with breakdown=True also the steps alone and the decode alone. Runs the
        frame eagerly once first, which modifies `chunk`."""
        self.run()
        if breakdown:
            self.run_decode()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.run()
        if breakdown:
            self.graph_steps = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph_steps):
                self.run_steps()
            self.graph_decode = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph_decode):
                self.run_decode()
        return self.graph

    def replay(self):
        if self.graph is None:
            raise RuntimeError("capture() first")
        self.graph.replay()


class VideoEngine:
    """The autoregressive video loop on the GPU (oasis_inference.py:2262-2310).

    Each `step()` generates one frame for B sessions (S DDIM steps + bridge + VAE
    through a FrameEngine, full-T or context-cached) and then rolls the context
    window on the device: the generated latent patches are patch-embedded straight
    into the newest context slot and the conditioning window rolls with them, so
    no frame data goes back to the host between frames (the reference reads the
    chunk back, unpatchifies and patch-embeds it on the host, :2296-2306).

    Per-frame inputs: the noise chunk [B, 144, 64], the generated frame's
    conditioning per step [S, B, 1024] and its context conditioning [B, 1024]
    (stabilisation level, same action) for when it joins the window."""

    def __init__(self, dw: DitDeviceWeights, vw: VaeDeviceWeights, batch: int, frames: int,
                 steps: list[H.DdimStep] | None = None, kv: bool = False, device_cond: bool = False):
        if frames < 2:
            raise ValueError("the video loop needs a context window (frames >= 2)")
        self.fe = FrameEngine(dw, vw, batch, frames, steps, kv=kv, device_cond=device_cond)
        self.dw, self.B, self.T = dw, batch, frames
        self.device_cond = device_cond
        dev = dw.device
        S = len(self.fe.steps)
        self.ctx_cond = torch.zeros(batch, frames - 1, H.D_MODEL, device=dev)
        self.gen_cond = torch.zeros(S, batch, H.D_MODEL, device=dev)      # staging, per frame
        self.new_ctx_cond = torch.zeros(batch, H.D_MODEL, device=dev)    # staging, per frame
        self.new_action = torch.zeros(batch, H.EXT_COND_DIM, device=dev)  # staging, per frame (device_cond)
        self._tmp_z = torch.empty(batch, max(frames - 2, 1), H.N_PATCHES, H.D_MODEL, device=dev)
        self._tmp_c = torch.empty(batch, max(frames - 2, 1), H.D_MODEL, device=dev)
        self._tmp_a = torch.empty(batch, max(frames - 2, 1), H.EXT_COND_DIM, device=dev)
        self.graph = None

    @property
    def context_z(self) -> torch.Tensor:
        return self.fe.context_z

    @property
    def image(self) -> torch.Tensor:
        return self.fe.image

    @property
    def ctx_actions(self) -> torch.Tensor:
        """device_cond: the context frames' actions [B, T-1, 25] (a view)."""
        return self.fe.actions[:, :self.T - 1]

    def set_context(self, context_z: torch.Tensor, ctx_cond: torch.Tensor):
        """context_z [B, T-1, 144, 1024]; ctx_cond: the context conditioning
        [B, T-1, 1024], or with device_cond the context frames' actions [B, T-1, 25]."""
        self.fe.context_z.copy_(context_z)
        if self.device_cond:
            self.ctx_actions.copy_(ctx_cond)
        else:
            self.ctx_cond.copy_(ctx_cond)

    def set_prompt(self, ew: VaeEncoderDeviceWeights, image: torch.Tensor, prompt_cond: torch.Tensor,
                   ws: torch.Tensor | None = None):
        """Starts the loop from B prompt images [B, 3, 360, 640] in [-1, 1] (the
        reference encodes the prompt on the CPU and fills every context slot with
        its patch embedding, oasis_inference.py:1744-1754, 1806-1813, 2248-2252):
        the VAE encoder writes the latent in the DiT's patch layout, which is
        patch-embedded into each of the T - 1 context slots; the conditioning
        window is filled with `prompt_cond` [B, 1024] (the context conditioning,
        stabilisation level and no action)."""
        B, T, dev = self.B, self.T, self.dw.device
        if tuple(prompt_cond.shape) != (B, H.D_MODEL):
            raise ValueError(f"prompt_cond must be [{B}, {H.D_MODEL}]")
        chunk = torch.empty(B, H.N_PATCHES, H.OUT_DIM, device=dev)
        if ws is None:
            ws = workspace(vae_encoder_workspace_bytes(B), dev)
        vae_encode(ew, image, ws, chunk=chunk)
        for slot in range(T - 1):
            patch_embed(self.dw, chunk.view(-1, H.OUT_DIM), self.fe.context_z, (T - 1) * H.N_PATCHES,
                        slot * H.N_PATCHES)
        if self.device_cond:
            self.ctx_actions.zero_()  # the prompt frames carry no action (oasis_inference.py:1801)
        else:
            self.ctx_cond.copy_(prompt_cond.to(dev).unsqueeze(1).expand(-1, T - 1, -1))
        return chunk

    def _frame_and_roll(self, stream=None):
        if self.device_cond:
            return self._frame_and_roll_device_cond(stream)
        fe, T = self.fe, self.T
        fe.cond[:, :, :T - 1].copy_(self.ctx_cond.unsqueeze(0).expand(fe.cond.shape[0], -1, -1, -1))
        fe.cond[:, :, T - 1].copy_(self.gen_cond)
        fe.run(stream)
        if T > 2:  # drop the oldest context frame (through a scratch copy: the ranges overlap)
            self._tmp_z.copy_(fe.context_z[:, 1:])
            fe.context_z[:, :-1].copy_(self._tmp_z)
            self._tmp_c.copy_(self.ctx_cond[:, 1:])
            self.ctx_cond[:, :-1].copy_(self._tmp_c)
        # the generated latent patches -> newest context slot (rows (T-2) 144 .. of each session)
        patch_embed(self.dw, fe.chunk.view(-1, H.OUT_DIM), fe.context_z, (T - 1) * H.N_PATCHES,
                    (T - 2) * H.N_PATCHES, stream)
        self.ctx_cond[:, -1].copy_(self.new_ctx_cond)

    def _frame_and_roll_device_cond(self, stream=None):
        """The frame with its conditioning computed on the GPU from the action
        window: context frames at the stabilisation level with their own actions,
        the generated frame at each step's noise level with the new action; the
        new action then joins the window with the frame."""
        fe, T = self.fe, self.T
        fe.actions[:, T - 1].copy_(self.new_action)
        fe.run(stream)
        if T > 2:
            self._tmp_z.copy_(fe.context_z[:, 1:])
            fe.context_z[:, :-1].copy_(self._tmp_z)
            self._tmp_a.copy_(fe.actions[:, 1:T - 1])
            fe.actions[:, :T - 2].copy_(self._tmp_a)
        patch_embed(self.dw, fe.chunk.view(-1, H.OUT_DIM), fe.context_z, (T - 1) * H.N_PATCHES,
                    (T - 2) * H.N_PATCHES, stream)
        fe.actions[:, T - 2].copy_(self.new_action)

    def step_actions(self, noise: torch.Tensor, action: torch.Tensor) -> torch.Tensor:
        """device_cond: one frame from its noise chunk [B, 144, 64] and action
        [B, 25] (host or device tensors); returns the decoded image buffer
        [B, 3, 360, 640] (overwritten by the next step)."""
        if not self.device_cond:
            raise RuntimeError("step_actions needs VideoEngine(..., device_cond=True)")
        self.fe.chunk.copy_(noise, non_blocking=True)
        self.new_action.copy_(action, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._frame_and_roll()
        return self.fe.image

    def step(self, noise: torch.Tensor, gen_cond: torch.Tensor, new_ctx_cond: torch.Tensor) -> torch.Tensor:
        """One frame; returns the decoded image buffer [B, 3, 360, 640] (overwritten
        by the next step)."""
        if self.device_cond:
            raise RuntimeError("this engine computes the conditioning on the GPU: use step_actions")
        self.fe.chunk.copy_(noise, non_blocking=True)
        self.gen_cond.copy_(gen_cond, non_blocking=True)
        self.new_ctx_cond.copy_(new_ctx_cond, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._frame_and_roll()
        return self.fe.image

    def capture(self):
        """Records frame + context roll as one CUDA graph (its inputs are the
        staging buffers `step()` fills). Runs one eager frame first: call it
        before `set_context`, or set the context again afterwards."""
        self._frame_and_roll()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._frame_and_roll()
        self.graph = g
        return g
