"""Seeded random-init weights in the reference checkpoint layout, and their
packing into the device layout the kernels read (bf16 GEMM operands, fp32
biases/norms/tables).

Checkpoint keys follow Etched/oasis-500m as read by preload_dit_weights /
preload_vae_decoder_weights (zoecarver/open-oasis oasis_inference.py:505-761).
No checkpoint ships here, so every weight is N(0, std) from a seeded generator
(std 0.02 per the benchmark configs; biases 0 unless bias_std is given).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from . import host as H


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def init_dit_weights(seed: int = 1, n_blocks: int = H.N_BLOCKS, std: float = 0.02,
                     bias_std: float = 0.0) -> dict[str, torch.Tensor]:
    """Reference-keyed fp32 CPU state dict of the DiT (n_blocks spatial+temporal pairs)."""
    g = _gen(seed)

    def w(*shape):
        return torch.randn(*shape, generator=g) * std

    def b(n):
        return torch.randn(n, generator=g) * bias_std if bias_std > 0 else torch.zeros(n)

    D = H.D_MODEL
    sd = {
        "t_embedder.mlp.0.weight": w(D, H.FREQ_DIM), "t_embedder.mlp.0.bias": b(D),
        "t_embedder.mlp.2.weight": w(D, D), "t_embedder.mlp.2.bias": b(D),
        "external_cond.weight": w(D, H.EXT_COND_DIM), "external_cond.bias": b(D),
        "x_embedder.proj.weight": w(D, H.IN_CHANNELS, H.PATCH_SIZE, H.PATCH_SIZE),
        "x_embedder.proj.bias": b(D),
    }
    for i in range(n_blocks):
        for s in ("s", "t"):
            p = f"blocks.{i}.{s}"
            sd[f"{p}_adaLN_modulation.1.weight"] = w(6 * D, D)
            sd[f"{p}_adaLN_modulation.1.bias"] = b(6 * D)
            sd[f"{p}_attn.to_qkv.weight"] = w(3 * D, D)
            sd[f"{p}_attn.to_out.weight"] = w(D, D)
            sd[f"{p}_attn.to_out.bias"] = b(D)
            sd[f"{p}_mlp.fc1.weight"] = w(H.D_MLP, D)
            sd[f"{p}_mlp.fc1.bias"] = b(H.D_MLP)
            sd[f"{p}_mlp.fc2.weight"] = w(D, H.D_MLP)
            sd[f"{p}_mlp.fc2.bias"] = b(D)
    sd["final_layer.adaLN_modulation.1.weight"] = w(2 * D, D)
    sd["final_layer.adaLN_modulation.1.bias"] = b(2 * D)
    sd["final_layer.linear.weight"] = w(H.OUT_DIM, D)
    sd["final_layer.linear.bias"] = b(H.OUT_DIM)
    sd["blocks.0.s_attn.rotary_emb.freqs"] = H.default_spatial_freqs()
    sd["blocks.0.t_attn.rotary_emb.freqs"] = H.default_temporal_freqs()
    return sd


def init_vae_weights(seed: int = 2, n_blocks: int = H.VAE_DEPTH, std: float = 0.02,
                     bias_std: float = 0.0, norm_std: float = 0.0) -> dict[str, torch.Tensor]:
    """Reference-keyed fp32 CPU state dict of the VAE decoder path."""
    g = _gen(seed)

    def w(*shape):
        return torch.randn(*shape, generator=g) * std

    def b(n):
        return torch.randn(n, generator=g) * bias_std if bias_std > 0 else torch.zeros(n)

    def nw(n):
        return 1.0 + (torch.randn(n, generator=g) * norm_std if norm_std > 0 else torch.zeros(n))

    D = H.VAE_DIM
    sd = {"post_quant_conv.weight": w(D, H.VAE_LATENT), "post_quant_conv.bias": b(D)}
    for i in range(n_blocks):
        p = f"decoder.{i}"
        sd[f"{p}.norm1.weight"] = nw(D)
        sd[f"{p}.norm1.bias"] = b(D)
        sd[f"{p}.attn.qkv.weight"] = w(3 * D, D)
        sd[f"{p}.attn.qkv.bias"] = b(3 * D)
        sd[f"{p}.attn.proj.weight"] = w(D, D)
        sd[f"{p}.attn.proj.bias"] = b(D)
        sd[f"{p}.norm2.weight"] = nw(D)
        sd[f"{p}.norm2.bias"] = b(D)
        sd[f"{p}.mlp.fc1.weight"] = w(4 * D, D)
        sd[f"{p}.mlp.fc1.bias"] = b(4 * D)
        sd[f"{p}.mlp.fc2.weight"] = w(D, 4 * D)
        sd[f"{p}.mlp.fc2.bias"] = b(D)
    sd["dec_norm.weight"] = nw(D)
    sd["dec_norm.bias"] = b(D)
    sd["predictor.weight"] = w(H.VAE_PATCH_DIM, D)
    sd["predictor.bias"] = b(H.VAE_PATCH_DIM)
    sd["rotary_freqs"] = H.default_vae_freqs()
    return sd


def init_vae_encoder_weights(seed: int = 4, n_blocks: int = H.VAE_ENC_DEPTH, std: float = 0.02,
                             bias_std: float = 0.0, norm_std: float = 0.0) -> dict[str, torch.Tensor]:
    """Reference-keyed fp32 CPU state dict of the VAE encoder (the `encoder.*`,
    `patch_embed.*`, `enc_norm.*` and `quant_conv.*` keys of the VAE checkpoint)."""
    g = _gen(seed)

    def w(*shape):
        return torch.randn(*shape, generator=g) * std

    def b(n):
        return torch.randn(n, generator=g) * bias_std if bias_std > 0 else torch.zeros(n)

    def nw(n):
        return 1.0 + (torch.randn(n, generator=g) * norm_std if norm_std > 0 else torch.zeros(n))

    D = H.VAE_DIM
    sd = {"patch_embed.proj.weight": w(D, 3, H.VAE_PATCH, H.VAE_PATCH), "patch_embed.proj.bias": b(D)}
    for i in range(n_blocks):
        p = f"encoder.{i}"
        sd[f"{p}.norm1.weight"] = nw(D)
        sd[f"{p}.norm1.bias"] = b(D)
        sd[f"{p}.attn.qkv.weight"] = w(3 * D, D)
        sd[f"{p}.attn.qkv.bias"] = b(3 * D)
        sd[f"{p}.attn.proj.weight"] = w(D, D)
        sd[f"{p}.attn.proj.bias"] = b(D)
        sd[f"{p}.norm2.weight"] = nw(D)
        sd[f"{p}.norm2.bias"] = b(D)
        sd[f"{p}.mlp.fc1.weight"] = w(4 * D, D)
        sd[f"{p}.mlp.fc1.bias"] = b(4 * D)
        sd[f"{p}.mlp.fc2.weight"] = w(D, 4 * D)
        sd[f"{p}.mlp.fc2.bias"] = b(D)
    sd["enc_norm.weight"] = nw(D)
    sd["enc_norm.bias"] = b(D)
    sd["quant_conv.weight"] = w(2 * H.VAE_LATENT, D)
    sd["quant_conv.bias"] = b(2 * H.VAE_LATENT)
    sd["rotary_freqs"] = H.default_vae_freqs()
    return sd


def count_blocks(sd: dict, prefix: str = "blocks.") -> int:
    ids = {int(k.split(".")[1]) for k in sd if k.startswith(prefix)}
    return max(ids) + 1 if ids else 0


class CondDeviceWeights:
    """The conditioning weights (t_embedder MLP, external_cond) on one GPU in fp32,
    plus the ctypes OasisCondWeights struct (the device copies of the host
    tensors compute_cond_for_frame reads, oasis_inference.py:1406-1427)."""

    def __init__(self, sd: dict, device: torch.device | str = "cuda"):
        dev = torch.device(device)
        self.device = dev

        def f32(t):
            return t.to(dev, torch.float32).contiguous()

        self.tensors = {
            "t_freqs": f32(H.timestep_freqs()),
            "t_w0": f32(sd["t_embedder.mlp.0.weight"]), "t_b0": f32(sd["t_embedder.mlp.0.bias"]),
            "t_w2": f32(sd["t_embedder.mlp.2.weight"]), "t_b2": f32(sd["t_embedder.mlp.2.bias"]),
            "ext_w": f32(sd["external_cond.weight"]), "ext_b": f32(sd["external_cond.bias"])}
        st = _lib.OasisCondWeights()
        for k, t in self.tensors.items():
            setattr(st, k, t.data_ptr())
        self.struct = st

    def ref(self):
        return C.byref(self.struct)


class DitDeviceWeights:
    """DiT weights resident on one GPU in the kernels' layout, plus the ctypes
    OasisDitWeights struct pointing at them (replaces the `dev` dict of
    preload_dit_weights)."""

    def __init__(self, sd: dict, device: torch.device | str = "cuda"):
        dev = torch.device(device)
        self.device = dev
        nb = count_blocks(sd)
        self.n_blocks = nb
        D = H.D_MODEL

        def bf(t):
            return t.to(dev, torch.bfloat16).contiguous()

        def f32(t):
            return t.to(dev, torch.float32).contiguous()

        self.tensors = {}
        ada_w, ada_b = [], []
        for i in range(nb):
            for s in ("s", "t"):
                p = f"blocks.{i}.{s}"
                ada_w.append(sd[f"{p}_adaLN_modulation.1.weight"])
                bias = sd[f"{p}_adaLN_modulation.1.bias"].clone().float()
                bias[D:2 * D] += 1.0  # (1 + scale_msa)
                bias[4 * D:5 * D] += 1.0  # (1 + scale_mlp)
                ada_b.append(bias)
                self.tensors[p] = dict(
                    qkv_w=bf(sd[f"{p}_attn.to_qkv.weight"]), out_w=bf(sd[f"{p}_attn.to_out.weight"]),
                    out_b=f32(sd[f"{p}_attn.to_out.bias"]), fc1_w=bf(sd[f"{p}_mlp.fc1.weight"]),
                    fc1_b=f32(sd[f"{p}_mlp.fc1.bias"]), fc2_w=bf(sd[f"{p}_mlp.fc2.weight"]),
                    fc2_b=f32(sd[f"{p}_mlp.fc2.bias"]))
        ada_w.append(sd["final_layer.adaLN_modulation.1.weight"])
        fb = sd["final_layer.adaLN_modulation.1.bias"].clone().float()
        fb[D:2 * D] += 1.0
        ada_b.append(fb)
        self.adaln_w = bf(torch.cat(ada_w, 0))
        self.adaln_b = f32(torch.cat(ada_b, 0))
        self.final_w = bf(sd["final_layer.linear.weight"])
        self.final_b = f32(sd["final_layer.linear.bias"])
        self.embed_w = f32(H.patch_embed_matrix(sd["x_embedder.proj.weight"]))
        self.embed_b = f32(sd["x_embedder.proj.bias"])
        self.rope_spatial = f32(H.rope_quad_table(H.spatial_rope_angles(sd["blocks.0.s_attn.rotary_emb.freqs"].float())))
        self.rope_temporal = f32(H.rope_quad_table(H.temporal_rope_angles(sd["blocks.0.t_attn.rotary_emb.freqs"].float())))
        # host-side conditioning weights stay on the CPU in fp32 (as in the reference)
        self.host = {k: sd[k].float() for k in ("t_embedder.mlp.0.weight", "t_embedder.mlp.0.bias",
                                                 "t_embedder.mlp.2.weight", "t_embedder.mlp.2.bias",
                                                 "external_cond.weight", "external_cond.bias")}
        # the same weights on the device for oasis_compute_cond (conditioning inside the frame graph)
        self.cond = CondDeviceWeights(sd, dev)
        self.conv_w = sd["x_embedder.proj.weight"].float()
        self.conv_b = sd["x_embedder.proj.bias"].float()

        st = _lib.OasisDitWeights()
        st.num_subblocks = 2 * nb
        for i in range(2 * nb):
            t = self.tensors[f"blocks.{i // 2}.{'s' if i % 2 == 0 else 't'}"]
            sb = st.sub[i]
            for k in ("qkv_w", "out_w", "out_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b"):
                setattr(sb, k, t[k].data_ptr())
        for k in ("adaln_w", "adaln_b", "final_w", "final_b", "embed_w", "embed_b", "rope_spatial", "rope_temporal"):
            setattr(st, k, getattr(self, k).data_ptr())
        self.struct = st

    def ref(self):
        return C.byref(self.struct)


class VaeDeviceWeights:
    """VAE decoder weights on one GPU + the ctypes OasisVaeWeights struct
    (replaces the `vae_dev` dict of preload_vae_decoder_weights)."""

    def __init__(self, sd: dict, device: torch.device | str = "cuda"):
        dev = torch.device(device)
        self.device = dev
        nb = count_blocks(sd, "decoder.")
        self.n_blocks = nb

        def bf(t):
            return t.to(dev, torch.bfloat16).contiguous()

        def f32(t):
            return t.to(dev, torch.float32).contiguous()

        self.post_quant_w = f32(sd["post_quant_conv.weight"].T)
        self.post_quant_b = f32(sd["post_quant_conv.bias"])
        self.blocks = []
        for i in range(nb):
            p = f"decoder.{i}"
            self.blocks.append(dict(
                norm1_w=f32(sd[f"{p}.norm1.weight"]), norm1_b=f32(sd[f"{p}.norm1.bias"]),
                qkv_w=bf(sd[f"{p}.attn.qkv.weight"]), qkv_b=f32(sd[f"{p}.attn.qkv.bias"]),
                proj_w=bf(sd[f"{p}.attn.proj.weight"]), proj_b=f32(sd[f"{p}.attn.proj.bias"]),
                norm2_w=f32(sd[f"{p}.norm2.weight"]), norm2_b=f32(sd[f"{p}.norm2.bias"]),
                fc1_w=bf(sd[f"{p}.mlp.fc1.weight"]), fc1_b=f32(sd[f"{p}.mlp.fc1.bias"]),
                fc2_w=bf(sd[f"{p}.mlp.fc2.weight"]), fc2_b=f32(sd[f"{p}.mlp.fc2.bias"])))
        self.norm_w = f32(sd["dec_norm.weight"])
        self.norm_b = f32(sd["dec_norm.bias"])
        self.pred_w = bf(sd["predictor.weight"])
        self.pred_b = f32(sd["predictor.bias"])
        # per-token angles from a checkpoint's RoPE table, else the axial frequencies
        ang = sd["rotary_angles"].float() if "rotary_angles" in sd else H.vae_rope_angles(sd["rotary_freqs"].float())
        self.rope = f32(H.rope_quad_table(ang))

        st = _lib.OasisVaeWeights()
        st.num_blocks = nb
        st.post_quant_w = self.post_quant_w.data_ptr()
        st.post_quant_b = self.post_quant_b.data_ptr()
        for i, blk in enumerate(self.blocks):
            for k, v in blk.items():
                setattr(st.blk[i], k, v.data_ptr())
        for k in ("norm_w", "norm_b", "pred_w", "pred_b", "rope"):
            setattr(st, k, getattr(self, k).data_ptr())
        self.struct = st

    def ref(self):
        return C.byref(self.struct)


class VaeEncoderDeviceWeights:
    """VAE encoder weights on one GPU + the ctypes OasisVaeEncoderWeights struct
    (the reference keeps the encoder on the CPU, oasis_inference.py:1738-1751)."""

    def __init__(self, sd: dict, device: torch.device | str = "cuda"):
        dev = torch.device(device)
        self.device = dev
        nb = count_blocks(sd, "encoder.")
        if nb > _lib.OASIS_VAE_BLOCKS:
            raise ValueError(f"VAE encoder with {nb} blocks; the library holds at most {_lib.OASIS_VAE_BLOCKS}")
        self.n_blocks = nb

        def bf(t):
            return t.to(dev, torch.bfloat16).contiguous()

        def f32(t):
            return t.to(dev, torch.float32).contiguous()

        pw = sd["patch_embed.proj.weight"].float().reshape(H.VAE_DIM, H.VAE_PATCH_DIM)  # (c, p, q) order
        self.patch_w = bf(torch.nn.functional.pad(pw, (0, H.VAE_ENC_K - H.VAE_PATCH_DIM)))
        self.patch_b = f32(sd["patch_embed.proj.bias"])
        self.blocks = []
        for i in range(nb):
            p = f"encoder.{i}"
            self.blocks.append(dict(
                norm1_w=f32(sd[f"{p}.norm1.weight"]), norm1_b=f32(sd[f"{p}.norm1.bias"]),
                qkv_w=bf(sd[f"{p}.attn.qkv.weight"]), qkv_b=f32(sd[f"{p}.attn.qkv.bias"]),
                proj_w=bf(sd[f"{p}.attn.proj.weight"]), proj_b=f32(sd[f"{p}.attn.proj.bias"]),
                norm2_w=f32(sd[f"{p}.norm2.weight"]), norm2_b=f32(sd[f"{p}.norm2.bias"]),
                fc1_w=bf(sd[f"{p}.mlp.fc1.weight"]), fc1_b=f32(sd[f"{p}.mlp.fc1.bias"]),
                fc2_w=bf(sd[f"{p}.mlp.fc2.weight"]), fc2_b=f32(sd[f"{p}.mlp.fc2.bias"])))
        self.norm_w = f32(sd["enc_norm.weight"])
        self.norm_b = f32(sd["enc_norm.bias"])
        self.quant_w = bf(sd["quant_conv.weight"].reshape(2 * H.VAE_LATENT, H.VAE_DIM))
        self.quant_b = f32(sd["quant_conv.bias"])
        ang = sd["rotary_angles"].float() if "rotary_angles" in sd else H.vae_rope_angles(sd["rotary_freqs"].float())
        self.rope = f32(H.rope_quad_table(ang))

        st = _lib.OasisVaeEncoderWeights()
        st.num_blocks = nb
        for i, blk in enumerate(self.blocks):
            for k, v in blk.items():
                setattr(st.blk[i], k, v.data_ptr())
        for k in ("patch_w", "patch_b", "norm_w", "norm_b", "quant_w", "quant_b", "rope"):
            setattr(st, k, getattr(self, k).data_ptr())
        self.struct = st

    def ref(self):
        return C.byref(self.struct)
