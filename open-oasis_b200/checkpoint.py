"""Loading the released Oasis-500M checkpoints (Etched/oasis-500m safetensors)
into the state dicts `DitDeviceWeights` / `VaeDeviceWeights` pack.

Reference: `oasis_inference.py:485-503` (`_find_weights_by_prefix`: the DiT file is
the safetensors blob with `blocks.*` keys, the VAE file the one with `encoder.*`
keys), `:505-677` (DiT keys read by `preload_dit_weights`) and `:679-761` (VAE
decoder keys read by `preload_vae_decoder_weights`). The key names are the
checkpoint's own; nothing is renamed.

The VAE's 2D pixel RoPE comes, in the reference, from the `rotary_freqs` buffer
of a VAE module built by `vae.py` (`:455-479`, shape (18, 32, 32): per token,
the angle of each of the 32 rotated head dims, pairs repeated). That file is not
part of the reference, so the buffer may be absent from the checkpoint: pass it
as `rotary_table` when it is available; otherwise the library's fixed axial
frequencies (`host.default_vae_freqs`) stand in, as for random-init weights.
"""
from __future__ import annotations

import os

import torch

from . import host as H

DIT_REQUIRED = [
    "x_embedder.proj.weight", "x_embedder.proj.bias",
    "t_embedder.mlp.0.weight", "t_embedder.mlp.0.bias", "t_embedder.mlp.2.weight", "t_embedder.mlp.2.bias",
    "external_cond.weight", "external_cond.bias",
    "final_layer.adaLN_modulation.1.weight", "final_layer.adaLN_modulation.1.bias",
    "final_layer.linear.weight", "final_layer.linear.bias",
    "blocks.0.s_attn.rotary_emb.freqs", "blocks.0.t_attn.rotary_emb.freqs",
]
DIT_BLOCK_KEYS = [
    "{p}_adaLN_modulation.1.weight", "{p}_adaLN_modulation.1.bias",
    "{p}_attn.to_qkv.weight", "{p}_attn.to_out.weight", "{p}_attn.to_out.bias",
    "{p}_mlp.fc1.weight", "{p}_mlp.fc1.bias", "{p}_mlp.fc2.weight", "{p}_mlp.fc2.bias",
]
VAE_REQUIRED = ["post_quant_conv.weight", "post_quant_conv.bias", "dec_norm.weight", "dec_norm.bias",
                "predictor.weight", "predictor.bias"]
VAE_BLOCK_KEYS = ["norm1.weight", "norm1.bias", "attn.qkv.weight", "attn.qkv.bias", "attn.proj.weight",
                  "attn.proj.bias", "norm2.weight", "norm2.bias", "mlp.fc1.weight", "mlp.fc1.bias",
                  "mlp.fc2.weight", "mlp.fc2.bias"]
VAE_ROTARY_BUFFER = "decoder.0.attn.rotary_freqs"
# The encoder half of the same file (vae.encode, oasis_inference.py:1748-1751). Its
# module definition is not in the reference; these names follow the decoder's.
VAE_ENC_REQUIRED = ["patch_embed.proj.weight", "patch_embed.proj.bias", "enc_norm.weight", "enc_norm.bias",
                    "quant_conv.weight", "quant_conv.bias"]
VAE_ENC_ROTARY_BUFFER = "encoder.0.attn.rotary_freqs"


def _load(path: str) -> dict:
    from safetensors.torch import load_file

    return load_file(path)


def _keys(path: str) -> list[str]:
    from safetensors import safe_open

    with safe_open(path, framework="pt") as st:
        return list(st.keys())


def find_weights_by_prefix(blob_dir: str, prefix: str) -> str:
    """The safetensors file in `blob_dir` that holds a key starting with `prefix`
    (files that are not safetensors are skipped), as `_find_weights_by_prefix`
    (oasis_inference.py:485-497) does in the Hugging Face blob directory."""
    for name in sorted(os.listdir(blob_dir)):
        path = os.path.join(blob_dir, name)
        try:
            if any(k.startswith(prefix) for k in _keys(path)):
                return path
        except Exception:  # not a safetensors file (README, .gitattributes, ...)
            continue
    raise FileNotFoundError(f"weights with prefix {prefix!r} not found in {blob_dir}")


def _count(sd: dict, prefix: str) -> int:
    idx = {int(k.split(".")[1]) for k in sd if k.startswith(prefix) and k.split(".")[1].isdigit()}
    return max(idx) + 1 if idx else 0


def load_dit_checkpoint(path: str) -> dict:
    """DiT state dict from a safetensors file; raises KeyError naming every missing key."""
    sd = _load(path)
    n = _count(sd, "blocks.")
    want = list(DIT_REQUIRED)
    for i in range(n):
        for s in ("s", "t"):
            want += [k.format(p=f"blocks.{i}.{s}") for k in DIT_BLOCK_KEYS]
    missing = [k for k in want if k not in sd]
    if n == 0 or missing:
        raise KeyError(f"{path}: not an Oasis DiT checkpoint ({n} blocks); missing {missing[:8]}"
                       f"{' ...' if len(missing) > 8 else ''}")
    return sd


def load_vae_checkpoint(path: str, rotary_table: torch.Tensor | None = None) -> dict:
    """VAE decoder state dict from a safetensors file. The pixel RoPE is taken from
    `rotary_table` (18, 32, 32) if given, else from the checkpoint's
    `decoder.0.attn.rotary_freqs` buffer if present, else the fixed default
    frequencies; it is stored as `rotary_angles` (576, 32) or `rotary_freqs`."""
    sd = _load(path)
    n = _count(sd, "decoder.")
    want = list(VAE_REQUIRED) + [f"decoder.{i}.{k}" for i in range(n) for k in VAE_BLOCK_KEYS]
    missing = [k for k in want if k not in sd]
    if n == 0 or missing:
        raise KeyError(f"{path}: not an Oasis VAE checkpoint ({n} decoder blocks); missing {missing[:8]}"
                       f"{' ...' if len(missing) > 8 else ''}")
    table = rotary_table if rotary_table is not None else sd.get(VAE_ROTARY_BUFFER)
    if table is not None:
        sd["rotary_angles"] = rotary_angles_from_table(table)
    elif "rotary_freqs" not in sd:
        sd["rotary_freqs"] = H.default_vae_freqs()
    return sd


def load_vae_encoder_checkpoint(path: str, rotary_table: torch.Tensor | None = None) -> dict:
    """VAE encoder state dict from the same safetensors file (the one
    `_find_weights_by_prefix("encoder.")` finds, oasis_inference.py:499-503).
    Pixel RoPE as in load_vae_checkpoint, from `encoder.0.attn.rotary_freqs` when
    the file holds it."""
    sd = _load(path)
    n = _count(sd, "encoder.")
    want = list(VAE_ENC_REQUIRED) + [f"encoder.{i}.{k}" for i in range(n) for k in VAE_BLOCK_KEYS]
    missing = [k for k in want if k not in sd]
    if n == 0 or missing:
        raise KeyError(f"{path}: not an Oasis VAE encoder checkpoint ({n} encoder blocks); missing {missing[:8]}"
                       f"{' ...' if len(missing) > 8 else ''}")
    table = rotary_table if rotary_table is not None else sd.get(VAE_ENC_ROTARY_BUFFER, sd.get(VAE_ROTARY_BUFFER))
    if table is not None:
        sd["rotary_angles"] = rotary_angles_from_table(table)
    elif "rotary_freqs" not in sd:
        sd["rotary_freqs"] = H.default_vae_freqs()
    return sd


def rotary_angles_from_table(table: torch.Tensor) -> torch.Tensor:
    """(18, 32, 32) per-token angles of the 32 rotated dims (pairs repeated, the
    layout of the reference's `rotary_freqs` buffer) -> (576, 32)."""
    t = table.float()
    if tuple(t.shape) != (H.VAE_H, H.VAE_W, H.VAE_ROT_DIM):
        raise ValueError(f"VAE rotary table must be ({H.VAE_H}, {H.VAE_W}, {H.VAE_ROT_DIM}), got {tuple(t.shape)}")
    return t.reshape(H.VAE_TOKENS, H.VAE_ROT_DIM).contiguous()
