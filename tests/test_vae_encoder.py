"""VAE encoder for the prompt image (`vae.encode(x).mean * SCALING_FACTOR`,
oasis_inference.py:1748-1751, then the rearrange + patchify that feeds the
context patch embed, :1752-1754, 1806-1809).

CPU: the kernel's patch-row order restated here reproduces the conv patch embed
with the packed weights; the encoder's chunk layout is the inverse of the DiT->VAE
bridge; the checkpoint loader reads the encoder half of the VAE file. GPU: the
C-ABI encoder against the oracle at the spec's bar (rel-L2 <= 1e-2, cos >= 0.999)."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F
from safetensors.torch import save_file

from oracle import oasis_oracle as O
from oasis_b200 import checkpoint as CK
from oasis_b200 import host as H
from oasis_b200.weights import VaeEncoderDeviceWeights, init_vae_encoder_weights
from tests.helpers import COS_TOL, REL_L2_TOL, cosine, rel_l2


def _image(B, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(B, 3, 360, 640, generator=g) * 2 - 1


def _patch_rows(img: torch.Tensor, kp: int) -> torch.Tensor:
    """image_patchify_kernel's map: row (b, i*32 + j), column c*400 + p*20 + q, zero pad to kp."""
    B = img.shape[0]
    x = img.reshape(B, 3, 18, 20, 32, 20).permute(0, 2, 4, 1, 3, 5).reshape(B, 576, 1200)
    return F.pad(x, (0, kp - 1200))


def test_patch_rows_and_packed_weights_reproduce_the_conv():
    sd = init_vae_encoder_weights(seed=7, n_blocks=0, bias_std=0.02)
    ew = VaeEncoderDeviceWeights(sd, "cpu")
    assert tuple(ew.patch_w.shape) == (1024, H.VAE_ENC_K) and ew.patch_w[:, 1200:].abs().max() == 0
    img = _image(2, 0)
    conv = F.conv2d(img, sd["patch_embed.proj.weight"], sd["patch_embed.proj.bias"], stride=20)
    conv = conv.permute(0, 2, 3, 1).reshape(2, 576, 1024)
    w = sd["patch_embed.proj.weight"].reshape(1024, 1200)
    gemm = _patch_rows(img, H.VAE_ENC_K) @ F.pad(w, (0, H.VAE_ENC_K - 1200)).T + sd["patch_embed.proj.bias"]
    assert torch.allclose(gemm, conv, atol=1e-4)
    # the patch rows are the inverse of the decoder's image unpatchify
    rows = _patch_rows(img, 1200)
    assert torch.equal(O.vae_unpatchify(rows), img)


def test_chunk_layout_is_the_inverse_of_the_bridge():
    g = torch.Generator().manual_seed(1)
    lat = torch.randn(3, 576, 16, generator=g)
    chunk = O.latent_to_chunk(lat)
    assert tuple(chunk.shape) == (3, 144, 64)
    assert torch.allclose(O.bridge(chunk) * H.SCALING_FACTOR, lat, atol=1e-6)
    # moments_to_latent_kernel's index map, restated
    b, t, c = 1, 5 * 32 + 7, 3
    row, col = t // 32, t % 32
    assert chunk[b, (row // 2) * 16 + col // 2, (row % 2) * 32 + (col % 2) * 16 + c] == lat[b, t, c]


def test_oracle_encoder_shape_and_mean():
    sd = init_vae_encoder_weights(seed=2, n_blocks=1, bias_std=0.02, norm_std=0.1)
    lat = O.vae_encode(_image(1, 3), sd)
    assert tuple(lat.shape) == (1, 576, 16) and torch.isfinite(lat).all()
    # the posterior mean is the first half of quant_conv
    sd2 = dict(sd)
    sd2["quant_conv.weight"] = sd["quant_conv.weight"].clone()
    sd2["quant_conv.weight"][16:] = 0
    assert torch.equal(O.vae_encode(_image(1, 3), sd2), lat)


def test_encoder_checkpoint_roundtrip(tmp_path):
    sd = init_vae_encoder_weights(seed=4, n_blocks=2)
    freqs = sd.pop("rotary_freqs")
    path = str(tmp_path / "vae.safetensors")
    save_file({k: v.contiguous() for k, v in sd.items()}, path)
    got = CK.load_vae_encoder_checkpoint(path)
    assert torch.equal(got["rotary_freqs"], H.default_vae_freqs()) and torch.equal(freqs, H.default_vae_freqs())
    for k in sd:
        assert torch.equal(got[k], sd[k]), k
    assert VaeEncoderDeviceWeights(got, "cpu").n_blocks == 2
    del sd["encoder.1.mlp.fc1.bias"]
    save_file({k: v.contiguous() for k, v in sd.items()}, path)
    with pytest.raises(KeyError, match="encoder.1.mlp.fc1.bias"):
        CK.load_vae_encoder_checkpoint(path)


@pytest.mark.gpu
@pytest.mark.parametrize("B,n_blocks", [(1, 1), (2, H.VAE_ENC_DEPTH)])
def test_vae_encode_matches_oracle(B, n_blocks):
    from oasis_b200 import engine as E

    dev = torch.device("cuda")
    sd = init_vae_encoder_weights(seed=5, n_blocks=n_blocks, bias_std=0.02, norm_std=0.1)
    ew = VaeEncoderDeviceWeights(sd, dev)
    img = _image(B, 11)
    ref = O.vae_encode(img, sd)
    lat = torch.empty(B, 576, 16, device=dev)
    chunk = torch.empty(B, 144, 64, device=dev)
    E.vae_encode(ew, img.to(dev), E.workspace(E.vae_encoder_workspace_bytes(B), dev), latent=lat, chunk=chunk)
    torch.cuda.synchronize()
    assert rel_l2(lat, ref) < REL_L2_TOL and cosine(lat, ref) > COS_TOL, (rel_l2(lat, ref), cosine(lat, ref))
    assert torch.equal(chunk.cpu(), O.latent_to_chunk(lat.cpu()))
    # chunk only
    chunk2 = torch.zeros_like(chunk)
    E.vae_encode(ew, img.to(dev), E.workspace(E.vae_encoder_workspace_bytes(B), dev), chunk=chunk2)
    assert torch.equal(chunk2, chunk)


def _prompt_context_case(dev):
    """VideoEngine.set_prompt on B = 2 prompt images with T = 3: the encoded prompt,
    patch-embedded into both context slots, against the oracle's encode ->
    latent_to_chunk -> patch_embed; the conditioning window is the prompt's."""
    from oasis_b200 import engine as E
    from oasis_b200.weights import DitDeviceWeights, VaeDeviceWeights, init_dit_weights, init_vae_weights

    dsd = init_dit_weights(seed=1, n_blocks=1, bias_std=0.02)
    esd = init_vae_encoder_weights(seed=5, n_blocks=1, bias_std=0.02, norm_std=0.1)
    dw = DitDeviceWeights(dsd, dev)
    vw = VaeDeviceWeights(init_vae_weights(seed=2, n_blocks=1), dev)
    ew = VaeEncoderDeviceWeights(esd, dev)
    B, T = 2, 3
    img = _image(B, 13)
    cond = torch.randn(B, 1024, generator=torch.Generator().manual_seed(14))
    ve = E.VideoEngine(dw, vw, B, T)
    ve.set_prompt(ew, img.to(dev), cond.to(dev))
    if dev.type == "cuda":
        torch.cuda.synchronize()
    z = O.patch_embed(O.unpatchify(O.latent_to_chunk(O.vae_encode(img, esd))), dsd)  # (B, 144, 1024)
    ref = z[:, None].expand(B, T - 1, 144, 1024)
    got = ve.context_z.cpu()
    assert rel_l2(got, ref) < REL_L2_TOL and cosine(got, ref) > COS_TOL, (rel_l2(got, ref), cosine(got, ref))
    assert torch.equal(got[:, 0], got[:, 1])
    assert torch.equal(ve.ctx_cond.cpu(), cond[:, None].expand(B, T - 1, 1024))


@pytest.mark.gpu
def test_video_engine_starts_from_prompt_images():
    _prompt_context_case(torch.device("cuda"))
