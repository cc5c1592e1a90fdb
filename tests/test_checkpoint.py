"""Checkpoint loading (CPU): the safetensors DiT / VAE files load into the state
dicts the device packers take, missing keys are named, the blob-directory search
matches the reference's, and a VAE RoPE table gives the same kernel table as the
frequencies it was built from."""
from __future__ import annotations

import os

import pytest
import torch
from safetensors.torch import save_file

from oasis_b200 import checkpoint as CK
from oasis_b200 import host as H
from oasis_b200.weights import VaeDeviceWeights, init_dit_weights, init_vae_weights


def _save(sd, path):
    save_file({k: v.contiguous() for k, v in sd.items()}, path)


def test_dit_roundtrip_and_missing_keys(tmp_path):
    sd = init_dit_weights(seed=3, n_blocks=2)
    path = str(tmp_path / "dit.safetensors")
    _save(sd, path)
    got = CK.load_dit_checkpoint(path)
    assert set(got) == set(sd)
    for k in sd:
        assert torch.equal(got[k], sd[k]), k
    del sd["blocks.1.t_mlp.fc2.bias"]
    bad = str(tmp_path / "bad.safetensors")
    _save(sd, bad)
    with pytest.raises(KeyError, match="blocks.1.t_mlp.fc2.bias"):
        CK.load_dit_checkpoint(bad)


def test_vae_rotary_table_matches_frequencies(tmp_path):
    sd = init_vae_weights(seed=4, n_blocks=1)
    freqs = sd.pop("rotary_freqs")
    path = str(tmp_path / "vae.safetensors")
    _save(sd, path)
    table = H.vae_rope_angles(freqs).reshape(H.VAE_H, H.VAE_W, H.VAE_ROT_DIM)
    with_table = CK.load_vae_checkpoint(path, rotary_table=table)
    default = CK.load_vae_checkpoint(path)
    assert "rotary_angles" in with_table and "rotary_freqs" in default
    a = VaeDeviceWeights(with_table, "cpu").rope
    b = VaeDeviceWeights({**default, "rotary_freqs": freqs}, "cpu").rope
    assert torch.allclose(a, b, atol=1e-6)
    # a table stored in the checkpoint under the module's buffer name is picked up
    _save({**sd, CK.VAE_ROTARY_BUFFER: table}, path)
    assert torch.equal(CK.load_vae_checkpoint(path)["rotary_angles"], table.reshape(H.VAE_TOKENS, -1))
    with pytest.raises(ValueError):
        CK.rotary_angles_from_table(torch.zeros(18, 32, 16))


def test_find_weights_by_prefix(tmp_path):
    d = tmp_path / "blobs"
    d.mkdir()
    (d / "0readme").write_text("not a safetensors file")
    _save({"encoder.x": torch.zeros(2)}, str(d / "a"))
    _save({"blocks.0.x": torch.zeros(2)}, str(d / "b"))
    assert os.path.basename(CK.find_weights_by_prefix(str(d), "blocks.")) == "b"
    assert os.path.basename(CK.find_weights_by_prefix(str(d), "encoder.")) == "a"
    with pytest.raises(FileNotFoundError):
        CK.find_weights_by_prefix(str(d), "decoder.")
