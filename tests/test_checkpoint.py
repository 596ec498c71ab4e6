"""Checkpoint formats on CPU (qvex.checkpoint): the MLX safetensors directory the reference
loads (engine/model.py:342-397) and the reference's .q35 file
(experiments/native/convert_native.py).  Every tensor must come back bit for bit."""
import json
import struct

import pytest
import torch

from test_model_oracle import small_cfg


@pytest.fixture(scope="module")
def params():
    from qvex.qwen35 import random_params
    cfg = small_cfg()
    return cfg, random_params(cfg, 5, "cpu")


def same(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a.view(torch.uint8) if a.dtype != torch.bool
                                                                      else a, b.view(torch.uint8))


def test_safetensors_round_trip(tmp_path):
    from qvex.checkpoint import read_safetensors, write_safetensors
    t = {"a": torch.randn(3, 5).to(torch.bfloat16), "w": torch.randint(-2 ** 31, 2 ** 31, (4, 2), dtype=torch.int64)
         .to(torch.int32), "f": torch.randn(7), "e": torch.zeros(0, 3)}
    write_safetensors(tmp_path / "x.safetensors", t, {"format": "mlx"})
    back, meta = read_safetensors(tmp_path / "x.safetensors")
    assert meta == {"format": "mlx"}
    for k in t:
        assert same(back[k].contiguous(), t[k].contiguous()), k
    # the header is the documented layout: 8-byte length, JSON, data
    raw = (tmp_path / "x.safetensors").read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + n])
    assert hdr["w"]["dtype"] == "U32" and hdr["a"]["shape"] == [3, 5]


def test_checkpoint_directory_round_trip(tmp_path, params):
    from qvex.checkpoint import expected_keys, read_checkpoint, save_checkpoint, write_safetensors
    from qvex.qwen35 import Config
    cfg, P = params
    save_checkpoint(tmp_path, cfg, P, shards=3)
    # a tensor of the vision tower is never read (engine/model.py keeps language_model.* only)
    write_safetensors(tmp_path / "vision.safetensors", {"vision_tower.blocks.0.w": torch.zeros(2, 2)})
    back = read_checkpoint(tmp_path)
    assert set(back) == set(P) == set(expected_keys(cfg))
    for k in P:
        assert same(back[k], P[k].contiguous()), k
    c2 = Config.from_file(tmp_path / "config.json")
    assert c2 == cfg


def test_model_prefix_remap_and_mtp_refused(tmp_path, params):
    from qvex.checkpoint import read_checkpoint, remap_key, save_checkpoint
    cfg, P = params
    assert remap_key("model.language_model.layers.0.x") == "model.layers.0.x"
    assert remap_key("language_model.lm_head.weight") == "lm_head.weight"
    assert remap_key("vision_tower.patch_embed") is None
    save_checkpoint(tmp_path, cfg, {**P, "mtp.fc.weight": torch.zeros(2, 2, dtype=torch.int32)}, shards=1)
    with pytest.raises(ValueError, match="mtp"):
        read_checkpoint(tmp_path)


def test_load_model_builds_the_fused_layers(tmp_path, params):
    from qvex.checkpoint import load_model, save_checkpoint
    cfg, P = params
    save_checkpoint(tmp_path, cfg, P)
    m = load_model(tmp_path, device="cpu")
    la = "model.layers.0.linear_attn"
    want = torch.cat([P[f"{la}.{n}.weight"] for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")])
    assert torch.equal(m.layers[0].mixer.in_proj.w, want)
    sa = "model.layers.3.self_attn"
    want = torch.cat([P[f"{sa}.{n}.scales"] for n in ("q_proj", "k_proj", "v_proj")])
    assert same(m.layers[3].mixer.qkv.scales, want)
    assert m.layers[0].mixer.A_log.dtype == torch.float32


def test_other_quantization_refused(tmp_path, params):
    import dataclasses
    from qvex.checkpoint import load_model, save_checkpoint
    cfg, P = params
    c8 = dataclasses.replace(cfg, quant={"model.layers.1.mlp.down_proj": {"bits": 8, "group_size": 64}})
    save_checkpoint(tmp_path, c8, P)
    with pytest.raises(NotImplementedError, match="down_proj"):
        load_model(tmp_path, device="cpu")


def test_q35_layout_and_round_trip(tmp_path, params):
    from qvex.checkpoint import Q35_ALIGN, Q35_PAGE, q35_params, read_q35, write_q35
    cfg, P = params
    path = tmp_path / "model.q35"
    size = write_q35(path, cfg, P)
    raw = path.read_bytes()
    assert len(raw) == size and size % Q35_PAGE == 0 and raw[:4] == b"Q35W"
    assert struct.unpack_from("<I", raw, 4)[0] == 1
    ints = struct.unpack_from("<16i", raw, 8)
    assert ints[0] == cfg.hidden_size and ints[12] == cfg.vocab_size and ints[13] == cfg.rotary_dim
    c2, T = read_q35(path)
    # the layout keeps eps and rope theta as float32 (what the kernels use anyway)
    import dataclasses
    import numpy as np
    assert np.float32(c2.rms_norm_eps) == np.float32(cfg.rms_norm_eps)
    assert np.float32(c2.rope_theta) == np.float32(cfg.rope_theta)
    assert dataclasses.replace(c2, rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta) == cfg
    # fused as the native converter stores them (convert_native.py:13-16)
    assert "L0.in.w" in T and "L3.qkv.w" in T and "L0.gu.w" in T and "L0.conv" in T
    assert T["L0.conv"].dtype == torch.float32 and T["L0.conv"].shape == (2 * 256 + 512, 4)
    n = struct.unpack_from("<I", raw, 80)[0]
    for j in range(n):
        off = struct.unpack_from("<64sII4QQQ", raw, 84 + j * 120)[7]  # 120-byte entries
        assert off % Q35_ALIGN == 0
    back = q35_params(c2, T)
    assert set(back) == set(P)
    for k in P:
        assert same(back[k].contiguous(), P[k].contiguous()), k
