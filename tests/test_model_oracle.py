"""The CPU model oracle (oracle/qwen35_oracle.py) and the model's host-side pieces, on CPU.

The oracle's cache semantics are checked against themselves: feeding a sequence in one
prefill or in pieces (prefill then decode steps), or verifying two tokens with keep_prev
and rolling one back, must give bit-identical logits, because every restated op is
sequential in the tokens (conv window, recurrence, attention over the same keys in the
same order) and row-independent elsewhere.  Also: Config.from_dict reads a checkpoint's
config.json the way the reference does (engine/model.py:39-66)."""
import numpy as np
import pytest
import torch

import oracle as O
import qwen35_oracle as QO


def small_cfg(layers=4):
    from qvex.qwen35 import Config
    return Config(hidden_size=512, intermediate_size=1024, num_hidden_layers=layers, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=128, linear_num_key_heads=2, linear_num_value_heads=4,
                  linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
                  full_attention_interval=4, rms_norm_eps=1e-6, vocab_size=2048, rope_theta=1e7, rotary_dim=32)


def numpy_params(P):
    out = {}
    for k, v in P.items():
        v = v.cpu()
        if v.dtype == torch.bfloat16:
            out[k] = v.view(torch.int16).numpy().view(np.uint16)
        elif v.dtype == torch.int32:
            out[k] = v.numpy().view(np.uint32)
        else:
            out[k] = v.numpy()
    return out


@pytest.fixture(scope="module")
def model_np():
    from qvex.qwen35 import random_params
    cfg = small_cfg()
    return cfg, numpy_params(random_params(cfg, 7, "cpu"))


def test_prefill_equals_prefill_then_decode(model_np):
    cfg, P = model_np
    ids = np.random.default_rng(0).integers(0, cfg.vocab_size, (2, 7))
    c1 = QO.Cache(cfg, 2, 16)
    full, _ = QO.forward(cfg, P, ids, c1)
    c2 = QO.Cache(cfg, 2, 16)
    QO.forward(cfg, P, ids[:, :5], c2)
    QO.forward(cfg, P, ids[:, 5:6], c2)
    last, _ = QO.forward(cfg, P, ids[:, 6:7], c2)
    assert np.array_equal(last[:, 0], full[:, 6])


def test_verify_then_rollback(model_np):
    cfg, P = model_np
    rng = np.random.default_rng(1)
    ids = rng.integers(0, cfg.vocab_size, (1, 6))
    other = rng.integers(0, cfg.vocab_size, (1, 1))
    c = QO.Cache(cfg, 1, 16)
    QO.forward(cfg, P, ids[:, :4], c)
    QO.forward(cfg, P, ids[:, 4:6], c, keep_prev=True)  # verify two tokens
    c.rollback()                                         # reject the second
    got, _ = QO.forward(cfg, P, other, c)
    ref_ids = np.concatenate([ids[:, :5], other], axis=1)
    ref, _ = QO.forward(cfg, P, ref_ids, QO.Cache(cfg, 1, 16))
    assert np.array_equal(got[:, 0], ref[:, 5])


def test_config_from_checkpoint_json():
    from qvex.qwen35 import Config
    raw = {"text_config": {"hidden_size": 4096, "intermediate_size": 12288, "num_hidden_layers": 32,
                           "num_attention_heads": 32, "num_key_value_heads": 4, "head_dim": 256,
                           "linear_num_key_heads": 16, "linear_num_value_heads": 32, "linear_key_head_dim": 128,
                           "linear_value_head_dim": 128, "linear_conv_kernel_dim": 4, "rms_norm_eps": 1e-6,
                           "vocab_size": 248320, "rope_parameters": {"rope_theta": 1e7, "partial_rotary_factor": 0.25}},
           "quantization": {"group_size": 64, "bits": 4, "language_model.model.layers.3.mlp.down_proj": {"bits": 8}}}
    c = Config.from_dict(raw)
    assert c.rotary_dim == 64 and c.head_dim == 256 and c.full_attention_interval == 4
    assert c.qparams("model.layers.3.mlp.down_proj") == (64, 8) and c.qparams("lm_head") == (64, 4)
    assert [c.is_linear(i) for i in range(8)] == [True, True, True, False] * 2


def test_qwen35_9b_projection_shapes():
    from qvex.qwen35 import Config, quantized_shapes
    from qvex.shapes import Qwen35Shape
    cfg = Config.qwen35_9b()
    q = quantized_shapes(cfg)
    # the fused decode projections of the benchmark's step come out of the same shapes
    in_proj = sum(q[f"model.layers.0.linear_attn.{n}"][0] for n in ("in_proj_qkv", "in_proj_z", "in_proj_b",
                                                                      "in_proj_a"))
    names = {n: N for n, N, _ in Qwen35Shape().decode_linears()}
    assert in_proj == names["layers.0.linear_attn.in_proj"] == 12352
    assert q["model.layers.3.self_attn.q_proj"] == (8192, 4096) and q["lm_head"] == (248320, 4096)
