"""CPU restatement of the Qwen3.5 forward pass (engine/model.py:305-336) for small shapes.

TEST INFRASTRUCTURE ONLY: the checker the GPU model (qvex.qwen35) is compared against.

Composes the oracle's restatements -- qmm_exact for every projection (double accumulation,
one bf16 rounding), deltanet_conv / gated_delta / gated_rms_norm for the DeltaNet mixer
(engine/model.py:257-291), attention for the attention mixer (:210-232), swiglu for the MLP
(:300-302), rms_norm with the residual add for the layer glue (:313-316, :335) and
dequantize for the embedding (:126-130) -- in the order of the reference's code.  The
residual stream is kept as the GPU model keeps it: the MLP output of a layer is added
inside the next rms_norm, which gives the same bf16 rounding as the reference's separate
add (one rounding of x + y either way).

Parameters are a dict of numpy arrays named as the reference's checkpoint keys (bf16 as
uint16, packed weights as uint32, A_log fp32).
"""
from __future__ import annotations

import numpy as np

import oracle as O


def _lin(P, name):
    return P[f"{name}.weight"].view(np.uint32), P[f"{name}.scales"], P[f"{name}.biases"]


def _fuse(P, names):
    ws, ss, bs = zip(*(_lin(P, n) for n in names))
    return np.concatenate(ws), np.concatenate(ss), np.concatenate(bs)


def _proj(x, lin):
    """x bf16 [..., K] @ dequant(w)^T -> bf16 [..., N] (exact accumulation)."""
    w, s, b = lin
    lead = x.shape[:-1]
    y = O.qmm_exact(np.ascontiguousarray(x.reshape(-1, x.shape[-1])), w, s, b)
    return y.reshape(*lead, w.shape[0])


class Cache:
    """Per-layer state: DeltaNet conv window + recurrent matrix (+ their pre-last-token
    copies), attention key/value caches (fixed capacity) and offsets."""

    def __init__(self, cfg, B, cap):
        self.layers = []
        kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
        vd = cfg.linear_num_value_heads * cfg.linear_value_head_dim
        for i in range(cfg.num_hidden_layers):
            if cfg.is_linear(i):
                self.layers.append({
                    "conv": np.zeros((B, cfg.linear_conv_kernel_dim - 1, 2 * kd + vd), np.uint16),
                    "ssm": np.zeros((B, cfg.linear_num_value_heads, cfg.linear_value_head_dim,
                                     cfg.linear_key_head_dim), np.float32),
                    "conv_prev": None, "ssm_prev": None, "offset": 0})
            else:
                shape = (B, cfg.num_key_value_heads, cap, cfg.head_dim)
                self.layers.append({"k": np.zeros(shape, np.uint16), "v": np.zeros(shape, np.uint16), "offset": 0})

    def rollback(self):
        """RecurrentCache.rollback / KVCache.rollback (engine/model.py:175-176,189-193)."""
        for c in self.layers:
            if "ssm" in c:
                assert c["ssm_prev"] is not None
                c["conv"], c["ssm"] = c["conv_prev"], c["ssm_prev"]
                c["conv_prev"] = c["ssm_prev"] = None
            c["offset"] -= 1


def forward(cfg, P, ids, cache: Cache, keep_prev: bool = False):
    """ids int [B, L] -> (logits bf16 [B, L, vocab], pre-norm hidden bf16 [B, L, hidden])."""
    eps = cfg.rms_norm_eps
    B, L = ids.shape
    ew, es, eb = _lin(P, "model.embed_tokens")
    flat = ids.reshape(-1)
    x = O.dequantize(ew[flat], es[flat], eb[flat]).reshape(B, L, -1)
    pending = None
    for i in range(cfg.num_hidden_layers):
        pre = f"model.layers.{i}"
        c = cache.layers[i]
        if pending is None:
            n = O.rms_norm(x, P[f"{pre}.input_layernorm.weight"], eps)
        else:
            n, x = O.rms_norm(pending, P[f"{pre}.input_layernorm.weight"], eps, resid=x)
        if cfg.is_linear(i):
            la = f"{pre}.linear_attn"
            Hk, Hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
            Dk, Dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
            proj = _proj(n, _fuse(P, [f"{la}.in_proj_qkv", f"{la}.in_proj_z", f"{la}.in_proj_b", f"{la}.in_proj_a"]))
            C = 2 * Hk * Dk + Hv * Dv
            conv_w = O.bf16_to_f32(P[f"{la}.conv1d.weight"]).reshape(C, -1)
            r = O.deltanet_conv(proj, conv_w, c["conv"], Hk, Hv, Dk, Dv, keep_mid=keep_prev)
            q, k, v, a, b, c["conv"] = r[:6]
            if keep_prev:
                c["conv_prev"] = r[6]
            A_log = np.asarray(P[f"{la}.A_log"], np.float32)
            dt = O.bf16_to_f32(P[f"{la}.dt_bias"])
            g = O.gated_delta(q, k, v, a, b, A_log, dt, c["ssm"], keep_mid=keep_prev)
            y, c["ssm"] = g[0], g[1]
            if keep_prev:
                c["ssm_prev"] = g[2]
            c["offset"] += L
            z = np.ascontiguousarray(proj.reshape(B * L, -1)[:, C:C + Hv * Dv])
            yn = O.gated_rms_norm(y.reshape(B * L, Hv, Dv), z, P[f"{la}.norm.weight"], eps)
            m = _proj(yn.reshape(B, L, -1), _lin(P, f"{la}.out_proj"))
        else:
            sa = f"{pre}.self_attn"
            H, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
            qkv = _proj(n, _fuse(P, [f"{sa}.q_proj", f"{sa}.k_proj", f"{sa}.v_proj"]))
            o = O.attention(qkv, P[f"{sa}.q_norm.weight"], P[f"{sa}.k_norm.weight"], c["k"], c["v"], c["offset"], H,
                            Hkv, D, cfg.rotary_dim, cfg.rope_theta, eps, D ** -0.5)
            c["offset"] += L
            m = _proj(o, _lin(P, f"{sa}.o_proj"))
        n2, x = O.rms_norm(m, P[f"{pre}.post_attention_layernorm.weight"], eps, resid=x)
        mlp = f"{pre}.mlp"
        gu = _proj(n2, _fuse(P, [f"{mlp}.gate_proj", f"{mlp}.up_proj"]))
        pending = _proj(O.swiglu(gu.reshape(B * L, -1)).reshape(B, L, -1), _lin(P, f"{mlp}.down_proj"))
    n, h = O.rms_norm(pending, P["model.norm.weight"], eps, resid=x)
    return _proj(n, _lin(P, "lm_head")), h
