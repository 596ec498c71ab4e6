"""Qwen3.5 hybrid decoder (gated DeltaNet + gated attention) on libqvex kernels.

Mirrors the reference's forward pass (engine/model.py): the classes ``Config``,
``KVCache``, ``RecurrentCache``, ``Attention``, ``GatedDeltaNet``, ``MLP``, ``Layer`` and
``Qwen35`` keep the reference's constructor arguments, call signatures and cache
semantics (keep_prev snapshots, one-token rollback, KV offset rollback), with torch CUDA
tensors in place of MLX arrays.  Every layer op runs a libqvex kernel:

  projections           qvx_qmv (M <= 8) / qvx_qmm (M > 8)          QLinear
  rms_norm (+ residual) qvx_rms_norm                                engine/model.py:314-316,335
  DeltaNet conv path    qvx_deltanet_conv                           :259-277
  recurrence            qvx_gated_delta                             :279-286
  gated rms_norm        qvx_gated_rms_norm                          :289-290
    (up to 4 tokens, while the clusters fit: the three in qvx_deltanet_decode)
  attention             qvx_attention (one decode kernel, or prep + prefill)  :213-232
  SwiGLU                gate|up epilogue (decode) / qvx_swiglu_pairs  :300-302
  residual add          qvx_add (or fused into the next rms_norm)   :316
  embedding             qvx_dequantize_rows                         :126-130

Projections that share an input are fused at construction, as the reference does for
DeltaNet's qkv|z|b|a and the MLP's gate|up (engine/model.py:244-246,296) and as its native
converter does for attention's q|k|v (experiments/native/convert_native.py:13-16).

``Qwen35.random(cfg, ...)`` builds a random-initialised model of any shape with synthetic
4-bit weights (codes uniform in 0..15, scales |N(0,1)|*0.002, biases -8*scale).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

import torch

from . import glue
from .core import QMM_MIN_M_PREPARED, dequantize_rows, qmv_fused
from .kernels import gated_delta
from .model import QEmbedding, QLinear, RecurrentCache

__all__ = ["Config", "KVCache", "RecurrentCache", "Attention", "GatedDeltaNet", "MLP", "Layer", "Qwen35"]


@dataclass
class Config:
    """Model hyper-parameters (the fields of engine/model.py:17-37)."""
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    full_attention_interval: int
    rms_norm_eps: float
    vocab_size: int
    rope_theta: float
    rotary_dim: int
    group_size: int = 64
    bits: int = 4
    quant: dict = field(default_factory=dict)

    @classmethod
    def from_dict(cls, raw: dict) -> "Config":
        """From a checkpoint's config.json contents (engine/model.py:39-66 reads the same keys:
        text_config nesting, rope_parameters, the quantization block with per-module overrides)."""
        t = raw.get("text_config", raw)
        rope = t.get("rope_parameters") or {}
        q = raw.get("quantization") or raw.get("quantization_config") or {}
        head_dim = t.get("head_dim") or t["hidden_size"] // t["num_attention_heads"]
        return cls(
            hidden_size=t["hidden_size"], intermediate_size=t["intermediate_size"],
            num_hidden_layers=t["num_hidden_layers"], num_attention_heads=t["num_attention_heads"],
            num_key_value_heads=t["num_key_value_heads"], head_dim=head_dim,
            linear_num_key_heads=t["linear_num_key_heads"], linear_num_value_heads=t["linear_num_value_heads"],
            linear_key_head_dim=t["linear_key_head_dim"], linear_value_head_dim=t["linear_value_head_dim"],
            linear_conv_kernel_dim=t["linear_conv_kernel_dim"],
            full_attention_interval=t.get("full_attention_interval", 4), rms_norm_eps=t["rms_norm_eps"],
            vocab_size=t["vocab_size"], rope_theta=rope.get("rope_theta", t.get("rope_theta", 10_000_000)),
            rotary_dim=int(head_dim * rope.get("partial_rotary_factor", 0.25)),
            group_size=q.get("group_size", 64), bits=q.get("bits", 4),
            quant={k.removeprefix("language_model."): v for k, v in q.items() if isinstance(v, dict)},
        )

    @classmethod
    def from_file(cls, path: Path) -> "Config":
        return cls.from_dict(json.loads(Path(path).read_text()))

    @classmethod
    def qwen35_9b(cls, kv_heads: int = 8, layers: int = 32) -> "Config":
        """The Qwen3.5-9B text shape the benchmark names: hidden 4096, MLP 12288, 32 layers
        (24 gated DeltaNet + 8 gated attention), 32 x 128 attention heads with ``kv_heads``
        KV heads, DeltaNet 16 key / 32 value heads of 128, conv kernel 4, vocab 248320."""
        return cls(hidden_size=4096, intermediate_size=12288, num_hidden_layers=layers, num_attention_heads=32,
                   num_key_value_heads=kv_heads, head_dim=128, linear_num_key_heads=16, linear_num_value_heads=32,
                   linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
                   full_attention_interval=4, rms_norm_eps=1e-6, vocab_size=248320, rope_theta=10_000_000.0,
                   rotary_dim=32)

    def qparams(self, module: str) -> tuple[int, int]:
        """(group_size, bits) of one quantized module, with per-module overrides."""
        o = self.quant.get(module, {})
        return o.get("group_size", self.group_size), o.get("bits", self.bits)

    def is_linear(self, i: int) -> bool:
        return (i + 1) % self.full_attention_interval != 0


# ---------------------------------------------------------------- caches


class KVCache:
    """Key/value cache of one attention layer (engine/model.py:149-176): bf16 [B, Hkv, cap,
    D] buffers grown in steps of 256 positions, ``offset`` positions filled; rollback only
    moves the offset back (later writes overwrite)."""
    step = 256

    def __init__(self, capacity: int | None = None):
        self.k = self.v = None
        self.offset = 0
        self.capacity = capacity  # fixed size (CUDA-graph decode) instead of growing

    def reserve(self, B: int, H: int, D: int, L: int, device) -> None:
        """Room for L more positions (the allocation half of KVCache.update)."""
        need = self.offset + L
        if self.k is not None and need <= self.k.shape[2]:
            return
        n = self.capacity if self.capacity is not None else ((need + self.step - 1) // self.step) * self.step
        if n < need:
            raise ValueError(f"KV cache of {n} positions cannot hold {need}")
        nk = torch.zeros((B, H, n, D), dtype=torch.bfloat16, device=device)
        nv = torch.zeros_like(nk)
        if self.k is not None:
            nk[:, :, :self.offset] = self.k[:, :, :self.offset]
            nv[:, :, :self.offset] = self.v[:, :, :self.offset]
        self.k, self.v = nk, nv

    def state(self):
        return [self.k, self.v] if self.k is not None else []

    def rollback(self, n: int = 1) -> None:
        self.offset -= n


# ---------------------------------------------------------------- layers


def _qlin(p) -> QLinear:
    return p if isinstance(p, QLinear) else QLinear(*p)


def _fused(lin: QLinear, x: torch.Tensor, prologue: str, **kw) -> torch.Tensor:
    return qmv_fused(x, lin.w, lin.scales, lin.biases, prologue=prologue, group_size=lin.group_size, bits=lin.bits,
                     **kw)


class Attention:
    """Gated full attention (engine/model.py:199-232)."""

    def __init__(self, cfg: Config, p: dict):
        self.cfg = cfg
        self.n_heads, self.n_kv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.head_dim = cfg.head_dim
        self.scale = cfg.head_dim ** -0.5
        # q_proj | k_proj | v_proj share the input: one projection (rows concatenated)
        self.qkv = QLinear.fuse([_qlin(p["q_proj"]), _qlin(p["k_proj"]), _qlin(p["v_proj"])])
        self.o_proj = _qlin(p["o_proj"])
        self.q_norm, self.k_norm = p["q_norm"], p["k_norm"]
        self.inv_freq = glue.rope_inv_freq(cfg.rotary_dim, cfg.rope_theta, self.q_norm.device)
        self._ws = {}

    def workspace(self, B: int, L: int, nsplit: int):
        key = (B, L, nsplit)
        if key not in self._ws:
            self._ws[key] = glue.attention_workspace(B, self.n_kv, self.n_heads // self.n_kv, L, self.head_dim, nsplit,
                                                     self.q_norm.device)
        return self._ws[key]

    def mix(self, x: torch.Tensor, cache: KVCache, pos=None) -> torch.Tensor:
        """The o_proj input [B, L, H*D] (everything of __call__ but o_proj).  ``pos`` (a device
        int32 tensor) overrides cache.offset for CUDA-graph decode."""
        return self.attend(self.qkv(x), cache, pos)

    def attend(self, qkv: torch.Tensor, cache: KVCache, pos=None) -> torch.Tensor:
        """From the fused q|k|v projection output [B, L, *] to the o_proj input."""
        B, L, _ = qkv.shape
        x = qkv
        cache.reserve(B, self.n_kv, self.head_dim, L, x.device)
        G = self.n_heads // self.n_kv
        ws, ns = None, 0
        if G * L <= 8:
            ns = glue.default_splits(B, self.n_kv, x.device, cap=cache.k.shape[2])
            ws = self.workspace(B, L, ns)
        o = glue.attention(qkv, self.q_norm, self.k_norm, self.cfg.rms_norm_eps, self.inv_freq, cache.k, cache.v,
                           cache.offset if pos is None else pos, self.n_heads, self.n_kv, self.head_dim,
                           scale=self.scale, workspace=ws, nsplit=ns)
        cache.offset += L
        return o

    def __call__(self, x: torch.Tensor, cache: KVCache) -> torch.Tensor:
        return self.o_proj(self.mix(x, cache))


class GatedDeltaNet:
    """Gated DeltaNet linear attention (engine/model.py:235-291)."""

    # up to 4 tokens (decode, verify) in one kernel where the shape allows; False runs the
    # three-kernel path (conv, recurrence, gated norm), which gives the same bits
    fused_decode = True

    def __init__(self, cfg: Config, p: dict):
        self.cfg = cfg
        self.hk, self.hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        self.key_dim, self.value_dim = self.hk * self.dk, self.hv * self.dv
        self.conv_dim = 2 * self.key_dim + self.value_dim
        self.K = cfg.linear_conv_kernel_dim
        # qkv | z | b | a share the input -> one fused quantized matmul
        self.in_proj = QLinear.fuse([_qlin(p["in_proj_qkv"]), _qlin(p["in_proj_z"]), _qlin(p["in_proj_b"]),
                                     _qlin(p["in_proj_a"])])
        self.splits = [self.conv_dim, self.conv_dim + self.value_dim, self.conv_dim + self.value_dim + self.hv]
        cw = p["conv1d"]
        self.conv_w = cw.reshape(self.conv_dim, self.K).to(torch.float32).contiguous()  # [conv_dim, K]
        self.A_log = p["A_log"].to(torch.float32).contiguous()
        self.dt_bias = p["dt_bias"].to(torch.float32).contiguous()
        self.norm_w = p["norm"]
        self.out_proj = _qlin(p["out_proj"])

    def init_state(self, cache: RecurrentCache, B: int, device) -> None:
        """Zero conv window and recurrent state for B sequences."""
        cache.conv = torch.zeros((B, self.K - 1, self.conv_dim), dtype=torch.bfloat16, device=device)
        cache.ssm = torch.zeros((B, self.hv, self.dv, self.dk), dtype=torch.float32, device=device)

    def mix(self, x: torch.Tensor, cache: RecurrentCache, keep_prev: bool = False,
            inplace: bool = False) -> torch.Tensor:
        """The out_proj input [B, S, Hv*Dv] (everything of __call__ but out_proj).  With
        ``inplace`` the conv window and recurrent state are updated in their own buffers (the
        form a CUDA graph replays); otherwise new tensors replace them, as in the reference."""
        return self.mix_proj(self.in_proj(x), cache, keep_prev, inplace)

    def mix_proj(self, proj: torch.Tensor, cache: RecurrentCache, keep_prev: bool = False,
                 inplace: bool = False) -> torch.Tensor:
        """mix() from the in_proj output [B, S, *] on."""
        B, S, _ = proj.shape
        x = proj
        if self.fused_decode and glue.deltanet_decode_preferred(B, S, self.hk, self.hv, self.dk, self.dv, x.device):
            # decode / verify: conv, recurrence and gated norm in one kernel (same bits)
            if cache.conv is None:
                self.init_state(cache, B, x.device)
            r = glue.deltanet_decode(proj, self.conv_w, cache.conv, self.A_log, self.dt_bias, cache.ssm, self.norm_w,
                                     self.cfg.rms_norm_eps, self.hk, self.hv, self.dk, self.dv,
                                     conv_out=cache.conv if inplace else None, state_out=cache.ssm if inplace else None,
                                     keep_mid=keep_prev)
            out, cache.conv, cache.ssm = r[:3]
            if keep_prev:
                cache.conv_prev, cache.ssm_prev = r[3], r[4]
            cache.offset += S
            return out
        y = self.recur(proj, cache, keep_prev, inplace)
        z = proj.view(B * S, -1)[:, self.conv_dim:self.conv_dim + self.value_dim]
        return glue.gated_rms_norm(y, z, self.norm_w, self.cfg.rms_norm_eps).view(B, S, self.value_dim)

    def recur(self, proj: torch.Tensor, cache: RecurrentCache, keep_prev: bool = False,
              inplace: bool = False) -> torch.Tensor:
        """From the in_proj output [B, S, *] to the recurrence output y [B, S, Hv, Dv]."""
        B, S, _ = proj.shape
        x = proj
        if cache.conv is None:
            self.init_state(cache, B, x.device)
        r = glue.deltanet_conv(proj, self.conv_w, cache.conv, self.hk, self.hv, self.dk, self.dv, keep_mid=keep_prev,
                               state_out=cache.conv if inplace else None)
        q, k, v, a, b, cache.conv = r[:6]
        if keep_prev:
            cache.conv_prev = r[6]
        g = gated_delta(q, k, v, a, b, self.A_log, self.dt_bias, cache.ssm, keep_mid=keep_prev,
                        out_state=cache.ssm if inplace else None)
        y, cache.ssm = g[0], g[1]
        if keep_prev:
            cache.ssm_prev = g[2]
        cache.offset += S
        return y

    def __call__(self, x: torch.Tensor, cache: RecurrentCache, keep_prev: bool = False) -> torch.Tensor:
        return self.out_proj(self.mix(x, cache, keep_prev))


class MLP:
    """SwiGLU MLP (engine/model.py:294-302).  gate_proj and up_proj run as one projection
    (the reference fuses them too, :296) with their rows interleaved in pairs (g_0, u_0, g_1,
    u_1, ...): a decode batch (<= 8 rows) gets silu(g) * u straight from the projection's
    epilogue (qvx_qmv_fused, swiglu_pairs), a prefill chunk from qvx_swiglu_pairs after the
    matmul -- the same bits as [gate | up] followed by qvx_swiglu, one launch fewer per
    decode layer."""

    def __init__(self, p: dict):
        g, u = _qlin(p["gate_proj"]), _qlin(p["up_proj"])
        self.gate_up = QLinear.interleave(g, u)
        self.down = _qlin(p["down_proj"])
        self.hidden = g.w.shape[0]

    def act(self, x: torch.Tensor) -> torch.Tensor:
        """silu(x @ gate^T) * (x @ up^T): x [..., H] -> [..., I]."""
        x2 = x.reshape(-1, x.shape[-1])
        gu = self.gate_up
        if x2.shape[0] < QMM_MIN_M_PREPARED and gu.in_features % 512 == 0 and gu.in_features <= 12288 \
                and gu.group_size == 64 and gu.bits == 4:
            y = qmv_fused(x2, gu.w, gu.scales, gu.biases, epilogue="swiglu_pairs", group_size=gu.group_size,
                          bits=gu.bits)
        else:
            y = glue.swiglu_pairs(gu(x2))
        return y.view(*x.shape[:-1], -1)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.down(self.act(x))


class Layer:
    """One decoder layer (engine/model.py:305-316): pre-norm mixer and MLP with residuals."""

    def __init__(self, cfg: Config, i: int, p: dict):
        self.linear = cfg.is_linear(i)
        self.mixer = GatedDeltaNet(cfg, p["linear_attn"]) if self.linear else Attention(cfg, p["self_attn"])
        self.mlp = MLP(p["mlp"])
        self.ln1, self.ln2 = p["input_layernorm"], p["post_attention_layernorm"]
        self.eps = cfg.rms_norm_eps
        self.tp = None        # qvex.tp.TP when the layer is one rank's shard
        self.tp_desc = None   # (mixer output, MLP down) reduce descriptors for fused decode

    def _row_parallel(self, lin: QLinear, xin: torch.Tensor, desc) -> torch.Tensor:
        """A projection whose input columns may be sharded over ranks (out_proj, o_proj,
        down_proj): one GPU computes it whole; sharded, each rank's partial sums are added
        over the ranks -- inside the projection kernel for decode (qvx_qmv_fused with the
        reduce exchange, B <= 8 rows), else by an NCCL all-reduce."""
        if self.tp is None:
            return lin(xin)
        rows = xin.numel() // xin.shape[-1]
        if desc is not None and rows <= 8:
            y = qmv_fused(xin.reshape(rows, -1), lin.w, lin.scales, lin.biases, gather=desc,
                          group_size=lin.group_size, bits=lin.bits)
            return y.view(*xin.shape[:-1], -1)
        return self.tp.all_reduce(lin(xin))

    def _mixer(self, n, cache, keep_prev, pos=None):
        desc = self.tp_desc[0] if self.tp_desc is not None else None
        if self.linear:
            return self._row_parallel(self.mixer.out_proj, self.mixer.mix(n, cache, keep_prev, inplace=pos is not None),
                                      desc)
        return self._row_parallel(self.mixer.o_proj, self.mixer.mix(n, cache, pos), desc)

    def _mlp(self, n2):
        desc = self.tp_desc[1] if self.tp_desc is not None else None
        return self._row_parallel(self.mlp.down, self.mlp.act(n2), desc)

    def forward_deferred(self, x: torch.Tensor, pending: torch.Tensor | None, cache, keep_prev: bool = False,
                         pos=None):
        """The layer on the residual stream x + pending (pending None: x alone), with this
        layer's MLP output returned unadded: (h, mlp_out) such that the layer's output is
        h + mlp_out.  The add then rides in the next rms_norm (one kernel less per layer).
        ``pos`` (device int32) selects the graph-replayable form: states updated in place,
        attention positions read on the device."""
        if pending is None:
            n = glue.rms_norm(x, self.ln1, self.eps)
        else:
            n, x = glue.rms_norm(pending, self.ln1, self.eps, resid=x)
        m = self._mixer(n, cache, keep_prev, pos)   # summed over the ranks when sharded
        n2, h = glue.rms_norm(m, self.ln2, self.eps, resid=x)
        return h, self._mlp(n2)

    def __call__(self, x: torch.Tensor, cache, keep_prev: bool = False) -> torch.Tensor:
        h, mo = self.forward_deferred(x, None, cache, keep_prev)
        return glue.add(h, mo)

    def forward_fused(self, x: torch.Tensor, cache, pos: torch.Tensor) -> None:
        """Decode form with the glue fused into the projections (B <= 8 tokens, one per
        sequence): the residual stream x [B, 1, H] is updated in place, every norm, SwiGLU and
        residual add riding in the projections' prologues and epilogues (qvx_qmv_fused), the
        DeltaNet conv, recurrence and gated norm in one kernel.  Gives the same bits as
        forward_deferred with two launches fewer per layer; measured on B200 (batch 1, 4096
        context, same box) the two forms take the same time (1.81 against 1.80 ms per
        token)."""
        B = x.shape[0]
        x2 = x.view(B, -1)
        mx = self.mixer
        # sharded: the row-parallel projections sum their partials across the ranks in-kernel
        red_mix, red_down = self.tp_desc if self.tp_desc is not None else (None, None)
        if self.linear:
            proj = _fused(mx.in_proj, x2, "rms_norm", norm_w=self.ln1, eps=self.eps)
            # conv, recurrence and gated norm (one kernel where the shape allows)
            y = mx.mix_proj(proj.view(B, 1, -1), cache, inplace=True)
            _fused(mx.out_proj, y.view(B, -1), "plain", resid=x2, out=x2, gather=red_mix)
        else:
            qkv = _fused(mx.qkv, x2, "rms_norm", norm_w=self.ln1, eps=self.eps)
            o = mx.attend(qkv.view(B, 1, -1), cache, pos)
            _fused(mx.o_proj, o.view(B, -1), "plain", resid=x2, out=x2, gather=red_mix)
        act = _fused(self.mlp.gate_up, x2, "rms_norm", norm_w=self.ln2, eps=self.eps, epilogue="swiglu_pairs")
        _fused(self.mlp.down, act, "plain", resid=x2, out=x2, gather=red_down)

    def fusable(self, B: int) -> bool:
        """Whether forward_fused applies: B <= 8 and every projection's K a multiple of 512."""
        lins = [self.mlp.gate_up, self.mlp.down] + (
            [self.mixer.in_proj, self.mixer.out_proj] if self.linear else [self.mixer.qkv, self.mixer.o_proj])
        return B <= 8 and all(l.in_features % 512 == 0 and l.group_size == 64 and l.bits == 4 for l in lins)


class Qwen35:
    """The whole model (engine/model.py:319-336)."""

    def __init__(self, cfg: Config, embed: QEmbedding, layers: list[Layer], norm: torch.Tensor, lm_head: QLinear):
        self.cfg = cfg
        self.embed, self.layers, self.norm, self.lm_head = embed, layers, norm, lm_head
        self.tp = None       # qvex.tp.TP when this is one rank's shard (qvex.tp.attach)
        self.lm_desc = None  # gather descriptor of lm_head for fused decode (sharded)

    def _logits(self, n: torch.Tensor) -> torch.Tensor:
        y = self.lm_head(n)
        if self.tp is not None:
            y = self.tp.all_gather_cols(y)  # vocabulary rows of every rank, in rank order
        return y

    def make_cache(self, capacity: int | None = None):
        return [RecurrentCache() if l.linear else KVCache(capacity) for l in self.layers]

    def hidden(self, ids: torch.Tensor, cache, keep_prev: bool = False, pos=None):
        """(h, pending): the pre-norm hidden state is h + pending (the last MLP output not yet
        added)."""
        x = self.embed(ids)
        pending = None
        for layer, c in zip(self.layers, cache):
            x, pending = layer.forward_deferred(x, pending, c, keep_prev, pos)
        return x, pending

    def prepare_decode(self, cache, B: int, device) -> None:
        """Allocates every state buffer a graph-replayed decode step updates in place: zero
        recurrent states where none exist yet; KV caches at their fixed capacity."""
        for layer, c in zip(self.layers, cache):
            if layer.linear:
                if c.conv is None:
                    layer.mixer.init_state(c, B, device)
            else:
                if c.capacity is None:
                    raise ValueError("graph decode needs KV caches of fixed capacity (make_cache(capacity))")
                c.reserve(B, layer.mixer.n_kv, layer.mixer.head_dim, 0, device)

    def fusable(self, B: int) -> bool:
        """Whether the fused decode form applies to B sequences (B <= 8, every projection's K a
        multiple of 512 with 4-bit g64 weights)."""
        return all(l.fusable(B) for l in self.layers) and self.lm_head.in_features % 512 == 0

    def decode_step(self, ids: torch.Tensor, cache, pos: torch.Tensor, fused: bool | None = None) -> torch.Tensor:
        """One decode step of B sequences, ids [B, 1] int32 at the device position ``pos``
        (int32 [1]): every state updated in its own buffer and nothing read on the host, so the
        step can be captured once and replayed for every token.  Returns logits [B, 1, V].
        The fused form (the default where ``fusable`` and B < QMM_MIN_M_PREPARED) carries the
        norms and residual adds in the projection kernels' prologues and epilogues: 5 launches
        per layer instead of 7, the same bits; ``fused=False`` runs the separate glue kernels.
        From QMM_MIN_M_PREPARED sequences on, the default is the separate-glue form, whose
        projections then run on the tensor-core kernel (faster there than the decode kernel
        that the fused form is built on)."""
        B = ids.shape[0]
        if fused is None:
            fused = B < QMM_MIN_M_PREPARED and self.fusable(B)
        if fused and not self.fusable(B):
            raise ValueError("the fused decode form needs B <= 8 and projections with K % 512 == 0")
        if not fused:
            x, pending = self.hidden(ids, cache, pos=pos)
            n = glue.rms_norm(pending, self.norm, self.cfg.rms_norm_eps, resid=x)[0]
            if self.lm_desc is not None and B <= 8:  # sharded: vocabulary rows gathered in-kernel
                _fused(self.lm_head, n.view(B, -1), "plain", gather=self.lm_desc)
                return self.tp.peer.output(self.lm_desc.slot, B, self.lm_desc.n_total).view(B, 1, -1)
            return self._logits(n)
        x = self.embed(ids)  # [B, 1, H], the residual stream, updated in place below
        for layer, c in zip(self.layers, cache):
            layer.forward_fused(x, c, pos)
        if self.lm_desc is not None:  # sharded: vocabulary rows gathered inside the kernel
            _fused(self.lm_head, x.view(B, -1), "rms_norm", norm_w=self.norm, eps=self.cfg.rms_norm_eps,
                   gather=self.lm_desc)
            return self.tp.peer.output(self.lm_desc.slot, B, self.lm_desc.n_total).view(B, 1, -1)
        return _fused(self.lm_head, x.view(B, -1), "rms_norm", norm_w=self.norm,
                      eps=self.cfg.rms_norm_eps).view(B, 1, -1)

    def __call__(self, ids: torch.Tensor, cache, last_only: bool = True, return_hidden: bool = False,
                 keep_prev: bool = False):
        """ids: [B, L] int32 -> logits [B, L or 1, vocab] (and the pre-norm hidden [B, L, H])."""
        x, pending = self.hidden(ids, cache, keep_prev)
        if last_only and not return_hidden:
            n = glue.rms_norm(pending[:, -1:].contiguous(), self.norm, self.cfg.rms_norm_eps,
                              resid=x[:, -1:].contiguous())[0]
            return self._logits(n)
        n, h = glue.rms_norm(pending, self.norm, self.cfg.rms_norm_eps, resid=x)
        if last_only:
            n = n[:, -1:].contiguous()
        logits = self._logits(n)
        return (logits, h) if return_hidden else logits

    # ------------------------------------------------------------ random initialisation

    @classmethod
    def random(cls, cfg: Config, seed: int = 0, device=None) -> "Qwen35":
        """A random-initialised model of shape ``cfg`` (synthetic 4-bit weights)."""
        device = torch.device(device or "cuda")
        return cls.from_params(cfg, random_params(cfg, seed, device))

    @classmethod
    def from_params(cls, cfg: Config, P: dict) -> "Qwen35":
        """From a flat dict of reference-named parameters (checkpoint keys after the
        'language_model.' prefix is stripped): quantized modules as (w, scales, biases)."""
        def ql(prefix):
            return QLinear(P[f"{prefix}.weight"], P[f"{prefix}.scales"], P[f"{prefix}.biases"], *cfg.qparams(prefix))
        layers = []
        for i in range(cfg.num_hidden_layers):
            pre = f"model.layers.{i}"
            p = {"input_layernorm": P[f"{pre}.input_layernorm.weight"],
                 "post_attention_layernorm": P[f"{pre}.post_attention_layernorm.weight"],
                 "mlp": {n: ql(f"{pre}.mlp.{n}") for n in ("gate_proj", "up_proj", "down_proj")}}
            if cfg.is_linear(i):
                la = f"{pre}.linear_attn"
                p["linear_attn"] = {**{n: ql(f"{la}.{n}") for n in
                                       ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj")},
                                    "conv1d": P[f"{la}.conv1d.weight"], "A_log": P[f"{la}.A_log"],
                                    "dt_bias": P[f"{la}.dt_bias"], "norm": P[f"{la}.norm.weight"]}
            else:
                sa = f"{pre}.self_attn"
                p["self_attn"] = {**{n: ql(f"{sa}.{n}") for n in ("q_proj", "k_proj", "v_proj", "o_proj")},
                                  "q_norm": P[f"{sa}.q_norm.weight"], "k_norm": P[f"{sa}.k_norm.weight"]}
            layers.append(Layer(cfg, i, p))
        e = "model.embed_tokens"
        embed = QEmbedding(P[f"{e}.weight"], P[f"{e}.scales"], P[f"{e}.biases"], *cfg.qparams(e))
        return cls(cfg, embed, layers, P["model.norm.weight"], ql("lm_head"))


def quantized_shapes(cfg: Config) -> dict[str, tuple[int, int]]:
    """(N, K) of every quantized module, by its reference parameter name."""
    h, I = cfg.hidden_size, cfg.intermediate_size
    kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
    vd = cfg.linear_num_value_heads * cfg.linear_value_head_dim
    out = {"model.embed_tokens": (cfg.vocab_size, h), "lm_head": (cfg.vocab_size, h)}
    for i in range(cfg.num_hidden_layers):
        pre = f"model.layers.{i}"
        out.update({f"{pre}.mlp.gate_proj": (I, h), f"{pre}.mlp.up_proj": (I, h), f"{pre}.mlp.down_proj": (h, I)})
        if cfg.is_linear(i):
            la = f"{pre}.linear_attn"
            out.update({f"{la}.in_proj_qkv": (2 * kd + vd, h), f"{la}.in_proj_z": (vd, h),
                        f"{la}.in_proj_b": (cfg.linear_num_value_heads, h),
                        f"{la}.in_proj_a": (cfg.linear_num_value_heads, h), f"{la}.out_proj": (h, vd)})
        else:
            sa = f"{pre}.self_attn"
            H, Hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
            out.update({f"{sa}.q_proj": (2 * H * D, h), f"{sa}.k_proj": (Hkv * D, h), f"{sa}.v_proj": (Hkv * D, h),
                        f"{sa}.o_proj": (h, H * D)})
    return out


def random_params(cfg: Config, seed: int, device) -> dict:
    """Reference-named random parameters: quantized modules with codes uniform in 0..15,
    scales |N(0,1)|*0.002 and biases -8*scale (bf16); norm weights 1 + N(0,1)*0.05; conv
    weights N(0,1)*0.3; A_log N(0,1)*0.5; dt_bias N(0,1)*0.5."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    P = {}
    for name, (N, K) in quantized_shapes(cfg).items():
        gs, bits = cfg.qparams(name)
        w = torch.randint(-2 ** 31, 2 ** 31, (N, K * bits // 32), dtype=torch.int64, device=device, generator=g)
        s = (torch.randn((N, K // gs), device=device, generator=g).abs() * 0.002).to(torch.bfloat16)
        P[f"{name}.weight"] = w.to(torch.int32)
        P[f"{name}.scales"] = s
        P[f"{name}.biases"] = (-8.0 * s.float()).to(torch.bfloat16)

    def norm(n):
        return (1.0 + 0.05 * torch.randn(n, device=device, generator=g)).to(torch.bfloat16)
    h = cfg.hidden_size
    kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
    vd = cfg.linear_num_value_heads * cfg.linear_value_head_dim
    for i in range(cfg.num_hidden_layers):
        pre = f"model.layers.{i}"
        P[f"{pre}.input_layernorm.weight"] = norm(h)
        P[f"{pre}.post_attention_layernorm.weight"] = norm(h)
        if cfg.is_linear(i):
            la = f"{pre}.linear_attn"
            C = 2 * kd + vd
            P[f"{la}.conv1d.weight"] = (0.3 * torch.randn((C, cfg.linear_conv_kernel_dim, 1), device=device,
                                                          generator=g)).to(torch.bfloat16)
            P[f"{la}.A_log"] = 0.5 * torch.randn(cfg.linear_num_value_heads, device=device, generator=g)
            P[f"{la}.dt_bias"] = (0.5 * torch.randn(cfg.linear_num_value_heads, device=device,
                                                    generator=g)).to(torch.bfloat16)
            P[f"{la}.norm.weight"] = norm(cfg.linear_value_head_dim)
        else:
            sa = f"{pre}.self_attn"
            P[f"{sa}.q_norm.weight"] = norm(cfg.head_dim)
            P[f"{sa}.k_norm.weight"] = norm(cfg.head_dim)
    P["model.norm.weight"] = norm(h)
    return P


class DecodeGraph:
    """Greedy decode of B sequences with one CUDA graph per step (the decode loop of
    engine/speculative.py:103-118 without host round trips): embed the current tokens, run
    every layer at the device position, final norm, lm_head, argmax; the picked tokens are
    the next step's input and the position advances on the device.  ``run(n)`` replays the
    graph n times and returns the n x B tokens.  The caches must come from
    ``model.make_cache(capacity)``; states before the graph are kept (warm-up is undone)."""

    def __init__(self, model: Qwen35, cache, first_ids: torch.Tensor, pos: int, fused: bool | None = None):
        from .sampler import sample_pick, sample_scores
        self.model, self.cache = model, cache
        dev = first_ids.device
        B = first_ids.shape[0]
        self.B = B
        model.prepare_decode(cache, B, dev)
        self.ids = first_ids.reshape(B, 1).to(torch.int32).clone()
        self.pos = torch.tensor([pos], dtype=torch.int32, device=dev)
        self.start = pos
        self.steps = 0
        self.hist = None

        def step():
            logits = model.decode_step(self.ids, cache, self.pos, fused=fused)
            scores = sample_scores(logits.view(B, -1), temperature=0.0)
            sample_pick(scores, True, out=self.ids)
            self.pos.add_(1)
            return logits

        # warm-up outside the graph (module loads, launch attributes, workspaces), then undo
        # its state changes so the graph starts from the caller's state
        saved = [(c.conv.clone(), c.ssm.clone()) if isinstance(c, RecurrentCache) else None for c in cache]
        offsets = [c.offset for c in cache]
        ids0 = self.ids.clone()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream(dev).wait_stream(s)
        for c, sv in zip(cache, saved):
            if sv is not None:
                c.conv.copy_(sv[0])
                c.ssm.copy_(sv[1])
        self.ids.copy_(ids0)
        self.pos.fill_(pos)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = step()
        for c, o in zip(cache, offsets):  # warm-up and capture ran the Python side twice
            c.offset = o

    def replay(self) -> None:
        """One decode step on the current stream (no host synchronisation)."""
        self.graph.replay()
        self.steps += 1
        for c in self.cache:
            c.offset += 1

    def run(self, n: int) -> torch.Tensor:
        """n steps; returns the tokens picked at each step, int32 [n, B] (one sync at the end)."""
        out = torch.empty((n, self.B), dtype=torch.int32, device=self.ids.device)
        for i in range(n):
            self.replay()
            out[i].copy_(self.ids.view(-1))
        return out
