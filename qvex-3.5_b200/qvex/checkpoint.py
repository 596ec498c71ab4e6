"""Checkpoints of Qwen3.5 4-bit models: the MLX safetensors layout the reference's engine
loads, and the reference's native ``.q35`` single-file layout.

* ``load_model(model_dir)`` follows engine/model.py:342-397: config.json through
  Config.from_file (text_config nesting, rope parameters, quantization block with
  per-module overrides, :39-71); every ``*.safetensors`` file, keys remapped from
  ``language_model.*`` to ``*`` and from ``model.language_model.*`` to ``model.*``
  (:347-352); a checkpoint that still carries MTP weights is refused (:353-354); the vision
  tower and other unused tensors are never copied to the GPU.  The kernels here implement
  the 4-bit group-64 format only; a module quantized otherwise is refused at load time.
* ``write_q35`` / ``load_q35`` follow experiments/native/convert_native.py:5-17,57-133:
  "Q35W", version 1, 16 int32 and 2 float32 of configuration, a table of
  (name[64], dtype, ndim, shape[4], offset, nbytes) entries, 256-byte aligned tensors in a
  16 KB aligned data section; projections that share an input stored fused (DeltaNet
  in_proj_qkv|z|b|a as L{i}.in, attention q|k|v as L{i}.qkv, MLP gate|up as L{i}.gu), norm,
  conv, A_log and dt_bias tensors as float32.
* safetensors is read and written without the safetensors package: an 8-byte little-endian
  header length, a JSON header {name: {dtype, shape, data_offsets}}, then the data.
"""
from __future__ import annotations

import json
import mmap
import struct
from pathlib import Path

import numpy as np
import torch

# ---------------------------------------------------------------- safetensors

_ST_DTYPES = {"BF16": (torch.bfloat16, 2), "F16": (torch.float16, 2), "F32": (torch.float32, 4),
              "U32": (torch.int32, 4), "I32": (torch.int32, 4), "U8": (torch.uint8, 1), "I64": (torch.int64, 8)}
_ST_NAMES = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32", torch.int32: "U32",
             torch.uint8: "U8", torch.int64: "I64"}


def read_safetensors(path: Path, keep=None) -> tuple[dict[str, torch.Tensor], dict]:
    """{name: CPU tensor} and the metadata of one safetensors file; ``keep(name)`` selects
    which tensors are materialised (the others are never read from disk).  U32 tensors come
    back as int32 holding the same bits."""
    path = Path(path)
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
        meta = header.pop("__metadata__", {}) or {}
        out = {}
        if not header:
            return out, meta
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            for name, info in header.items():
                if keep is not None and not keep(name):
                    continue
                if info["dtype"] not in _ST_DTYPES:
                    raise ValueError(f"{path.name}: tensor {name} has unsupported dtype {info['dtype']}")
                dt, size = _ST_DTYPES[info["dtype"]]
                a, b = info["data_offsets"]
                count = (b - a) // size
                shape = tuple(info["shape"])
                if int(np.prod(shape)) != count:
                    raise ValueError(f"{path.name}: tensor {name} holds {count} values for shape {shape}")
                buf = bytearray(mm[base + a:base + b])  # a private copy; the map closes below
                t = torch.frombuffer(buf, dtype=dt).reshape(shape) if count else torch.empty(shape, dtype=dt)
                out[name] = t
        finally:
            mm.close()
    return out, meta


def write_safetensors(path: Path, tensors: dict[str, torch.Tensor], metadata: dict | None = None) -> None:
    """Writes CPU tensors (int32 tensors as U32, the packed-weight convention)."""
    header, blobs, at = {}, [], 0
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _ST_NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [at, at + len(raw)]}
        blobs.append(raw)
        at += len(raw)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


# ---------------------------------------------------------------- MLX checkpoint directory


def remap_key(k: str) -> str | None:
    """engine/model.py:349-352: the text model's keys without the multimodal prefixes;
    None for keys outside the language model (vision tower and the like)."""
    if k.startswith("language_model."):
        return k[len("language_model."):]
    if k.startswith("model.language_model."):
        return "model." + k[len("model.language_model."):]
    return None


def read_checkpoint(model_dir: Path) -> dict[str, torch.Tensor]:
    """Every language-model tensor of a checkpoint directory, reference-named, on the CPU."""
    model_dir = Path(model_dir)
    files = sorted(model_dir.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {model_dir}")
    weights = {}
    for f in files:
        part, _ = read_safetensors(f, keep=lambda n: remap_key(n) is not None)
        for k, v in part.items():
            weights[remap_key(k)] = v
    if any("mtp." in k for k in weights):
        raise ValueError("unsanitized checkpoint (mtp weights present): convert with mlx first")
    return weights


def _check_formats(cfg, P: dict) -> None:
    for k in P:
        if k.endswith(".scales"):
            module = k[:-len(".scales")]
            gs, bits = cfg.qparams(module)
            if (gs, bits) != (64, 4):
                raise NotImplementedError(f"{module} is quantized with group_size={gs}, bits={bits}; "
                                          "the B200 kernels implement the 4-bit group-64 format only")


def load_model(model_dir: str | Path, device="cuda"):
    """A Qwen35 model from an MLX 4-bit checkpoint directory (engine/model.py:342-397)."""
    from .qwen35 import Config, Qwen35
    model_dir = Path(model_dir)
    cfg = Config.from_file(model_dir / "config.json")
    P = read_checkpoint(model_dir)
    _check_formats(cfg, P)
    needed = set(expected_keys(cfg))
    missing = sorted(needed - set(P))
    if missing:
        raise KeyError(f"checkpoint lacks {len(missing)} tensors, e.g. {missing[:3]}")
    dev = torch.device(device)
    P = {k: (v.to(torch.float32) if k.endswith(".A_log") else v).to(dev)  # A_log in fp32: engine/model.py:374
         for k, v in P.items() if k in needed}
    return Qwen35.from_params(cfg, P)


def expected_keys(cfg) -> list[str]:
    """The reference-named tensors a Qwen3.5 text model of shape ``cfg`` consists of."""
    from .qwen35 import quantized_shapes
    keys = []
    for name in quantized_shapes(cfg):
        keys += [f"{name}.weight", f"{name}.scales", f"{name}.biases"]
    keys.append("model.norm.weight")
    for i in range(cfg.num_hidden_layers):
        pre = f"model.layers.{i}"
        keys += [f"{pre}.input_layernorm.weight", f"{pre}.post_attention_layernorm.weight"]
        if cfg.is_linear(i):
            la = f"{pre}.linear_attn"
            keys += [f"{la}.conv1d.weight", f"{la}.A_log", f"{la}.dt_bias", f"{la}.norm.weight"]
        else:
            sa = f"{pre}.self_attn"
            keys += [f"{sa}.q_norm.weight", f"{sa}.k_norm.weight"]
    return keys


def save_checkpoint(model_dir: str | Path, cfg, P: dict, shards: int = 2, prefix: str = "language_model.") -> None:
    """Writes ``P`` (reference-named) as an MLX-style checkpoint directory: config.json and
    ``shards`` safetensors files with keys under ``prefix`` (how the multimodal checkpoints
    name them).  Used to produce test fixtures of the loader."""
    model_dir = Path(model_dir)
    model_dir.mkdir(parents=True, exist_ok=True)
    text = {"hidden_size": cfg.hidden_size, "intermediate_size": cfg.intermediate_size,
            "num_hidden_layers": cfg.num_hidden_layers, "num_attention_heads": cfg.num_attention_heads,
            "num_key_value_heads": cfg.num_key_value_heads, "head_dim": cfg.head_dim,
            "linear_num_key_heads": cfg.linear_num_key_heads, "linear_num_value_heads": cfg.linear_num_value_heads,
            "linear_key_head_dim": cfg.linear_key_head_dim, "linear_value_head_dim": cfg.linear_value_head_dim,
            "linear_conv_kernel_dim": cfg.linear_conv_kernel_dim,
            "full_attention_interval": cfg.full_attention_interval, "rms_norm_eps": cfg.rms_norm_eps,
            "vocab_size": cfg.vocab_size,
            "rope_parameters": {"rope_theta": cfg.rope_theta, "partial_rotary_factor": cfg.rotary_dim / cfg.head_dim}}
    quant = {"group_size": cfg.group_size, "bits": cfg.bits,
             **{f"language_model.{k}": v for k, v in cfg.quant.items()}}
    (model_dir / "config.json").write_text(json.dumps({"text_config": text, "quantization": quant}, indent=1))
    names = sorted(P)
    for s in range(shards):
        part = {prefix + k: P[k] for k in names[s::shards]}
        write_safetensors(model_dir / f"model-{s + 1:05d}-of-{shards:05d}.safetensors", part)


# ---------------------------------------------------------------- .q35


Q35_MAGIC = b"Q35W"
Q35_VERSION = 1
Q35_PAGE = 16384
Q35_ALIGN = 256
Q35_F32, Q35_BF16, Q35_U32 = 0, 1, 2
_Q35_ENTRY = struct.Struct("<64sII4QQQ")


def _q35_config(cfg) -> tuple[list[int], list[float]]:
    ints = [cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers, cfg.num_attention_heads,
            cfg.num_key_value_heads, cfg.head_dim, cfg.linear_num_key_heads, cfg.linear_num_value_heads,
            cfg.linear_key_head_dim, cfg.linear_value_head_dim, cfg.linear_conv_kernel_dim,
            cfg.full_attention_interval, cfg.vocab_size, cfg.rotary_dim, cfg.group_size, cfg.bits]
    return ints, [float(cfg.rms_norm_eps), float(cfg.rope_theta)]


def q35_tensors(cfg, P: dict) -> list[tuple[str, torch.Tensor, int]]:
    """(name, tensor, dtype code) in the .q35 order, projections sharing an input fused."""
    out = []

    def add(name, t, as_f32=False):
        t = t.detach().cpu()
        if as_f32 or t.dtype == torch.float32:
            out.append((name, t.to(torch.float32).contiguous(), Q35_F32))
        elif t.dtype == torch.bfloat16:
            out.append((name, t.contiguous(), Q35_BF16))
        else:
            out.append((name, t.to(torch.int32).contiguous(), Q35_U32))

    def add_q(name, prefixes):
        for suffix, short in (("weight", "w"), ("scales", "s"), ("biases", "b")):
            add(f"{name}.{short}", torch.cat([P[f"{p}.{suffix}"] for p in prefixes]))

    add_q("embed", ["model.embed_tokens"])
    add_q("lm_head", ["lm_head"])
    add("norm", P["model.norm.weight"], True)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}"
        add(f"L{i}.ln1", P[f"{p}.input_layernorm.weight"], True)
        add(f"L{i}.ln2", P[f"{p}.post_attention_layernorm.weight"], True)
        add_q(f"L{i}.gu", [f"{p}.mlp.gate_proj", f"{p}.mlp.up_proj"])
        add_q(f"L{i}.down", [f"{p}.mlp.down_proj"])
        if cfg.is_linear(i):
            la = f"{p}.linear_attn"
            add_q(f"L{i}.in", [f"{la}.in_proj_qkv", f"{la}.in_proj_z", f"{la}.in_proj_b", f"{la}.in_proj_a"])
            add_q(f"L{i}.out", [f"{la}.out_proj"])
            add(f"L{i}.conv", P[f"{la}.conv1d.weight"].reshape(-1, cfg.linear_conv_kernel_dim), True)
            add(f"L{i}.A_log", P[f"{la}.A_log"], True)
            add(f"L{i}.dt_bias", P[f"{la}.dt_bias"], True)
            add(f"L{i}.gnorm", P[f"{la}.norm.weight"], True)
        else:
            sa = f"{p}.self_attn"
            add_q(f"L{i}.qkv", [f"{sa}.q_proj", f"{sa}.k_proj", f"{sa}.v_proj"])
            add_q(f"L{i}.o", [f"{sa}.o_proj"])
            add(f"L{i}.qnorm", P[f"{sa}.q_norm.weight"], True)
            add(f"L{i}.knorm", P[f"{sa}.k_norm.weight"], True)
    return out


def write_q35(path: str | Path, cfg, P: dict) -> int:
    """Writes a .q35 file; returns its size in bytes."""
    if (cfg.group_size, cfg.bits) != (64, 4) or cfg.quant:
        raise NotImplementedError(".q35 holds 4-bit group-64 weights only")
    tensors = q35_tensors(cfg, P)
    ints, floats = _q35_config(cfg)
    header = Q35_MAGIC + struct.pack("<I", Q35_VERSION) + struct.pack("<16i", *ints) + struct.pack("<2f", *floats)
    header += struct.pack("<I", len(tensors))
    data_start = (len(header) + _Q35_ENTRY.size * len(tensors) + Q35_PAGE - 1) // Q35_PAGE * Q35_PAGE
    offset, table, placed = data_start, b"", []
    for name, t, dt in tensors:
        if len(name) >= 64:
            raise ValueError(f"tensor name {name} too long for .q35")
        offset = (offset + Q35_ALIGN - 1) // Q35_ALIGN * Q35_ALIGN
        raw = t.view(torch.uint8).numpy().tobytes()
        shape = list(t.shape) + [0] * (4 - t.dim())
        table += _Q35_ENTRY.pack(name.encode(), dt, t.dim(), *shape, offset, len(raw))
        placed.append((offset, raw))
        offset += len(raw)
    total = (offset + Q35_PAGE - 1) // Q35_PAGE * Q35_PAGE
    with open(path, "wb") as f:
        f.write(header + table)
        for off, raw in placed:
            f.seek(off)
            f.write(raw)
        f.truncate(total)
    return total


def read_q35(path: str | Path):
    """(Config, {name: CPU tensor}) of a .q35 file (names as stored: embed.w, L3.qkv.s, ...)."""
    from .qwen35 import Config
    with open(path, "rb") as f:
        buf = f.read()
    if buf[:4] != Q35_MAGIC:
        raise ValueError(f"{path} is not a .q35 file")
    (version,) = struct.unpack_from("<I", buf, 4)
    if version != Q35_VERSION:
        raise ValueError(f"{path}: .q35 version {version}, {Q35_VERSION} supported")
    ints = struct.unpack_from("<16i", buf, 8)
    floats = struct.unpack_from("<2f", buf, 72)
    (n,) = struct.unpack_from("<I", buf, 80)
    H, I, layers, heads, kvh, hd, lkh, lvh, lkd, lvd, ck, fai, vocab, rd, gs, bits = ints
    cfg = Config(hidden_size=H, intermediate_size=I, num_hidden_layers=layers, num_attention_heads=heads,
                 num_key_value_heads=kvh, head_dim=hd, linear_num_key_heads=lkh, linear_num_value_heads=lvh,
                 linear_key_head_dim=lkd, linear_value_head_dim=lvd, linear_conv_kernel_dim=ck,
                 full_attention_interval=fai, rms_norm_eps=floats[0], vocab_size=vocab, rope_theta=floats[1],
                 rotary_dim=rd, group_size=gs, bits=bits)
    out = {}
    dtypes = {Q35_F32: (torch.float32, 4), Q35_BF16: (torch.bfloat16, 2), Q35_U32: (torch.int32, 4)}
    for j in range(n):
        name, dt, ndim, s0, s1, s2, s3, off, nbytes = _Q35_ENTRY.unpack_from(buf, 84 + j * _Q35_ENTRY.size)
        name = name.rstrip(b"\0").decode()
        tdt, size = dtypes[dt]
        shape = (s0, s1, s2, s3)[:ndim]
        raw = bytearray(buf[off:off + nbytes])
        out[name] = torch.frombuffer(raw, dtype=tdt).reshape(shape) if nbytes else torch.empty(shape, dtype=tdt)
    return cfg, out


def q35_params(cfg, T: dict) -> dict:
    """Reference-named parameters from .q35 tensors: fused projections split back into their
    parts, float32 norm weights back to bf16 (exact: the converter widened them from bf16)."""
    P = {}

    def q(short, parts):
        w, s, b = T[f"{short}.w"], T[f"{short}.s"], T[f"{short}.b"]
        at = 0
        for part, rows in parts:
            for suffix, t in (("weight", w), ("scales", s), ("biases", b)):
                P[f"{part}.{suffix}"] = t[at:at + rows].contiguous()
            at += rows
        if at != w.shape[0]:
            raise ValueError(f"{short}: {w.shape[0]} rows, parts add up to {at}")

    def bf(t):
        return t.to(torch.bfloat16).contiguous()
    from .qwen35 import quantized_shapes
    shapes = quantized_shapes(cfg)
    q("embed", [("model.embed_tokens", cfg.vocab_size)])
    q("lm_head", [("lm_head", cfg.vocab_size)])
    P["model.norm.weight"] = bf(T["norm"])
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}"
        P[f"{p}.input_layernorm.weight"] = bf(T[f"L{i}.ln1"])
        P[f"{p}.post_attention_layernorm.weight"] = bf(T[f"L{i}.ln2"])
        m = f"{p}.mlp"
        q(f"L{i}.gu", [(f"{m}.gate_proj", cfg.intermediate_size), (f"{m}.up_proj", cfg.intermediate_size)])
        q(f"L{i}.down", [(f"{m}.down_proj", cfg.hidden_size)])
        if cfg.is_linear(i):
            la = f"{p}.linear_attn"
            q(f"L{i}.in", [(f"{la}.{n}", shapes[f"{la}.{n}"][0]) for n in
                               ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")])
            q(f"L{i}.out", [(f"{la}.out_proj", cfg.hidden_size)])
            P[f"{la}.conv1d.weight"] = bf(T[f"L{i}.conv"]).unsqueeze(-1)
            P[f"{la}.A_log"] = T[f"L{i}.A_log"].to(torch.float32)
            P[f"{la}.dt_bias"] = bf(T[f"L{i}.dt_bias"])
            P[f"{la}.norm.weight"] = bf(T[f"L{i}.gnorm"])
        else:
            sa = f"{p}.self_attn"
            q(f"L{i}.qkv", [(f"{sa}.{n}", shapes[f"{sa}.{n}"][0]) for n in ("q_proj", "k_proj", "v_proj")])
            q(f"L{i}.o", [(f"{sa}.o_proj", cfg.hidden_size)])
            P[f"{sa}.q_norm.weight"] = bf(T[f"L{i}.qnorm"])
            P[f"{sa}.k_norm.weight"] = bf(T[f"L{i}.knorm"])
    return P


def load_q35(path: str | Path, device="cuda"):
    """A Qwen35 model from a .q35 file."""
    from .qwen35 import Qwen35
    cfg, T = read_q35(path)
    P = {k: v.to(torch.device(device)) for k, v in q35_params(cfg, T).items()}
    return Qwen35.from_params(cfg, P)


def convert(model_dir: str | Path, out: str | Path) -> int:
    """MLX checkpoint directory -> .q35 (experiments/native/convert_native.py)."""
    from .qwen35 import Config
    cfg = Config.from_file(Path(model_dir) / "config.json")
    P = read_checkpoint(model_dir)
    _check_formats(cfg, P)
    return write_q35(out, cfg, P)


if __name__ == "__main__":
    import sys
    if len(sys.argv) != 4 or sys.argv[1] != "convert":
        raise SystemExit("usage: python -m qvex.checkpoint convert MODEL_DIR OUT.q35")
    print(f"wrote {sys.argv[3]}: {convert(sys.argv[2], sys.argv[3]) / 1e9:.2f} GB")
