"""Checkpoint I/O: MLX / Hugging Face safetensors directories <-> engine weights.

The reference loads targets with mlx-lm (``load``, adapters.py:822-846) and
drafters with ``mx.load`` + ``load_weights`` (draft.py:370-382).  Here a
checkpoint directory (``config.json`` + ``model*.safetensors``) is read
straight into the engine's packed layouts:

* Qwen3 (``model_type`` "qwen3"): ``model.layers.{i}.self_attn.{q,k,v,o}_proj``,
  ``q_norm`` / ``k_norm``, ``mlp.{gate,up,down}_proj``, the two layer norms,
  ``model.embed_tokens`` (tied LM head) and ``model.norm``.  MLX 4-bit
  layers (``.weight`` uint32 [out, in/8] + ``.scales`` / ``.biases`` bf16
  [out, in/64], mlx ``quantize`` layout) load as ``Q4Tensor``; a quantized
  embedding is kept as the 4-bit tied LM head and its dequantized bf16 rows
  become the lookup table.
* Qwen3.5 (``model_type`` "qwen3_5", the text model of a "text_config"
  checkpoint): the reference's ``sanitize`` rules
  (custom_qwen35_model.py:1251-1275, 1365-1379) -- vision / ``mtp.`` tensors
  dropped, ``model.language_model.`` prefixes folded, a Hugging Face conv1d
  weight [C, 1, K] moved to MLX's [C, K, 1], and on an unsanitized
  checkpoint (one with ``mtp.`` tensors or an unmoved conv1d) the
  ``1 + weight`` RMSNorm weights (layer norms, final norm, q/k norms; not the
  gated norm) shifted by +1.
* DFlash drafter (draft.py:312-367): ``layers.{i}.…`` decoder layers,
  ``fc``, ``hidden_norm``, ``norm`` and the ``dflash_config``
  (``target_layer_ids``, ``mask_token_id``) / ``block_size`` of config.json.

Writers produce the same layouts (MLX for Qwen3 / the drafter, Hugging Face
unsanitized for Qwen3.5) so a model can be exported and read back.

The safetensors format is read here directly (an 8-byte little-endian header
length, a JSON header of dtype / shape / byte offsets, then the raw
little-endian data), memory-mapped, without the ``safetensors`` package.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Any

import numpy as np
import torch

from .config import DraftConfig, Qwen3Config, Qwen35Config
from .synthetic import Q4Tensor, Qwen3Weights, Qwen35Weights, interleave_gate_up

# ---------------------------------------------------------------- safetensors
_DT = {
    "BF16": (np.uint16, torch.bfloat16),
    "F16": (np.float16, torch.float16),
    "F32": (np.float32, torch.float32),
    "F64": (np.float64, torch.float64),
    "I64": (np.int64, torch.int64),
    "I32": (np.int32, torch.int32),
    "U32": (np.uint32, torch.int32),  # bit patterns kept in int32 (MLX packed words)
    "I16": (np.int16, torch.int16),
    "I8": (np.int8, torch.int8),
    "U8": (np.uint8, torch.uint8),
    "BOOL": (np.bool_, torch.bool),
}
_TORCH_TO_ST = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32", torch.float64: "F64",
                torch.int64: "I64", torch.int32: "I32", torch.int16: "I16", torch.int8: "I8", torch.uint8: "U8",
                torch.bool: "BOOL"}


def read_safetensors(path: str | Path, device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    """All tensors of one .safetensors file (U32 arrives as int32 bit patterns)."""
    path = Path(path)
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    base = 8 + n
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    out: dict[str, torch.Tensor] = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        np_dt, t_dt = _DT[info["dtype"]]
        b0, b1 = info["data_offsets"]
        arr = np.frombuffer(raw[base + b0: base + b1], dtype=np_dt).reshape(info["shape"])
        if info["dtype"] == "BF16":
            t = torch.from_numpy(arr.astype(np.int16, copy=True).view(np.int16)).view(torch.bfloat16)
        elif info["dtype"] == "U32":
            t = torch.from_numpy(arr.view(np.int32).copy())
        else:
            t = torch.from_numpy(arr.copy())
        out[name] = t.to(device)
    return out


def write_safetensors(path: str | Path, tensors: dict[str, torch.Tensor], metadata: dict[str, str] | None = None,
                      u32: set[str] = frozenset()) -> None:
    """Write tensors (names in ``u32`` are int32 bit patterns stored as U32)."""
    header: dict[str, Any] = {}
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        dt = "U32" if name in u32 else _TORCH_TO_ST[t.dtype]
        b = (t.view(torch.int16) if t.dtype == torch.bfloat16 else t).numpy().tobytes()
        header[name] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_checkpoint_dir(path: str | Path, device: str | torch.device = "cpu") -> tuple[dict, dict[str, torch.Tensor]]:
    """config.json and every ``model*.safetensors`` of a checkpoint directory."""
    path = Path(path)
    cfg_file = path / "config.json"
    if not cfg_file.exists():
        raise FileNotFoundError(f"{path} has no config.json")
    config = json.loads(cfg_file.read_text())
    files = sorted(path.glob("model*.safetensors"))
    if not files:
        raise FileNotFoundError(f"No model*.safetensors weights found in {path}")
    tensors: dict[str, torch.Tensor] = {}
    for f in files:
        tensors.update(read_safetensors(f, device))
    return config, tensors


# ---------------------------------------------------------------- helpers
def dequantize_q4(q: Q4Tensor) -> torch.Tensor:
    """bf16 of an MLX affine 4-bit matrix: scale * q + bias per group of 64."""
    words = q.packed.to(torch.int64) & 0xFFFFFFFF
    n = words.shape[0]
    shifts = torch.arange(8, device=words.device) * 4
    qv = ((words[..., None] >> shifts) & 0xF).reshape(n, -1).float()
    s = q.scales.float().repeat_interleave(q.group_size, dim=1)
    b = q.biases.float().repeat_interleave(q.group_size, dim=1)
    return (s * qv + b).to(torch.bfloat16)


def _linear(t: dict[str, torch.Tensor], prefix: str, device, group_size: int = 64):
    """A linear layer ``prefix`` as bf16 [out, in] or a Q4Tensor (4-bit MLX)."""
    w = t[prefix + ".weight"]
    if prefix + ".scales" in t:
        q = Q4Tensor(w.to(torch.int32).contiguous().to(device), t[prefix + ".scales"].to(torch.bfloat16).to(device),
                     t[prefix + ".biases"].to(torch.bfloat16).to(device), group_size)
        if q.shape[1] != q.scales.shape[1] * group_size:
            raise ValueError(f"{prefix}: only 4-bit weights with group size {group_size} are supported")
        return q
    return w.to(torch.bfloat16).contiguous().to(device)


def _cat_rows(parts):
    if isinstance(parts[0], Q4Tensor):
        return Q4Tensor(*(torch.cat([getattr(p, f) for p in parts]).contiguous()
                          for f in ("packed", "scales", "biases")), parts[0].group_size)
    return torch.cat(parts).contiguous()


def _interleave(gate, up):
    if isinstance(gate, Q4Tensor):
        return Q4Tensor(*(interleave_gate_up(getattr(gate, f), getattr(up, f)).contiguous()
                          for f in ("packed", "scales", "biases")), gate.group_size)
    return interleave_gate_up(gate, up)


def _bf16(t, device):
    return t.to(torch.bfloat16).contiguous().to(device)


# ---------------------------------------------------------------- Qwen3
def qwen3_config_from_dict(c: dict) -> Qwen3Config:
    return Qwen3Config(hidden_size=c["hidden_size"], num_hidden_layers=c["num_hidden_layers"],
                       num_attention_heads=c["num_attention_heads"], num_key_value_heads=c["num_key_value_heads"],
                       head_dim=c.get("head_dim", c["hidden_size"] // c["num_attention_heads"]),
                       intermediate_size=c["intermediate_size"], vocab_size=c["vocab_size"],
                       rope_theta=float(c.get("rope_theta", (c.get("rope_parameters") or {}).get("rope_theta", 1e6))),
                       rms_norm_eps=float(c.get("rms_norm_eps", 1e-6)),
                       tie_word_embeddings=bool(c.get("tie_word_embeddings", True)))


def qwen3_weights_from_tensors(config: dict, t: dict[str, torch.Tensor], device="cuda") -> Qwen3Weights:
    """Engine layout of a Qwen3 checkpoint (bf16 or MLX 4-bit projections)."""
    cfg = qwen3_config_from_dict(config)
    q = config.get("quantization") or {}
    gs = int(q.get("group_size", 64))
    if q and int(q.get("bits", 4)) != 4:
        raise ValueError("only 4-bit MLX quantization is supported")
    emb = _linear(t, "model.embed_tokens", device, gs)
    emb_q = None
    if isinstance(emb, Q4Tensor):
        emb_q, emb = emb, dequantize_q4(emb)
    if not cfg.tie_word_embeddings and "lm_head.weight" in t:
        raise NotImplementedError("untied LM heads are not supported by the verify engine (the tied head is "
                                  "the embedding)")
    w = Qwen3Weights(cfg, embed=_bf16(emb, device), final_norm=_bf16(t["model.norm.weight"], device), embed_q4=emb_q)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        lin = lambda n: _linear(t, p + n, device, gs)  # noqa: E731
        w.input_norm.append(_bf16(t[p + "input_layernorm.weight"], device))
        w.qkv.append(_cat_rows([lin("self_attn.q_proj"), lin("self_attn.k_proj"), lin("self_attn.v_proj")]))
        w.q_norm.append(_bf16(t[p + "self_attn.q_norm.weight"], device))
        w.k_norm.append(_bf16(t[p + "self_attn.k_norm.weight"], device))
        w.o_proj.append(lin("self_attn.o_proj"))
        w.post_norm.append(_bf16(t[p + "post_attention_layernorm.weight"], device))
        w.gate_up.append(_interleave(lin("mlp.gate_proj"), lin("mlp.up_proj")))
        w.down.append(lin("mlp.down_proj"))
    return w


def _put_linear(out: dict, name: str, v, u32: set):
    if isinstance(v, Q4Tensor):
        out[name + ".weight"] = v.packed
        out[name + ".scales"] = v.scales
        out[name + ".biases"] = v.biases
        u32.add(name + ".weight")
    else:
        out[name + ".weight"] = v


def save_qwen3_mlx(w: Qwen3Weights, path: str | Path) -> None:
    """Write a Qwen3 target as an MLX checkpoint directory (mlx-lm names)."""
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    c = w.cfg
    out: dict[str, torch.Tensor] = {"model.embed_tokens.weight": w.embed, "model.norm.weight": w.final_norm}
    u32: set[str] = set()
    if w.embed_q4 is not None:
        _put_linear(out, "model.embed_tokens", w.embed_q4, u32)
    for i in range(c.num_hidden_layers):
        r = w.reference_weights(i)
        p = f"model.layers.{i}."
        for n in ("input_layernorm", "post_attention_layernorm"):
            out[p + n + ".weight"] = r[n]
        for n in ("q_norm", "k_norm"):
            out[p + "self_attn." + n + ".weight"] = r[n]
        for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
            _put_linear(out, p + "self_attn." + n, r[n], u32)
        for n in ("gate_proj", "up_proj", "down_proj"):
            _put_linear(out, p + "mlp." + n, r[n], u32)
    write_safetensors(path / "model.safetensors", out, metadata={"format": "mlx"}, u32=u32)
    cfg = {"model_type": "qwen3", "hidden_size": c.hidden_size, "num_hidden_layers": c.num_hidden_layers,
           "num_attention_heads": c.num_attention_heads, "num_key_value_heads": c.num_key_value_heads,
           "head_dim": c.head_dim, "intermediate_size": c.intermediate_size, "vocab_size": c.vocab_size,
           "rope_theta": c.rope_theta, "rms_norm_eps": c.rms_norm_eps, "tie_word_embeddings": True}
    if w.quant_bits == 4:
        cfg["quantization"] = {"group_size": 64, "bits": 4}
    (path / "config.json").write_text(json.dumps(cfg, indent=2) + "\n")


# ---------------------------------------------------------------- Qwen3.5
_NORM_SUFFIXES = (".input_layernorm.weight", ".post_attention_layernorm.weight", "model.norm.weight",
                  ".q_norm.weight", ".k_norm.weight")


def sanitize_qwen35(weights: dict[str, torch.Tensor], tie_word_embeddings: bool = True) -> dict[str, torch.Tensor]:
    """The reference's Qwen3.5 ``sanitize`` rules on a text-model state dict
    (custom_qwen35_model.py:1251-1275, prefixes :1365-1379).  Keys come out
    as ``model.layers.{i}.…``, ``model.embed_tokens.weight``,
    ``model.norm.weight``; conv1d weights as MLX [C, K, 1]."""
    folded: dict[str, torch.Tensor] = {}
    for k, v in weights.items():
        if k.startswith(("vision_tower", "model.visual")):
            continue
        for pre in ("model.language_model.", "language_model.model.", "language_model."):
            if k.startswith(pre):
                k = "model." + k[len(pre):] if pre != "language_model." else k[len(pre):]
                break
        folded[k] = v
    has_mtp = any("mtp." in k for k in folded)
    has_raw_conv = any("conv1d.weight" in k and v.shape[-1] != 1 for k, v in folded.items())
    shift = has_mtp or has_raw_conv
    out = {k: v for k, v in folded.items() if "mtp." not in k}
    if tie_word_embeddings:
        out.pop("lm_head.weight", None)
    for k, v in list(out.items()):
        if "conv1d.weight" in k and v.shape[-1] != 1:
            out[k] = v.movedim(2, 1)
        if shift and any(k.endswith(sfx) for sfx in _NORM_SUFFIXES) and v.ndim == 1:
            out[k] = (v.float() + 1.0).to(v.dtype)
    return out


def qwen35_config_from_dict(config: dict) -> Qwen35Config:
    c = config.get("text_config", config)
    rp = c.get("rope_parameters") or {}
    types = c.get("layer_types")
    interval = int(c.get("full_attention_interval", 4))
    if types:
        full = [i for i, t in enumerate(types) if t == "full_attention"]
        if full and all((i + 1) % (full[0] + 1) == 0 for i in full) and len(full) == len(types) // (full[0] + 1):
            interval = full[0] + 1
        else:
            raise NotImplementedError("only a repeating k-linear : 1-full-attention layer pattern is supported")
    return Qwen35Config(hidden_size=c["hidden_size"], num_hidden_layers=c["num_hidden_layers"],
                        intermediate_size=c["intermediate_size"], vocab_size=c["vocab_size"],
                        num_attention_heads=c["num_attention_heads"], num_key_value_heads=c["num_key_value_heads"],
                        head_dim=c.get("head_dim", 256), linear_num_key_heads=c["linear_num_key_heads"],
                        linear_num_value_heads=c["linear_num_value_heads"],
                        linear_key_head_dim=c["linear_key_head_dim"],
                        linear_value_head_dim=c["linear_value_head_dim"],
                        linear_conv_kernel_dim=c.get("linear_conv_kernel_dim", 4), full_attention_interval=interval,
                        rope_theta=float(rp.get("rope_theta", c.get("rope_theta", 1e5))),
                        partial_rotary_factor=float(rp.get("partial_rotary_factor",
                                                           c.get("partial_rotary_factor", 0.25))),
                        rms_norm_eps=float(c.get("rms_norm_eps", 1e-6)),
                        tie_word_embeddings=bool(c.get("tie_word_embeddings", config.get("tie_word_embeddings",
                                                                                          True))))


def qwen35_weights_from_tensors(config: dict, raw: dict[str, torch.Tensor], device="cuda") -> Qwen35Weights:
    """Engine layout of a Qwen3.5 text checkpoint (MLX or Hugging Face, bf16)."""
    cfg = qwen35_config_from_dict(config)
    t = sanitize_qwen35(raw, cfg.tie_word_embeddings)
    if any(k.endswith(".scales") for k in t):
        raise NotImplementedError("4-bit weights are implemented for the Qwen3 target only")
    w = Qwen35Weights(cfg, embed=_bf16(t["model.embed_tokens.weight"], device),
                      final_norm=_bf16(t["model.norm.weight"], device))
    a_log, dt_bias = [], []
    for l in range(cfg.num_hidden_layers):
        p = f"model.layers.{l}."
        L = {"input_norm": _bf16(t[p + "input_layernorm.weight"], device),
             "post_norm": _bf16(t[p + "post_attention_layernorm.weight"], device),
             "gate_up": interleave_gate_up(_bf16(t[p + "mlp.gate_proj.weight"], device),
                                           _bf16(t[p + "mlp.up_proj.weight"], device)),
             "down": _bf16(t[p + "mlp.down_proj.weight"], device)}
        if cfg.is_linear(l):
            a = p + "linear_attn."
            L["in_proj"] = torch.cat([_bf16(t[a + n + ".weight"], device)
                                      for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")]).contiguous()
            conv = t[a + "conv1d.weight"]  # MLX [C, K, 1]
            L["conv_weight"] = _bf16(conv[..., 0].t(), device)  # engine [K, C]
            L["norm"] = _bf16(t[a + "norm.weight"], device)
            L["out_proj"] = _bf16(t[a + "out_proj.weight"], device)
            a_log.append(t[a + "A_log"].float().to(device))
            dt_bias.append(_bf16(t[a + "dt_bias"], device))
        else:
            a = p + "self_attn."
            L["qkv"] = torch.cat([_bf16(t[a + n + ".weight"], device) for n in ("q_proj", "k_proj", "v_proj")]
                                 ).contiguous()
            L["q_norm"] = _bf16(t[a + "q_norm.weight"], device)
            L["k_norm"] = _bf16(t[a + "k_norm.weight"], device)
            L["o_proj"] = _bf16(t[a + "o_proj.weight"], device)
        w.layers.append(L)
    w.a_log = torch.stack(a_log).float().contiguous()
    w.dt_bias = torch.stack(dt_bias).contiguous()
    return w


def save_qwen35_hf(w: Qwen35Weights, path: str | Path) -> None:
    """Write a Qwen3.5 target as a Hugging Face checkpoint (unsanitized: conv1d
    [C, 1, K], ``1 + weight`` norms stored as weight - 1, language-model
    prefixes): the layout ``sanitize_qwen35`` converts back."""
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    c = w.cfg
    shift = lambda v: (v.float() - 1.0).to(torch.bfloat16)  # noqa: E731
    pre = "model.language_model."
    out = {pre + "embed_tokens.weight": w.embed, pre + "norm.weight": shift(w.final_norm)}
    for l in range(c.num_hidden_layers):
        r = w.reference_layer(l)
        p = f"{pre}layers.{l}."
        out[p + "input_layernorm.weight"] = shift(r["input_layernorm"])
        out[p + "post_attention_layernorm.weight"] = shift(r["post_attention_layernorm"])
        for n in ("gate_proj", "up_proj", "down_proj"):
            out[p + "mlp." + n + ".weight"] = r[n]
        if c.is_linear(l):
            a = p + "linear_attn."
            for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
                out[a + n + ".weight"] = r[n]
            out[a + "conv1d.weight"] = r["conv_weight"].t().unsqueeze(1)  # [C, 1, K]
            out[a + "norm.weight"] = r["norm"]
            out[a + "A_log"] = r["A_log"].float()
            out[a + "dt_bias"] = r["dt_bias"]
        else:
            a = p + "self_attn."
            for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
                out[a + n + ".weight"] = r[n]
            out[a + "q_norm.weight"] = shift(r["q_norm"])
            out[a + "k_norm.weight"] = shift(r["k_norm"])
    write_safetensors(path / "model.safetensors", {k: v.contiguous() for k, v in out.items()})
    types = ["linear_attention" if c.is_linear(l) else "full_attention" for l in range(c.num_hidden_layers)]
    text = {"model_type": "qwen3_5_text", "hidden_size": c.hidden_size, "num_hidden_layers": c.num_hidden_layers,
            "intermediate_size": c.intermediate_size, "vocab_size": c.vocab_size,
            "num_attention_heads": c.num_attention_heads, "num_key_value_heads": c.num_key_value_heads,
            "head_dim": c.head_dim, "linear_num_key_heads": c.linear_num_key_heads,
            "linear_num_value_heads": c.linear_num_value_heads, "linear_key_head_dim": c.linear_key_head_dim,
            "linear_value_head_dim": c.linear_value_head_dim, "linear_conv_kernel_dim": c.linear_conv_kernel_dim,
            "layer_types": types, "rms_norm_eps": c.rms_norm_eps,
            "rope_parameters": {"rope_type": "default", "rope_theta": c.rope_theta,
                                "partial_rotary_factor": c.partial_rotary_factor},
            "tie_word_embeddings": True}
    (path / "config.json").write_text(json.dumps({"model_type": "qwen3_5", "text_config": text,
                                                  "tie_word_embeddings": True}, indent=2) + "\n")


# ---------------------------------------------------------------- drafter
def draft_config_from_dict(c: dict) -> DraftConfig:
    dc = c.get("dflash_config") or {}
    if "target_layer_ids" not in dc or "mask_token_id" not in dc:
        raise ValueError("DFlash config.json needs dflash_config.target_layer_ids and mask_token_id")
    return DraftConfig(hidden_size=c["hidden_size"], num_hidden_layers=c["num_hidden_layers"],
                       num_attention_heads=c["num_attention_heads"], num_key_value_heads=c["num_key_value_heads"],
                       head_dim=c.get("head_dim", c["hidden_size"] // c["num_attention_heads"]),
                       intermediate_size=c["intermediate_size"], vocab_size=c["vocab_size"],
                       target_layer_ids=tuple(int(i) for i in dc["target_layer_ids"]),
                       block_size=int(c.get("block_size", 16)), mask_token_id=int(dc["mask_token_id"]),
                       rope_theta=float(c.get("rope_theta", 1e6)), rms_norm_eps=float(c.get("rms_norm_eps", 1e-6)))


def dflash_weights_from_tensors(config: dict, raw: dict[str, torch.Tensor], target_embed: torch.Tensor):
    """Engine layout of a DFlash drafter checkpoint on the target's embedding."""
    from .draft import DFlashWeights

    cfg = draft_config_from_dict(config)
    dev = target_embed.device
    t = {(k[len("model."):] if k.startswith("model.") else k): v for k, v in raw.items()}
    qcfg = Qwen3Config(hidden_size=cfg.hidden_size, num_hidden_layers=cfg.num_hidden_layers,
                       num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                       head_dim=cfg.head_dim, intermediate_size=cfg.intermediate_size, vocab_size=cfg.vocab_size,
                       rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_norm_eps)
    layers = Qwen3Weights(qcfg, embed=target_embed, final_norm=_bf16(t["norm.weight"], dev))
    for i in range(cfg.num_hidden_layers):
        p = f"layers.{i}."
        b = lambda n: _bf16(t[p + n + ".weight"], dev)  # noqa: E731
        layers.input_norm.append(b("input_layernorm"))
        layers.qkv.append(torch.cat([b("self_attn.q_proj"), b("self_attn.k_proj"), b("self_attn.v_proj")])
                          .contiguous())
        layers.q_norm.append(b("self_attn.q_norm"))
        layers.k_norm.append(b("self_attn.k_norm"))
        layers.o_proj.append(b("self_attn.o_proj"))
        layers.post_norm.append(b("post_attention_layernorm"))
        layers.gate_up.append(interleave_gate_up(b("mlp.gate_proj"), b("mlp.up_proj")))
        layers.down.append(b("mlp.down_proj"))
    return DFlashWeights(cfg, layers, _bf16(t["fc.weight"], dev), _bf16(t["hidden_norm.weight"], dev))


def save_dflash_mlx(w, path: str | Path) -> None:
    """Write a DFlash drafter (DFlashWeights) as a checkpoint directory."""
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    c = w.cfg
    out = {"fc.weight": w.fc, "hidden_norm.weight": w.hidden_norm, "norm.weight": w.layers.final_norm}
    for i in range(c.num_hidden_layers):
        r = w.layers.reference_weights(i)
        p = f"layers.{i}."
        for n in ("input_layernorm", "post_attention_layernorm"):
            out[p + n + ".weight"] = r[n]
        for n in ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"):
            out[p + "self_attn." + n + ".weight"] = r[n]
        for n in ("gate_proj", "up_proj", "down_proj"):
            out[p + "mlp." + n + ".weight"] = r[n]
    write_safetensors(path / "model.safetensors", {k: v.contiguous() for k, v in out.items()})
    cfg = {"model_type": "qwen3", "hidden_size": c.hidden_size, "num_hidden_layers": c.num_hidden_layers,
           "intermediate_size": c.intermediate_size, "num_attention_heads": c.num_attention_heads,
           "num_key_value_heads": c.num_key_value_heads, "head_dim": c.head_dim, "vocab_size": c.vocab_size,
           "rms_norm_eps": c.rms_norm_eps, "rope_theta": c.rope_theta, "max_position_embeddings": 40960,
           "tie_word_embeddings": True, "block_size": c.block_size,
           "dflash_config": {"target_layer_ids": list(c.target_layer_ids), "mask_token_id": c.mask_token_id}}
    (path / "config.json").write_text(json.dumps(cfg, indent=2) + "\n")


def load_target_weights(path: str | Path, device="cuda"):
    """(model_type, weights) of a checkpoint directory."""
    config, t = read_checkpoint_dir(path, "cpu")
    mt = config.get("model_type")
    if mt == "qwen3":
        return mt, qwen3_weights_from_tensors(config, t, device)
    if mt in ("qwen3_5", "qwen3_5_text"):
        return "qwen3_5", qwen35_weights_from_tensors(config, t, device)
    raise NotImplementedError(f"Unsupported target model_type={mt!r}")
