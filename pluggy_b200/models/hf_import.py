"""Hugging Face checkpoint import for the decoder families.

Parity: reference ``pluggy/models/hf_import.py:35-175``: a self-contained
safetensors reader and writer, the HF -> framework parameter-name map, shard
resolution for a local directory or a Hub id (``model.safetensors`` or
``model.safetensors.index.json``), and :func:`load_hf_weights`, which fails loudly
on unmapped or missing keys and on shape mismatches and copies (bf16) weights into
the model's fp32 parameters.

The safetensors layout (format as published by Hugging Face): an 8-byte
little-endian header length, a JSON header mapping each tensor name to
``{"dtype", "shape", "data_offsets": [begin, end]}`` (offsets relative to the end
of the header), optional ``"__metadata__"``, then the raw little-endian bytes.
"""

from __future__ import annotations

import json
import os
import re
import struct

import torch
import torch.nn as nn

_DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8,
    "U8": torch.uint8, "BOOL": torch.bool,
}
_NAMES = {v: k for k, v in _DTYPES.items()}


# ------------------------------------------------------------------ safetensors
def read_safetensors(path: str) -> dict[str, torch.Tensor]:
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
        data = bytearray(f.read())
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = _DTYPES.get(meta["dtype"])
        if dt is None:
            raise ValueError(f"{path}: tensor {name} has unsupported dtype {meta['dtype']}")
        b, e = meta["data_offsets"]
        buf = data[b:e]
        t = torch.frombuffer(buf, dtype=dt) if len(buf) else torch.empty(0, dtype=dt)
        out[name] = t.reshape(meta["shape"]).clone()
    return out


def write_safetensors(tensors: dict[str, torch.Tensor], path: str,
                      metadata: dict[str, str] | None = None) -> None:
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blobs, off = [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)  # keep the data 8-byte aligned
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


# ------------------------------------------------------------------- name map
_LAYER = re.compile(r"^model\.layers\.(\d+)\.(.+)$")
_LAYER_MAP = {
    "self_attn.q_proj.weight": "{att}.q_proj.weight",
    "self_attn.k_proj.weight": "{att}.k_proj.weight",
    "self_attn.v_proj.weight": "{att}.v_proj.weight",
    "self_attn.o_proj.weight": "{att}.o_proj.weight",
    "self_attn.q_norm.weight": "{att}.q_norm.weight",
    "self_attn.k_norm.weight": "{att}.k_norm.weight",
    "mlp.gate_proj.weight": "ffn.gate_proj.weight",
    "mlp.up_proj.weight": "ffn.up_proj.weight",
    "mlp.down_proj.weight": "ffn.down_proj.weight",
    "input_layernorm.weight": "norm1.weight",
    "post_attention_layernorm.weight": "norm2.weight",
}


def _attn_name(model: nn.Module) -> str:
    blk = model.blocks[0]
    return getattr(type(blk), "attn_name", "gqa")


def hf_to_local(name: str, attn: str = "gqa") -> str | None:
    """Framework parameter name of an HF Qwen3/Llama tensor name (None if unmapped)."""
    if name == "model.embed_tokens.weight":
        return "token_emb.weight"
    if name == "model.norm.weight":
        return "norm.weight"
    if name == "lm_head.weight":
        return "lm_head.weight"
    m = _LAYER.match(name)
    if not m:
        return None
    tail = _LAYER_MAP.get(m.group(2))
    return None if tail is None else f"blocks.{m.group(1)}." + tail.format(att=attn)


def local_to_hf(name: str, attn: str = "gqa") -> str | None:
    """Inverse of :func:`hf_to_local` (used to export and by the tests)."""
    if name == "token_emb.weight":
        return "model.embed_tokens.weight"
    if name in ("norm.weight", "lm_head.weight"):
        return "model.norm.weight" if name == "norm.weight" else name
    m = re.match(r"^blocks\.(\d+)\.(.+)$", name)
    if not m:
        return None
    for hf_tail, tail in _LAYER_MAP.items():
        if tail.format(att=attn) == m.group(2):
            return f"model.layers.{m.group(1)}.{hf_tail}"
    return None


# ---------------------------------------------------------------- resolution
def weight_files(src: str) -> list[str]:
    """Shard files of a local directory (or file), or of a Hub id resolved through
    ``huggingface_hub`` (downloads need network access)."""
    if os.path.isfile(src):
        return [src]
    if not os.path.isdir(src):
        try:
            from huggingface_hub import snapshot_download
        except ImportError as e:  # pragma: no cover - depends on the environment
            raise FileNotFoundError(f"{src!r} is not a local path and huggingface_hub is missing") from e
        src = snapshot_download(src, allow_patterns=["*.safetensors", "*.json"])
    index = os.path.join(src, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            wm = json.load(f)["weight_map"]
        return [os.path.join(src, fn) for fn in sorted(set(wm.values()))]
    single = os.path.join(src, "model.safetensors")
    if os.path.exists(single):
        return [single]
    files = sorted(fn for fn in os.listdir(src) if fn.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors weights under {src}")
    return [os.path.join(src, fn) for fn in files]


@torch.no_grad()
def load_hf_weights(model: nn.Module, src: str) -> int:
    """Copy every HF tensor of ``src`` into ``model``; returns the number copied.

    Raises on an HF tensor with no mapping, on a model parameter that receives
    nothing (a tied ``lm_head`` may be absent from the checkpoint), and on any
    shape mismatch, before modifying the model.
    """
    attn = _attn_name(model)
    params = dict(model.named_parameters(remove_duplicate=False))
    tied = {n for n, p in params.items() if n == "lm_head.weight" and p is params.get("token_emb.weight")}
    staged: dict[str, torch.Tensor] = {}
    unmapped: list[str] = []
    for path in weight_files(src):
        for name, t in read_safetensors(path).items():
            local = hf_to_local(name, attn)
            if local is None or local not in params:
                unmapped.append(name)
                continue
            if tuple(t.shape) != tuple(params[local].shape):
                raise ValueError(f"shape mismatch for {name} -> {local}: checkpoint {tuple(t.shape)}, "
                                 f"model {tuple(params[local].shape)}")
            staged[local] = t
    if unmapped:
        raise KeyError(f"{len(unmapped)} checkpoint tensors have no mapping, e.g. {unmapped[:5]}")
    missing = [n for n in params if n not in staged and n not in tied]
    if missing:
        raise KeyError(f"{len(missing)} model parameters missing from the checkpoint, e.g. {missing[:5]}")
    for n, t in staged.items():
        params[n].copy_(t.to(params[n].dtype))
    if hasattr(model, "weight_cache"):
        model.weight_cache.clear()
    return len(staged)


__all__ = ["read_safetensors", "write_safetensors", "hf_to_local", "local_to_hf", "weight_files",
           "load_hf_weights"]
