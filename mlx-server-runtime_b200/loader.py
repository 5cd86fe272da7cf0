"""MLX-format quantized checkpoints into the B200 modules.

An MLX 4/8-bit checkpoint stores every quantized layer as three tensors next to
each other: ``<path>.weight`` (uint32 packed codes, [N, K*bits/32], or
[E, N, K*bits/32] for an expert bank), ``<path>.scales`` and ``<path>.biases``
([.., N, K/group_size], the activation dtype), plus ``<path>.bias`` for layers
with a bias. That is exactly the layout this library's operators take, so
loading is a copy: no repacking, no requantization.

The reference loads a checkpoint in two steps, which this module follows:
  * the weight index (``model.safetensors.index.json``: tensor name -> shard
    file) is validated and every referenced shard must exist
    (native_mlx/mapping.py:97-141, ``load_weight_index``); the tensors are then
    read shard by shard (mapping.py:61-94, ``load_mapped_weights``);
  * the model is quantized only where the checkpoint has ``<path>.scales``,
    with the ``quantization`` block of config.json giving group_size / bits /
    mode, overridden per layer by a dict stored under the layer's path
    (qwen2.py:309-324, lfm2.py:570-591).
Here the second step swaps each such layer for an *empty* quantized twin of
the right shapes (nothing is quantized on the way), and the tensors are then
assigned by name.
"""
from __future__ import annotations

import json
import os
from typing import Any

import torch

from . import nn

__all__ = ["WeightArtifactError", "load_weight_index", "load_weights", "quantize_like_checkpoint",
           "assign_weights", "load_checkpoint"]


class WeightArtifactError(ValueError):
    """A checkpoint's index, shards or tensors are missing or malformed."""


def load_weight_index(model_path: str) -> dict[str, str]:
    """tensor name -> shard file name, from model.safetensors.index.json (or the
    single model.safetensors when there is no index). Every shard must exist."""
    index_path = os.path.join(model_path, "model.safetensors.index.json")
    if not os.path.exists(index_path):
        single = os.path.join(model_path, "model.safetensors")
        if os.path.exists(single):
            from safetensors import safe_open
            with safe_open(single, framework="pt") as f:
                return {k: "model.safetensors" for k in f.keys()}
        raise WeightArtifactError(f"{model_path}: neither {os.path.basename(index_path)} nor model.safetensors exists")
    try:
        with open(index_path) as f:
            payload = json.load(f)
    except (OSError, json.JSONDecodeError) as e:
        raise WeightArtifactError(f"{os.path.basename(index_path)} is not readable JSON ({e})") from e
    wmap = payload.get("weight_map")
    if not isinstance(wmap, dict) or not wmap:
        raise WeightArtifactError("model.safetensors.index.json: weight_map is absent or empty")
    if not all(isinstance(k, str) and isinstance(v, str) for k, v in wmap.items()):
        raise WeightArtifactError("model.safetensors.index.json: weight_map must map tensor names to file names")
    missing = sorted({v for v in wmap.values() if not os.path.exists(os.path.join(model_path, v))})
    if missing:
        raise WeightArtifactError(f"{len(missing)} shard file(s) named by the index are not in {model_path}: " + ", ".join(missing))
    return dict(wmap)


def load_weights(model_path: str, device: str | torch.device = "cpu") -> dict[str, torch.Tensor]:
    """Every tensor of the checkpoint, read shard by shard onto `device`."""
    from safetensors.torch import load_file
    wmap = load_weight_index(model_path)
    by_file: dict[str, list[str]] = {}
    for name, fname in wmap.items():
        by_file.setdefault(fname, []).append(name)
    out: dict[str, torch.Tensor] = {}
    for fname, names in sorted(by_file.items()):
        try:
            tensors = load_file(os.path.join(model_path, fname), device=str(device))
        except Exception as e:  # a corrupt or truncated shard
            raise WeightArtifactError(f"could not load {fname}: {e}") from e
        for n in names:
            if n not in tensors:
                raise WeightArtifactError(f"missing tensor {n!r} in {fname}")
            out[n] = tensors[n]
    return out


def _layer_params(quantization: dict[str, Any], path: str) -> dict[str, Any]:
    over = quantization.get(path)
    src = over if isinstance(over, dict) else quantization
    return {"group_size": int(src["group_size"]), "bits": int(src["bits"]),
            "mode": str(src.get("mode", "affine"))}


def _empty_twin(m: nn.Module, group_size: int, bits: int, mode: str) -> nn.Module:
    """The quantized twin of a dense layer with zero tensors of the right shapes."""
    if mode != "affine":
        raise WeightArtifactError(f"quantization mode {mode!r} is not supported (affine only)")
    w = m.weight
    *lead, n, k = w.shape
    if k % group_size or (k * bits) % 32:
        raise WeightArtifactError(f"K={k} does not fit group_size={group_size}, bits={bits}")
    dev, dt = w.device, w.dtype
    if isinstance(m, nn.Linear):
        q = nn.QuantizedLinear.__new__(nn.QuantizedLinear)
    elif isinstance(m, nn.Embedding):
        q = nn.QuantizedEmbedding.__new__(nn.QuantizedEmbedding)
    elif isinstance(m, nn.SwitchLinear):
        q = nn.QuantizedSwitchLinear.__new__(nn.QuantizedSwitchLinear)
    else:
        raise WeightArtifactError(f"no quantized form for {type(m).__name__}")
    q.group_size, q.bits, q.mode = group_size, bits, mode
    q.weight = torch.zeros(*lead, n, k * bits // 32, dtype=torch.uint32, device=dev)
    q.scales = torch.zeros(*lead, n, k // group_size, dtype=dt, device=dev)
    q.biases = torch.zeros(*lead, n, k // group_size, dtype=dt, device=dev)
    if hasattr(m, "bias"):
        q.bias = m.bias
    return q


def quantize_like_checkpoint(model: nn.Module, weight_names, quantization: dict[str, Any] | None
                             ) -> list[str]:
    """Swap every layer that has a quantized form and whose ``<path>.scales`` is in
    the checkpoint for an empty quantized twin (group_size / bits / mode from
    `quantization`, or from the dict stored under the layer's path). Returns the
    swapped paths. Nothing is quantized: the checkpoint's tensors are assigned
    afterwards."""
    if quantization is None:
        return []
    names = set(weight_names)
    swaps = []
    for path, m in model.named_modules():
        if not path or not hasattr(m, "to_quantized") or f"{path}.scales" not in names:
            continue
        p = _layer_params(quantization, path)
        swaps.append((path, _empty_twin(m, p["group_size"], p["bits"], p["mode"])))
    for path, q in swaps:
        parent_path, _, leaf = path.rpartition(".")
        parent = model
        if parent_path:
            for part in parent_path.split("."):
                parent = parent[int(part)] if part.isdigit() else getattr(parent, part)
        if leaf.isdigit():
            parent[int(leaf)] = q
        else:
            setattr(parent, leaf, q)
    return [p for p, _ in swaps]


def assign_weights(model: nn.Module, weights: dict[str, torch.Tensor], strict: bool = True
                   ) -> None:
    """Assign checkpoint tensors to the module attributes they name ("a.0.b.weight"
    -> model.a[0].b.weight), moved to the attribute's device. Shapes and dtypes
    must match the attribute they replace; with `strict`, every tensor must land
    somewhere and every quantized layer must receive weight, scales and biases."""
    modules = dict(model.named_modules())
    filled: set[str] = set()
    for name, t in weights.items():
        mpath, _, attr = name.rpartition(".")
        m = modules.get(mpath)
        if m is None or not hasattr(m, attr):
            if strict:
                raise WeightArtifactError(f"checkpoint tensor {name!r} has no place in the model")
            continue
        cur = getattr(m, attr)
        if not isinstance(cur, torch.Tensor):
            raise WeightArtifactError(f"{name!r} does not name a tensor")
        if tuple(cur.shape) != tuple(t.shape) or cur.dtype != t.dtype:
            raise WeightArtifactError(
                f"{name!r}: checkpoint {tuple(t.shape)} {t.dtype} vs model "
                f"{tuple(cur.shape)} {cur.dtype}")
        setattr(m, attr, t.to(cur.device).contiguous())
        filled.add(name)
    if strict:
        for path, m in modules.items():
            if isinstance(m, (nn.QuantizedLinear, nn.QuantizedSwitchLinear, nn.QuantizedEmbedding)):
                for a in ("weight", "scales", "biases"):
                    if f"{path}.{a}" not in filled:
                        raise WeightArtifactError(f"checkpoint has no {path}.{a}")


def load_checkpoint(model: nn.Module, model_path: str, strict: bool = True) -> dict[str, Any]:
    """config.json's quantization block + the weight shards into `model` (built
    dense, on the device it should run on). Returns the parsed config."""
    with open(os.path.join(model_path, "config.json")) as f:
        config = json.load(f)
    weights = load_weights(model_path, "cpu")
    quantize_like_checkpoint(model, weights.keys(), config.get("quantization"))
    assign_weights(model, weights, strict=strict)
    return config
