"""Checkpoint loading (MLX layout) and top-k routing on the host: tensors are
read and assigned without any kernel, so these run on CPU."""
import json
import os

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

from mlx_server_runtime_b200 import loader, nn


class Block(nn.Module):
    def __init__(self):
        self.q = nn.Linear(128, 64, bias=True, device="cpu")
        self.o = nn.Linear(64, 128, bias=False, device="cpu")
        self.experts = nn.SwitchLinear(128, 32, 4, device="cpu")


class Tiny(nn.Module):
    def __init__(self):
        self.embed = nn.Embedding(50, 128, device="cpu")
        self.layers = [Block(), Block()]
        self.lm_head = nn.Linear(128, 50, bias=False, device="cpu")


def _q(g, lead, n, k, gs, bits):
    w = torch.randint(0, 2**31 - 1, (*lead, n, k * bits // 32), generator=g, dtype=torch.int64)
    s = torch.randn(*lead, n, k // gs, generator=g).to(torch.bfloat16)
    b = torch.randn(*lead, n, k // gs, generator=g).to(torch.bfloat16)
    return w.to(torch.int32).view(torch.uint32), s, b


def _checkpoint(tmp_path, override=True):
    g = torch.Generator().manual_seed(0)
    t = {}
    for i in range(2):
        gs, bits = (32, 8) if (override and i == 1) else (64, 4)
        t[f"layers.{i}.q.weight"], t[f"layers.{i}.q.scales"], t[f"layers.{i}.q.biases"] = \
            _q(g, (), 64, 128, gs, bits)
        t[f"layers.{i}.q.bias"] = torch.randn(64, generator=g).to(torch.bfloat16)
        # layer 0's o stays dense in the checkpoint
        if i == 0:
            t["layers.0.o.weight"] = torch.randn(128, 64, generator=g).to(torch.bfloat16)
        else:
            t["layers.1.o.weight"], t["layers.1.o.scales"], t["layers.1.o.biases"] = \
                _q(g, (), 128, 64, 64, 4)
        (t[f"layers.{i}.experts.weight"], t[f"layers.{i}.experts.scales"],
         t[f"layers.{i}.experts.biases"]) = _q(g, (4,), 32, 128, 64, 4)
    t["embed.weight"], t["embed.scales"], t["embed.biases"] = _q(g, (), 50, 128, 64, 4)
    t["lm_head.weight"], t["lm_head.scales"], t["lm_head.biases"] = _q(g, (), 50, 128, 64, 4)
    names = sorted(t)
    shards = {"model-00001-of-00002.safetensors": names[: len(names) // 2],
              "model-00002-of-00002.safetensors": names[len(names) // 2:]}
    wmap = {}
    for f, ns in shards.items():
        save_file({n: t[n].contiguous() for n in ns}, str(tmp_path / f))
        wmap.update({n: f for n in ns})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wmap}))
    quant = {"group_size": 64, "bits": 4}
    if override:
        quant["layers.1.q"] = {"group_size": 32, "bits": 8}
    (tmp_path / "config.json").write_text(json.dumps({"quantization": quant}))
    return t


def test_load_checkpoint_quantizes_where_scales_exist(tmp_path):
    t = _checkpoint(tmp_path)
    m = Tiny()
    loader.load_checkpoint(m, str(tmp_path))
    assert isinstance(m.layers[0].q, nn.QuantizedLinear)
    assert isinstance(m.layers[0].o, nn.Linear)          # no scales in the checkpoint
    assert isinstance(m.layers[1].o, nn.QuantizedLinear)
    assert isinstance(m.layers[0].experts, nn.QuantizedSwitchLinear)
    assert isinstance(m.embed, nn.QuantizedEmbedding)
    assert (m.layers[0].q.group_size, m.layers[0].q.bits) == (64, 4)
    assert (m.layers[1].q.group_size, m.layers[1].q.bits) == (32, 8)   # per-layer override
    for name, ref in t.items():
        mp, _, attr = name.rpartition(".")
        mod = dict(m.named_modules())[mp]
        got = getattr(mod, attr)
        assert got.dtype == ref.dtype and got.shape == ref.shape
        view = torch.int32 if ref.dtype == torch.uint32 else torch.int16
        assert torch.equal(got.view(view), ref.view(view)), name


def test_load_errors(tmp_path):
    _checkpoint(tmp_path)
    os.remove(tmp_path / "model-00002-of-00002.safetensors")
    with pytest.raises(loader.WeightArtifactError, match="shard file"):
        loader.load_checkpoint(Tiny(), str(tmp_path))


def test_assign_rejects_mismatch_and_strays(tmp_path):
    t = _checkpoint(tmp_path, override=False)
    m = Tiny()
    loader.quantize_like_checkpoint(m, t.keys(), {"group_size": 64, "bits": 4})
    bad = dict(t)
    bad["layers.0.q.scales"] = bad["layers.0.q.scales"][:, :1].contiguous()
    with pytest.raises(loader.WeightArtifactError, match="layers.0.q.scales"):
        loader.assign_weights(m, bad)
    stray = dict(t)
    stray["layers.0.nothing.weight"] = torch.zeros(2)
    with pytest.raises(loader.WeightArtifactError, match="no place"):
        loader.assign_weights(m, stray)
    missing = {k: v for k, v in t.items() if k != "lm_head.biases"}
    with pytest.raises(loader.WeightArtifactError, match="lm_head.biases"):
        loader.assign_weights(m, missing)


def test_route_topk_runs_on_the_device_only():
    """The router is a device kernel (core.moe_route; its parity test is
    tests/test_gpu_router.py): host tensors are refused, as every operator here does."""
    with pytest.raises(ValueError, match="CUDA"):
        nn.route_topk(torch.zeros(4, 16), 2)
