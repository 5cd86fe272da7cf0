"""A checkpoint written in MLX's layout from a model this library quantized
loads back bit for bit and computes the same outputs; the MoE block (router +
SwitchGLU over gather_qmm) matches a per-token, per-expert evaluation."""
import json

import pytest
import torch
from safetensors.torch import save_file

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import loader, nn

from gpu_util import close, to_np

pytestmark = pytest.mark.gpu


class Net(nn.Module):
    def __init__(self, seed):
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.embed = nn.Embedding(300, 256, generator=g)
        self.q = nn.Linear(256, 512, bias=True, generator=g)
        self.experts = nn.SwitchLinear(256, 128, 8, generator=g)
        self.lm_head = nn.Linear(256, 300, bias=False, generator=g)


def test_checkpoint_round_trip(tmp_path):
    src = Net(1)
    nn.quantize(src, 64, 4)
    tensors = {}
    for path, m in src.named_modules():
        for a in ("weight", "scales", "biases", "bias"):
            if path and isinstance(getattr(m, a, None), torch.Tensor):
                tensors[f"{path}.{a}"] = getattr(m, a).detach().cpu().contiguous()
    save_file(tensors, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps({"quantization": {"group_size": 64,
                                                                        "bits": 4}}))
    dst = Net(2)
    loader.load_checkpoint(dst, str(tmp_path))
    x = torch.randn(5, 256, device="cuda").to(torch.bfloat16)
    ids = torch.tensor([[3, 7, 299]], device="cuda")
    idx = torch.tensor([[0, 5], [7, 2], [1, 1], [4, 6], [3, 0]], device="cuda", dtype=torch.int32)
    assert torch.equal(dst.q(x), src.q(x))
    assert torch.equal(dst.lm_head(x), src.lm_head(x))
    assert torch.equal(dst.embed(ids), src.embed(ids))
    xe = x.unsqueeze(-2).unsqueeze(-3)
    assert torch.equal(dst.experts(xe, idx), src.experts(xe, idx))


@pytest.mark.parametrize("T", [1, 5, 96])
def test_moe_block_matches_per_expert_loop(T):
    g = torch.Generator(device="cuda").manual_seed(T)
    blk = nn.MoEBlock(256, 128, 16, 4, generator=g)
    with torch.no_grad():
        blk.gate.weight.mul_(8.0)  # spread the router so the top-k are well separated
    nn.quantize(blk, 64, 4, class_predicate=lambda p, m: p.startswith("switch_mlp"))
    x = torch.randn(T, 256, device="cuda", generator=g).to(torch.bfloat16)
    y = blk(x)
    idx, sc = nn.route_topk(blk.gate(x), 4, True)
    sw = blk.switch_mlp
    ref = torch.zeros(T, 256, device="cuda", dtype=torch.float32)
    for t in range(T):
        for j in range(4):
            e = int(idx[t, j])
            def qmm(layer, v):
                return mxq.quantized_matmul(v, layer.weight[e], layer.scales[e], layer.biases[e],
                                            group_size=64, bits=4)
            h = nn.silu(qmm(sw.gate_proj, x[t:t + 1])) * qmm(sw.up_proj, x[t:t + 1])
            ref[t] += (qmm(sw.down_proj, h)[0] * sc[t, j]).float()
    close(to_np(y.float()), to_np(ref), "float32")
