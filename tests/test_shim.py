"""CPU tests of the host-side mirror of MLX's API: argument checking raises
the errors MLX raises, broadcast planning for gather_qmm, and the module
protocol (to_quantized / nn.quantize class_predicate)."""
import pytest
import torch

import mlx_server_runtime_b200 as mxq
from mlx_server_runtime_b200 import core, nn


def test_cpu_tensors_are_rejected():
    w = torch.zeros(8, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        mxq.quantize(w)
    wq = torch.zeros(8, 8, dtype=torch.uint32)
    s = torch.zeros(8, 1, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        mxq.quantized_matmul(torch.zeros(1, 64, dtype=torch.bfloat16), wq, s, s)
    with pytest.raises(ValueError, match="CUDA"):
        mxq.dequantize(wq, s, s)


def test_mode_and_transpose_checks():
    w = torch.zeros(8, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="mode"):
        mxq.quantize(w, mode="mxfp4")
    x = torch.zeros(1, 64, dtype=torch.bfloat16)
    wq = torch.zeros(8, 8, dtype=torch.uint32)
    s = torch.zeros(8, 1, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="transpose"):
        mxq.quantized_matmul(x, wq, s, s, transpose=False)


@pytest.mark.parametrize("bx,bshape,expect", [
    ((5, 1), (5, 8), 8),          # SwitchGLU unsorted: x [T,1,1,K] vs indices [T,k]
    ((40,), (40,), 1),            # sorted: x rows already gathered
    ((), (5, 8), 40),             # one x for every entry
    ((1, 8), (5, 8), None),       # needs an explicit index tensor
    ((5, 1, 1), (5, 2, 3), 6),
    ((5, 2, 1), (5, 2, 3), 3),
])
def test_broadcast_divisor(bx, bshape, expect):
    assert core.broadcast_divisor(bx, bshape) == expect


class _Leaf(nn.Module):
    def __init__(self, tag):
        self.tag = tag

    def to_quantized(self, group_size=64, bits=4, mode="affine"):
        return ("q", self.tag, group_size, bits, mode)


class _Block(nn.Module):
    def __init__(self):
        self.q_proj = _Leaf("q")
        self.mlp = [_Leaf("m0"), _Leaf("m1")]
        self.norm = object()


def test_nn_quantize_predicate_and_overrides():
    root = _Block()
    seen = []

    def pred(path, m):
        seen.append(path)
        if path == "mlp.1":
            return {"group_size": 32, "bits": 8}
        return path != "mlp.0"

    nn.quantize(root, group_size=64, bits=4, class_predicate=pred)
    assert sorted(seen) == ["mlp.0", "mlp.1", "q_proj"]
    assert root.q_proj == ("q", "q", 64, 4, "affine")
    assert isinstance(root.mlp[0], _Leaf)
    assert root.mlp[1] == ("q", "m1", 32, 8, "affine")


def test_gather_sort_roundtrip_cpu():
    idx = torch.tensor([[3, 1], [0, 3], [2, 1]])
    x = torch.arange(3, dtype=torch.float32).reshape(3, 1, 1, 1).expand(3, 1, 1, 4)
    xs, sel, inv = nn._gather_sort(x, idx)
    assert sel.tolist() == sorted(idx.reshape(-1).tolist())
    # each sorted row carries its token's x row
    order = torch.argsort(idx.reshape(-1), stable=True)
    assert xs[:, 0, 0].tolist() == (order // 2).float().tolist()
    back = nn._scatter_unsort(sel.reshape(-1, 1, 1).float(), inv, idx.shape)
    assert back.reshape(3, 2).tolist() == idx.float().tolist()
