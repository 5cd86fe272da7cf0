"""numpy <-> torch conversions for the parity tests (bf16 travels as uint16 bits)."""
import numpy as np
import torch

from oracle import oracle_np as O

TORCH_DT = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def to_dev(a: np.ndarray, dtype: str | None = None, device="cuda") -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).view(torch.uint32).to(device)
    if dtype == "bfloat16":
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)
    if a.dtype == np.int32:
        return torch.from_numpy(a).to(device)
    return torch.from_numpy(a).to(device)


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.uint32:
        return t.view(torch.int32).numpy().view(np.uint32)
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def as_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    return O.to_f32(a, dtype)


def rand_weights(rng, shape, dtype, std=0.02):
    return O.from_f32((rng.standard_normal(shape) * std).astype(np.float32), dtype)


def rand_x(rng, shape, dtype):
    return O.from_f32(rng.standard_normal(shape).astype(np.float32), dtype)


def close(y_gpu: np.ndarray, y_ref: np.ndarray, dtype: str, rel: float = 2e-2):
    """The path's tolerance: max|d| <= rel * max|ref| (bf16/f16 output, fp32 accumulation)."""
    a, b = as_f32(y_gpu, dtype), as_f32(y_ref, dtype)
    assert a.shape == b.shape
    assert np.isfinite(a).all()
    err = np.abs(a - b).max() if a.size else 0.0
    scale = np.abs(b).max() if b.size else 0.0
    assert err <= rel * scale + 1e-30, f"max|d|={err} > {rel}*max|ref|={rel * scale}"
    return err / max(scale, 1e-30)
