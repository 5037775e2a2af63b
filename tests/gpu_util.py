"""Helpers for the -m gpu parity tests: move numpy bit patterns to and from
device tensors (torch is only used for device memory here)."""
import numpy as np
import torch


def dev_u16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).cuda()


def dev_f32(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def host_u16(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint16)


def host_f32(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


def empty_u16(n, fill=0x7E00) -> torch.Tensor:
    """Device buffer pre-filled with a NaN pattern so unwritten elements show up."""
    t = torch.empty(n, dtype=torch.int16, device="cuda")
    t.fill_(np.int16(np.uint16(fill).view(np.int16)))
    return t


def f16_of(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)
