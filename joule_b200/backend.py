"""KernelBackend over the CUDA library — same interface as the reference's
src/jouleai/native/backend.py:45-69, so engine code written against
``KernelBackend.auto().q4_gemv/q4_gemm`` runs unchanged.

Arguments keep the reference's meaning: ``packed``/``scales`` are one Q4
record's arrays (numpy host arrays, as Q4ExpertPool.gather(raw=True) returns
them, or CUDA tensors), ``x``/``X`` fp32. Host inputs are copied to the GPU and
the result comes back on the host, as the reference returns a CPU tensor;
CUDA inputs stay on the device.
"""
from __future__ import annotations

from abc import ABC, abstractmethod

import numpy as np
import torch

from joule_b200.native import check, get_dll


class KernelBackend(ABC):
    """Interface every native kernel backend implements (backend.py:45-69)."""

    name: str = "base"

    @abstractmethod
    def q4_gemv(self, x_f32: torch.Tensor, packed, scales, m: int, d: int,
                group: int = 64) -> torch.Tensor:
        """out[m] = dequant_q4(packed, scales) @ x[d]."""

    @abstractmethod
    def q4_gemm(self, out_f32: torch.Tensor, X_f32: torch.Tensor, packed, scales,
                m: int, d: int, group: int = 64) -> None:
        """out[T, m] (in place) = X[T, d] @ dequant(W)^T."""

    @staticmethod
    def auto() -> "KernelBackend":
        """The CUDA backend; there is no CPU fallback."""
        return CudaBackend()


def _dev_u8(a, dev) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(dev).view(torch.uint8).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8)).to(dev)


def _dev_u16(a, dev) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(dev).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)


class CudaBackend(KernelBackend):
    """sm_100a kernels of libjoule_moe.so (jl_q4_gemv_f32 / jl_q4_gemm_f32)."""

    name = "cuda_sm100a"

    def __init__(self, device: int | None = None):
        if not torch.cuda.is_available():
            raise RuntimeError("CudaBackend needs a CUDA device")
        self._dll = get_dll()
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)

    def q4_gemv(self, x_f32, packed, scales, m, d, group=64):
        assert x_f32.dtype == torch.float32 and x_f32.numel() == d
        host = not x_f32.is_cuda
        x = x_f32.to(self.device).contiguous().view(-1)
        pk, sc = _dev_u8(packed, self.device), _dev_u16(scales, self.device)
        assert pk.numel() == m * d // 2
        out = torch.empty(m, dtype=torch.float32, device=self.device)
        check(self._dll.jl_q4_gemv_f32(out.data_ptr(), x.data_ptr(), pk.data_ptr(), sc.data_ptr(),
                                       m, d, group, torch.cuda.current_stream().cuda_stream),
              "jl_q4_gemv_f32")
        return out.cpu() if host else out

    def q4_gemm(self, out_f32, X_f32, packed, scales, m, d, group=64):
        T = X_f32.shape[0]
        X = X_f32.to(self.device).contiguous()
        pk, sc = _dev_u8(packed, self.device), _dev_u16(scales, self.device)
        o = out_f32 if out_f32.is_cuda else torch.empty(T, m, dtype=torch.float32,
                                                        device=self.device)
        assert o.is_contiguous()
        check(self._dll.jl_q4_gemm_f32(o.data_ptr(), X.data_ptr(), T, pk.data_ptr(), sc.data_ptr(),
                                       m, d, group, torch.cuda.current_stream().cuda_stream),
              "jl_q4_gemm_f32")
        if not out_f32.is_cuda:
            out_f32.copy_(o.view_as(out_f32).cpu())
