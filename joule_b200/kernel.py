"""Module-level Q4 GEMV/GEMM, the same two functions as the reference's
src/jouleai/native/kernel.py:24-62 (``q4_gemv`` returns a new tensor,
``q4_gemm`` writes ``out_f32`` in place), backed by the CUDA library."""
from __future__ import annotations

import torch

from joule_b200.backend import CudaBackend

_BACKEND: CudaBackend | None = None


def _backend() -> CudaBackend:
    global _BACKEND
    if _BACKEND is None:
        _BACKEND = CudaBackend()
    return _BACKEND


def q4_gemv(x_f32: torch.Tensor, packed, scales, m: int, d: int, group: int = 64) -> torch.Tensor:
    """out[m] fp32 = dequant_q4(packed, scales) @ x (no dequant materialisation)."""
    return _backend().q4_gemv(x_f32, packed, scales, m, d, group)


def q4_gemm(out_f32: torch.Tensor, X_f32: torch.Tensor, packed, scales, m: int, d: int,
            group: int = 64) -> None:
    """out_f32 [T, m] (in place) = X_f32 [T, d] @ dequant(W)^T."""
    _backend().q4_gemm(out_f32, X_f32, packed, scales, m, d, group)
