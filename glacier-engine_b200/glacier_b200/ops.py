"""Reference-named operator wrappers over device tensors.

Each function mirrors one operator of the reference's compute seam and calls the
matching ``glacier_cuda_*`` entry point on torch CUDA tensors (torch is used only
for device memory and streams).  Shapes are validated by the library; errors
raise ``GlacierCudaError``.
"""
from __future__ import annotations

import torch

from ._lib import call


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def linear_int4_on_the_fly(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                           out_f: int, in_f: int, group: int, bias: torch.Tensor | None = None,
                           out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """int4_matmul.zig:215 linearInt4OnTheFly: out[b] = x[b] * dequant(W)^T + bias.

    ``scales`` is float32 or float16 (the reference's f32 scales or its fp16
    mirror, int4_weights.zig:86-90)."""
    x = x.reshape(-1, in_f)
    assert x.dtype == torch.float32 and x.is_contiguous()
    if out is None:
        out = torch.empty((x.shape[0], out_f), dtype=torch.float32, device=x.device)
    call("glacier_cuda_int4_linear", x.data_ptr(), x.shape[0], packed.data_ptr(), scales.data_ptr(),
         int(scales.dtype == torch.float16), _ptr(bias), out.data_ptr(), out_f, in_f, group,
         _stream(stream))
    return out
