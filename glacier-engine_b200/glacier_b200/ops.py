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


def linear_int4_tensor_core(x: torch.Tensor, packed: torch.Tensor, scales_f16: torch.Tensor, out_f: int,
                            in_f: int, group: int, bias: torch.Tensor | None = None, out=None, stream=None):
    """Batched linearInt4OnTheFly on the tcgen05 dequant GEMM (int4_neon.c:1439 M4 GEMM role)."""
    from ._lib import lib
    x = x.reshape(-1, in_f)
    b = x.shape[0]
    out = torch.empty((b, out_f), dtype=torch.float32, device=x.device) if out is None else out
    ws_n = lib().glacier_cuda_int4_matmul_workspace(b, in_f, out_f)
    ws = torch.empty(ws_n, dtype=torch.uint8, device=x.device)
    call("glacier_cuda_int4_matmul_f16scale", x.data_ptr(), b, packed.data_ptr(), scales_f16.data_ptr(), _ptr(bias),
         out.data_ptr(), out_f, in_f, group, ws.data_ptr(), ws_n, _stream(stream))
    return out


def rms_norm_f32(x: torch.Tensor, weight: torch.Tensor, eps: float, out=None, stream=None):
    """kernels.zig:141 rmsNormF32 over rows of x [batch, dim]."""
    b, d = x.shape
    out = torch.empty_like(x) if out is None else out
    call("glacier_cuda_rmsnorm_f32", x.data_ptr(), weight.data_ptr(), eps, out.data_ptr(), b, d, _stream(stream))
    return out


def add_rms_norm_f32(a, b, weight, eps: float, residual=None, out=None, stream=None):
    """kernels.zig:322 addRmsNormF32: residual = a + b, out = rmsnorm(residual)."""
    residual = torch.empty_like(a) if residual is None else residual
    out = torch.empty_like(a) if out is None else out
    call("glacier_cuda_add_rmsnorm_f32", a.data_ptr(), b.data_ptr(), residual.data_ptr(), weight.data_ptr(), eps,
         out.data_ptr(), a.shape[0], a.shape[1], _stream(stream))
    return residual, out


def silu_mul_f32(gate, up, out=None, stream=None):
    """kernels.zig:465 siluMulF32 over rows: silu(gate) * up."""
    b, n = gate.shape
    out = torch.empty_like(gate) if out is None else out
    call("glacier_cuda_silu_mul_f32", gate.data_ptr(), up.data_ptr(), gate.stride(0), out.data_ptr(), out.stride(0),
         b, n, _stream(stream))
    return out


def load_embedding_rows(table_f16, tokens, stream=None):
    """generate.zig:3653 loadEmbeddingRow for a batch of tokens (fp16 table)."""
    vocab, dim = table_f16.shape
    out = torch.empty((tokens.numel(), dim), dtype=torch.float32, device=tokens.device)
    call("glacier_cuda_embedding_f16", table_f16.data_ptr(), vocab, dim, tokens.data_ptr(), tokens.numel(),
         out.data_ptr(), _stream(stream))
    return out


def qkv_rope_append(qkv, bias, cos, sin, pos, num_heads, num_kv_heads, head_dim, kv_pages, page_floats,
                    block_tables, layer, stream=None):
    """RopeTable.apply (generate.zig:816) on q and k + appendRowTxn (paged_kv_cache.zig:1074)."""
    b = qkv.shape[0]
    q_out = torch.empty((b, num_heads * head_dim), dtype=torch.float32, device=qkv.device)
    call("glacier_cuda_qkv_rope_append_f32", qkv.data_ptr(), qkv.stride(0), _ptr(bias), cos.data_ptr(),
         sin.data_ptr(), cos.shape[0], pos.data_ptr(), b, num_heads, num_kv_heads, head_dim, q_out.data_ptr(),
         q_out.stride(0), kv_pages.data_ptr(), page_floats, block_tables.data_ptr(), block_tables.shape[1], layer,
         _stream(stream))
    return q_out


def paged_attention_f32(q, kv_pages, page_floats, block_tables, ctx_lens, max_ctx, layer, num_heads, num_kv_heads,
                        head_dim, stream=None):
    """paged_attention.zig:108 attentionMultiHead, one query row per lane."""
    from ._lib import lib
    lanes = q.shape[0]
    ws_n = lib().glacier_cuda_paged_attention_workspace(lanes, num_heads, num_kv_heads, head_dim, max_ctx)
    ws = torch.empty(ws_n, dtype=torch.float32, device=q.device)
    out = torch.empty((lanes, num_heads * head_dim), dtype=torch.float32, device=q.device)
    call("glacier_cuda_paged_attention_f32", q.data_ptr(), kv_pages.data_ptr(), page_floats, block_tables.data_ptr(),
         block_tables.shape[1], ctx_lens.data_ptr(), max_ctx, lanes, layer, num_heads, num_kv_heads, head_dim,
         out.data_ptr(), ws.data_ptr(), ws_n, _stream(stream))
    return out


def argmax_eligible(logits, words=None, stream=None):
    """sampling.zig:55 argmaxEligible per row -> (tokens int32, status int32)."""
    from ._lib import lib
    b, n = logits.shape
    ws_n = lib().glacier_cuda_argmax_workspace(b, n)
    ws = torch.empty(ws_n, dtype=torch.uint8, device=logits.device)
    tokens = torch.empty(b, dtype=torch.int32, device=logits.device)
    status = torch.empty(b, dtype=torch.int32, device=logits.device)
    wc = 0 if words is None else words.shape[-1]
    call("glacier_cuda_argmax_eligible_f32", logits.data_ptr(), b, n, _ptr(words), wc, tokens.data_ptr(),
         status.data_ptr(), None, ws.data_ptr(), ws_n, _stream(stream))
    return tokens, status
