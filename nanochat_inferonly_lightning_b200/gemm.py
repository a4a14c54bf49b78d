"""Python mirror of the GEMM entry points (nc_gemm_skinny for the decode step, nc_gemm for the
prompt pass) over the C ABI.

out[M, N] = epilogue(x[M, K] . w[N, K]^T) for M <= 64 rows, w in the reference layout W[out, in]
(src/model.h:30-47), with the RMSNorm that precedes the reference's projections
(kernels/rmsnorm.cu), the residual add of gemm_half_residual (kernels/gemm.cu:115-166), ReLU^2
and the logit tanh cap (kernels/ops.cu:23-46) fused in as flags.  Tensors are torch CUDA bf16;
the stream defaults to torch's current stream.  Raises NcError on a non-zero status.
Also here: the two small passes at the ends of a decode step (embedding gather + RMSNorm, and
greedy argmax on the device).
"""
import ctypes

import torch

from . import _lib
from .attn import _bf16, _ptr, _stream

NORM_INPUT = 1
RESIDUAL = 2
RELU2 = 4
TANH_CAP = 8
MAX_ROWS = 64


def gemm_skinny(out, x, w, residual=None, flags=0, cap=0.0, seg_cols=0, splits=0, stream=None):
    """out[M, N] (or N / seg_cols segments of [M, seg_cols]) = epilogue(x @ w.T).

    flags: NORM_INPUT (scale row m of the product by rsqrt(mean(x[m]^2) + 1e-6)), RESIDUAL
    (+ residual [M, N], which may be `out` itself), RELU2, TANH_CAP (cap * tanh(v / cap)),
    applied in that order before one bf16 rounding.  splits: K-split count (0 = automatic,
    at most 12)."""
    _bf16(out, x, w, residual)
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"w is {tuple(w.shape)}, x is {tuple(x.shape)}")
    if out.numel() != M * N:
        raise ValueError(f"out has {out.numel()} elements, expected {M * N}")
    if residual is not None:
        flags |= RESIDUAL
    lib = _lib.load()
    _lib.check("nc_gemm_skinny",
               lib.nc_gemm_skinny(_ptr(out), _ptr(x), _ptr(w), _ptr(residual), M, N, K, flags,
                                  ctypes.c_float(cap), seg_cols, splits, _stream(stream)))
    return out


def gemm(out, x, w, residual=None, flags=0, cap=0.0, seg_cols=0, stream=None):
    """The same product and fused steps as gemm_skinny for any number of rows, on the
    persistent tiled kernel (nc_gemm) laid out for the prompt pass."""
    _bf16(out, x, w, residual)
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"w is {tuple(w.shape)}, x is {tuple(x.shape)}")
    if out.numel() != M * N:
        raise ValueError(f"out has {out.numel()} elements, expected {M * N}")
    if residual is not None:
        flags |= RESIDUAL
    lib = _lib.load()
    _lib.check("nc_gemm",
               lib.nc_gemm(_ptr(out), _ptr(x), _ptr(w), _ptr(residual), M, N, K, flags,
                           ctypes.c_float(cap), seg_cols, _stream(stream)))
    return out


def gemm_half(C, A, B, M, N, K, stream=None):
    """kernels/gemm.cu:62-113 for M <= 64: C[M, N] = A[M, K] @ B[N, K]^T."""
    return gemm_skinny(C, A.view(M, K), B.view(N, K), stream=stream)


def gemm_half_residual(D, A, B, residual, M, N, K, stream=None):
    """kernels/gemm.cu:115-166 for M <= 64: D[M, N] = A[M, K] @ B[N, K]^T + residual[M, N]."""
    return gemm_skinny(D, A.view(M, K), B.view(N, K), residual=residual, stream=stream)


def embed_rmsnorm(out, table, tokens, stream=None):
    """kernels/ops.cu:9-20 + kernels/rmsnorm.cu:9-63 in one pass: out[r] = RMSNorm(table[tokens[r]]).
    tokens: int32 CUDA tensor [rows]; table [vocab, dim]; out [rows, dim]."""
    _bf16(out, table)
    if tokens.dtype != torch.int32:
        raise TypeError(f"tokens must be int32, got {tokens.dtype}")
    rows, dim = int(tokens.numel()), int(table.shape[1])
    lib = _lib.load()
    _lib.check("nc_embed_rmsnorm",
               lib.nc_embed_rmsnorm(_ptr(out), _ptr(table), _ptr(tokens), rows, dim,
                                    int(table.shape[0]), _stream(stream)))
    return out


def argmax_rows(out, logits, stream=None):
    """Greedy sampling of src/engine.cpp:88-95 on the device: out[r] (int32) = index of the
    first maximum of logits[r] (bf16 [rows, cols])."""
    _bf16(logits)
    if out.dtype != torch.int32:
        raise TypeError(f"out must be int32, got {out.dtype}")
    rows, cols = logits.shape
    lib = _lib.load()
    _lib.check("nc_argmax_rows",
               lib.nc_argmax_rows(_ptr(out), _ptr(logits), rows, cols, _stream(stream)))
    return out


def sample_rows(out, logits, temperature, top_k, top_p, uniforms, stream=None):
    """Engine::sample (src/engine.cpp:62-131) on the device: out[r] (int32) drawn from
    logits[r] (bf16 [rows, vocab]) with temperature, top-k (1..1024; 0 or >= vocab: off) and
    top-p (>= 1: off; with top-k off it cuts the whole row), using the uniform draw uniforms[r]
    (float32 CUDA tensor [rows]); temperature 0 is greedy."""
    _bf16(logits)
    if out.dtype != torch.int32:
        raise TypeError(f"out must be int32, got {out.dtype}")
    if uniforms is not None and uniforms.dtype != torch.float32:
        raise TypeError(f"uniforms must be float32, got {uniforms.dtype}")
    rows, vocab = logits.shape
    lib = _lib.load()
    _lib.check("nc_sample_rows",
               lib.nc_sample_rows(_ptr(out), _ptr(logits), rows, vocab, ctypes.c_float(temperature),
                                  int(top_k), ctypes.c_float(top_p), _ptr(uniforms),
                                  _stream(stream)))
    return out
