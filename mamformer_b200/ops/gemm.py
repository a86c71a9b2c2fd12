"""Python front-end of the tcgen05 GEMM (``csrc/gemm_tcgen05.cu``).

All functions compute in bf16 with fp32 accumulation on the tensor cores.

* ``mm(a, b)``                  a (M, K) @ b (N, K)^T         -> (M, N)       [nn.Linear forward]
* ``mm_nn(a, b)``               a (M, K) @ b (K, N)           -> (M, N)       [input gradient]
* ``mm_tn_acc(dy, x, out)``     out (N, K) (+)= dy (M, N)^T x (M, K)          [weight gradient]
* ``grouped_mm(x, w, seg, tile_off)``      per-group x_g @ w_g^T (w: G, N, K)
* ``grouped_mm_nn(x, w, seg, tile_off)``   per-group x_g @ w_g   (w: G, K, N)
* ``grouped_wgrad(dy, x, seg, out, acc)``  out[g] (+)= dy_g^T x_g

Grouped row segments are 64-aligned (zero-padded rows); ``tile_offsets`` builds the device-side
tile table, so no call here synchronises with the host.
"""

from __future__ import annotations

from typing import Optional

import torch

from mamformer_b200.ops._ext import require_native


def _C():
    return require_native()


def mm(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
       out_dtype: torch.dtype = torch.bfloat16, alpha: float = 1.0) -> torch.Tensor:
    M, N = a.shape[0], b.shape[0]
    out = torch.empty(M, N, device=a.device, dtype=out_dtype) if out is None else out
    _C().gemm_tn(a, False, b, False, out, False, None, None, 0, alpha)
    return out


def mm_nn(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
          out_dtype: torch.dtype = torch.bfloat16, alpha: float = 1.0) -> torch.Tensor:
    M, N = a.shape[0], b.shape[1]
    out = torch.empty(M, N, device=a.device, dtype=out_dtype) if out is None else out
    _C().gemm_tn(a, False, b, True, out, False, None, None, 0, alpha)
    return out


def mm_tn_acc(dy: torch.Tensor, x: torch.Tensor, out: torch.Tensor, accumulate: bool = True,
              alpha: float = 1.0) -> torch.Tensor:
    """out (N, K) (+)= alpha * dy^T @ x with dy (M, N), x (M, K); out fp32 (accumulate) or bf16."""
    _C().gemm_tn(dy, True, x, True, out, accumulate, None, None, 0, alpha)
    return out


def grouped_mm(x, w, seg, tile_off, out=None, out_dtype=torch.bfloat16):
    out = torch.empty(x.shape[0], w.shape[1], device=x.device, dtype=out_dtype) if out is None else out
    _C().gemm_tn(x, False, w, False, out, False, seg, tile_off, 1, 1.0)
    return out


def grouped_mm_nn(x, w, seg, tile_off, out=None, out_dtype=torch.bfloat16):
    out = torch.empty(x.shape[0], w.shape[2], device=x.device, dtype=out_dtype) if out is None else out
    _C().gemm_tn(x, False, w, True, out, False, seg, tile_off, 1, 1.0)
    return out


def grouped_wgrad(dy, x, seg, out, accumulate: bool = True):
    """out[g] (N, K) (+)= dy[rows_g]^T x[rows_g]; dy (Mt, N), x (Mt, K)."""
    _C().gemm_tn(dy, True, x, True, out, accumulate, seg, None, 2, 1.0)
    return out


def tile_offsets(seg: torch.Tensor, block_m: int = 128) -> torch.Tensor:
    """Cumulative m-tile counts (int32, device) for 64-aligned row segments."""
    tiles = (seg[1:] - seg[:-1] + block_m - 1) // block_m
    return torch.cat([seg.new_zeros(1), torch.cumsum(tiles, 0)]).to(torch.int32)


def check_error():
    err = int(_C().gemm_error())
    if err:
        _C().gemm_clear_error()
        raise RuntimeError(f"tcgen05 gemm reported a wait timeout (code {err})")
