"""Weight layouts shared by the tcgen05 GEMM and the decode GEMV.

* QKV is one [q_rows + 2*kv_rows, d_model] matrix (q heads, then k heads,
  then v heads), so one GEMM produces the whole projection and its epilogue
  can rotate and scatter per head.
* gate/up is one [2*ffn, d_model] matrix interleaved in blocks of 128 rows
  ([gate_0..127, up_0..127, gate_128..255, up_128..255, ...]) so every
  256-column GEMM tile (and every GEMV warp pair) holds a gate row and its
  matching up row and the SwiGLU is applied in the epilogue.
"""
from __future__ import annotations

import torch

GATE_UP_BLOCK = 128


def fuse_qkv(wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor) -> torch.Tensor:
    return torch.cat((wq, wk, wv), dim=0).contiguous()


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor, block: int = GATE_UP_BLOCK) -> torch.Tensor:
    ffn, d = w_gate.shape
    if w_up.shape != (ffn, d) or ffn % block:
        raise ValueError(f"gate/up must be [ffn, d] with ffn a multiple of {block}")
    g = w_gate.reshape(ffn // block, block, d)
    u = w_up.reshape(ffn // block, block, d)
    return torch.stack((g, u), dim=1).reshape(2 * ffn, d).contiguous()


def split_gate_up(w_gu: torch.Tensor, block: int = GATE_UP_BLOCK) -> tuple[torch.Tensor, torch.Tensor]:
    rows, d = w_gu.shape
    ffn = rows // 2
    pairs = w_gu.reshape(ffn // block, 2, block, d)
    return pairs[:, 0].reshape(ffn, d), pairs[:, 1].reshape(ffn, d)
