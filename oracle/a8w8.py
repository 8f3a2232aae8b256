"""CPU restatement of the reference's A8W8 linear (W8A8 int8 with int32 accumulation).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference: explore_runtime_quantization.py:129-181 (``PPUA8W8Linear``).

* Weights (:143-155): per output channel ``s_w = amax|W| / 127`` in FP32 (``1`` where the
  row is all zero), ``q_w = clamp(round(W / s_w), -127, 127)`` as int8.
* Activations (:167-172): dynamic symmetric per-token quantisation through vllm
  ``scaled_int8_quant(x, scale=None, azp=None, symmetric=True)`` (vllm 0.22.0 in this image;
  a compiled op). Restated from vllm's published per-token kernel: ``s_x = amax|x| / 127``
  (``0`` for an all-zero row) and ``q_x = sat_int8(rne(x * (127 / amax)))`` (``0`` for an
  all-zero row) -- a multiplication by the reciprocal, which rounds differently from the
  weight side's division at exact half-way values. A GPU test runs vllm's own op on the same
  rows and compares codes and scales bit for bit.
* Product (:173-180, acext ``int8_gemm``): exact int32 accumulation of int8 products,
  dequantised as ``bf16((float(acc) * s_x) * s_w)``.
"""

from __future__ import annotations

import torch

BF16 = torch.bfloat16


def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-row int8 quantisation; returns ``(q int8 [.., K], scale fp32 [.., 1])``."""
    x32 = x.float()
    absmax = x32.abs().amax(dim=-1, keepdim=True)
    scale = torch.where(absmax > 0, absmax / 127.0, torch.ones_like(absmax))
    q = torch.round(x32 / scale).clamp_(-127, 127).to(torch.int8)
    return q, scale


def quantize_tokens(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token activation quantisation with vllm ``scaled_int8_quant`` semantics; returns
    ``(q int8 [.., K], scale fp32 [.., 1])``. Every step is one IEEE float32 operation, as on the
    GPU: ``amax / 127``, ``127 / amax``, ``x * inv``, round half to even, saturate."""
    x32 = x.float()
    absmax = x32.abs().amax(dim=-1, keepdim=True)
    scale = absmax / 127.0
    inv = torch.where(absmax > 0, torch.full_like(absmax, 127.0) / absmax, torch.zeros_like(absmax))
    q = torch.round(x32 * inv).clamp_(-128, 127).to(torch.int8)
    return q, scale


def quantize_weight(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel weight quantisation, explore_runtime_quantization.py:143-155."""
    return quantize_rows(weight)


def int8_matmul_exact(qx: torch.Tensor, qw: torch.Tensor) -> torch.Tensor:
    """Exact int32 ``qx @ qw^T``. Float64 GEMM is exact here: every partial sum is an
    integer of magnitude below ``127*127*K < 2^53``."""
    acc = qx.reshape(-1, qx.shape[-1]).double() @ qw.double().T
    return acc.to(torch.int64).to(torch.int32).reshape(*qx.shape[:-1], qw.shape[0])


def dequantize(acc: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """``bf16((float(acc) * s_x) * s_w)`` with ``s_x [.., 1]`` and ``s_w [N, 1]``."""
    return ((acc.float() * sx) * sw.reshape(1, -1).float()).to(BF16)


def a8w8_linear(x: torch.Tensor, qw: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """Dynamic-per-token A8W8 linear, explore_runtime_quantization.py:161-181."""
    qx, sx = quantize_tokens(x)
    return dequantize(int8_matmul_exact(qx, qw), sx, sw)
