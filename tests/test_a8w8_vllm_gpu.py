"""A8W8 activation side pinned to the reference's own dependency.

The reference quantises activations with vllm ``scaled_int8_quant(x, scale=None, azp=None,
symmetric=True)`` (explore_runtime_quantization.py:114-126, 167-172). vllm is installed in this
image; its op is compiled CUDA, so it runs here only on the GPU. These tests run it on seeded rows
at the config-1 decode widths (1 x 2048, 1 x 6144) and the prefill-1024 shapes, plus rows built to
hit exact half-way products (entries at +-amax/2) and all-zero rows, and compare the int8 codes
and FP32 scales bit for bit with ``q35_quantize_tokens`` (the CUDA path) and with the CPU oracle.
When vllm cannot load on the box the tests skip with the import error as the reason.
"""

import pytest
import torch

from oracle import a8w8 as OQ
from ppu_b200 import kernels as K

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16


def _vllm_quant():
    try:
        from vllm import _custom_ops as vops

        probe = torch.ones(1, 16, device="cuda", dtype=BF16)
        vops.scaled_int8_quant(probe, scale=None, azp=None, symmetric=True)
    except Exception as exc:  # noqa: BLE001 - the reason is the skip message
        pytest.skip(f"vllm scaled_int8_quant unavailable: {exc!r}")
    return vops.scaled_int8_quant


def _rows(rows: int, width: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, width, generator=g).to(BF16)
    if rows >= 4:
        # half-way products: entries at +-amax/2 (x * 127/amax = +-63.5 up to the reciprocal's
        # rounding); with amax 1.125 / 1.1875 the reciprocal and the division round apart
        for r, amax in ((1, 1.125), (2, 1.1875), (3, 0.7)):
            a = torch.tensor(amax).to(BF16)
            x[r].clamp_(-float(a), float(a))
            x[r, 0] = a
            x[r, 1::7] = (a.float() / 2).to(BF16)
            x[r, 2::11] = (-a.float() / 2).to(BF16)
        x[rows - 1].zero_()  # all-zero row: zero codes and zero scale
    return x


@pytest.mark.parametrize("rows,width", [(1, 2048), (1, 6144), (1024, 2048), (1024, 6144), (7, 2048)])
def test_quantize_tokens_matches_vllm_bit_for_bit(rows, width):
    vq = _vllm_quant()
    x = _rows(rows, width, seed=rows * 7 + width)
    xd = x.cuda()
    q_v, s_v, azp = vq(xd, scale=None, azp=None, symmetric=True)
    q_c, s_c, _ = K.scaled_int8_quant(xd)
    q_o, s_o = OQ.quantize_tokens(x)
    torch.cuda.synchronize()
    assert azp is None
    q_v, s_v = q_v.cpu(), s_v.reshape(rows, 1).cpu()
    flips = int((q_c.cpu() != q_v).sum())
    assert flips == 0, f"{flips} codes differ from vllm (of {rows * width})"
    assert torch.equal(s_c.cpu(), s_v)
    assert torch.equal(q_o, q_v), int((q_o != q_v).sum())
    assert torch.equal(s_o, s_v)


def test_weight_side_formula_differs_from_the_activation_side_at_ties():
    """The weight side divides by the scale (a torch formula in the reference), the activation
    side multiplies by vllm's reciprocal: at +-amax/2 entries the two can round apart, which is
    why the two quantisers are separate entry points."""
    x = _rows(8, 2048, seed=11)
    q_rows, s_rows = K.quantize_rows(x.cuda())
    q_tok, s_tok, _ = K.scaled_int8_quant(x.cuda())
    torch.cuda.synchronize()
    assert torch.equal(q_rows.cpu(), OQ.quantize_rows(x)[0])
    assert torch.equal(q_tok.cpu(), OQ.quantize_tokens(x)[0])
    assert float(s_rows[7]) == 1.0 and float(s_tok[7]) == 0.0  # the all-zero row
    assert (q_rows[1:3].cpu() != q_tok[1:3].cpu()).any()  # the tie entries of rows 1-2
