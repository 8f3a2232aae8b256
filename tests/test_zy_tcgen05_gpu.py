"""tcgen05 / TMEM prefill GEMM (bf16 kind::f16 and A8W8 kind::i8) against the CPU oracle.

Collected after the other GPU tests: the tensor-core kernels are the newest code path."""

import pytest
import torch

from oracle import a8w8 as OQ
from oracle import ops as O
from ppu_b200 import kernels as K
from ppu_b200 import lib as L

from .helpers import BF16, assert_bf16_close, assert_residual_close, assert_swiglu_close, randn

pytestmark = pytest.mark.gpu


def cu(t):
    return t.cuda()


@pytest.fixture(autouse=True, params=[True, False], ids=["pairs", "single"])
def sm_pairs(request):
    """Every case runs on the CTA-pair kernel (the default) and on the single-CTA kernel."""
    K.set_gemm_tc_pairs(request.param)
    yield request.param
    K.set_gemm_tc_pairs(True)


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (1024, 8224, 2048), (77, 2048, 6144), (5, 5120, 2048)])
def test_gemm_tc_store(m, n, k):
    a = randn(m, k, seed=m + 1)
    w = randn(n, k, seed=n + 2, scale=0.02)
    out = K.gemm(cu(a), cu(w), tc=True)
    torch.cuda.synchronize()
    assert K.tc_error() == 0
    assert_bf16_close(out.cpu(), O.linear(a, w), max_ulp=2, max_frac=0.02)


def test_gemm_tc_epilogues():
    a = randn(300, 2048, seed=1)
    w = randn(2 * 6144, 2048, seed=2, scale=0.02)
    got = K.gemm(cu(a), cu(w), epilogue=L.EPI_SWIGLU, tc=True)
    assert_swiglu_close(got.cpu(), O.silu_and_mul(O.linear(a, w)))
    wd = randn(2048, 6144, seed=3, scale=0.02)
    act = randn(300, 6144, seed=4)
    r = randn(300, 2048, seed=5)
    rd = cu(r.clone())
    K.gemm(cu(act), cu(wd), epilogue=L.EPI_RESIDUAL, out=rd, tc=True)
    torch.cuda.synchronize()
    assert K.tc_error() == 0
    assert_residual_close(rd, r, O.linear(act, wd))


@pytest.mark.parametrize("epi", [L.EPI_STORE, L.EPI_SWIGLU, L.EPI_RESIDUAL])
def test_gemm_tc_a8w8_bit_exact(epi):
    m, k = 200, 2048
    n = 6144 if epi == L.EPI_SWIGLU else 2048
    rows = 2 * n if epi == L.EPI_SWIGLU else n
    x = randn(m, k, seed=7)
    w = randn(rows, k, seed=8, scale=0.02)
    qw, sw = OQ.quantize_weight(w)
    qx, sx = OQ.quantize_tokens(x)
    y = OQ.dequantize(OQ.int8_matmul_exact(qx, qw), sx, sw)
    if epi == L.EPI_SWIGLU:
        want = O.silu_and_mul(y)
        got = K.gemm_a8w8_tc(cu(qx), cu(sx.reshape(-1)), cu(qw), cu(sw.reshape(-1)), epilogue=epi)
    elif epi == L.EPI_RESIDUAL:
        r = randn(m, n, seed=9)
        want = (r.float() + y.float()).to(BF16)
        got = cu(r.clone())
        K.gemm_a8w8_tc(cu(qx), cu(sx.reshape(-1)), cu(qw), cu(sw.reshape(-1)), epilogue=epi, out=got)
    else:
        want = y
        got = K.gemm_a8w8_tc(cu(qx), cu(sx.reshape(-1)), cu(qw), cu(sw.reshape(-1)))
    torch.cuda.synchronize()
    assert K.tc_error() == 0
    assert torch.equal(got.cpu(), want)


def test_gemm_tc_persistent_many_tiles():
    """Several output tiles per CTA (528 bf16 tiles; 384 A8W8 SwiGLU tiles on 148 CTAs): both TMEM
    accumulators are reused many times, with a ragged last column tile."""
    a = randn(2048, 2048, seed=21)
    w = randn(8224, 2048, seed=22, scale=0.02)
    out = K.gemm(cu(a), cu(w), tc=True)
    torch.cuda.synchronize()
    assert K.tc_error() == 0
    assert_bf16_close(out.cpu(), O.linear(a, w), max_ulp=2, max_frac=0.02)
    x = randn(1024, 2048, seed=23)
    wg = randn(2 * 6144, 2048, seed=24, scale=0.02)
    qw, sw = OQ.quantize_weight(wg)
    qx, sx = OQ.quantize_tokens(x)
    want = O.silu_and_mul(OQ.dequantize(OQ.int8_matmul_exact(qx, qw), sx, sw))
    got = K.gemm_a8w8_tc(cu(qx), cu(sx.reshape(-1)), cu(qw), cu(sw.reshape(-1)), epilogue=L.EPI_SWIGLU)
    torch.cuda.synchronize()
    assert K.tc_error() == 0
    assert torch.equal(got.cpu(), want)

