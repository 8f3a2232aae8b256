"""Per-operator parity of the sm_100a kernels (through the C ABI) against the CPU oracle.

Bar: bit-exact for int8 quantisation and int32 accumulation; <= 1e-2 relative error (and at
most 1-2 BF16 ulps on a small fraction of elements) for BF16 paths; identical top-1 indices
with the lowest-index tie rule. Inputs are seeded; shapes follow validate_kernels.py and the
BASELINE configs.
"""

from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from oracle import a8w8 as OQ
from oracle import ops as O
from ppu_b200 import kernels as K
from ppu_b200 import lib as L

from .helpers import BF16, assert_bf16_close, assert_residual_close, assert_swiglu_close, randn, rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden.pt")


def cu(t):
    return t.to(DEV)


# ------------------------------------------------------------------ golden vectors through the GPU
def test_golden_norms_and_activations():
    for w in (128, 256, 2048):
        c = GOLDEN[f"rms_{w}"]
        assert_bf16_close(K.rms_norm(cu(c["x"]), cu(c["w"])).cpu(), c["out"])
    c = GOLDEN["residual_add_rms"]
    r, n = K.residual_add_rms_norm(cu(c["r"]), cu(c["u"]), cu(c["w"]))
    assert torch.equal(r.cpu(), c["added"])
    assert_bf16_close(n.cpu(), c["out"])
    for key in ("gated_rms", "gated_rms_hf"):
        c = GOLDEN[key]
        assert_bf16_close(K.gated_rms_norm(cu(c["x"]), cu(c["gate"]), cu(c["w"])).cpu(), c["out"])
    c = GOLDEN["silu_mul"]
    assert_bf16_close(K.silu_and_mul(cu(c["packed"])).cpu(), c["out"])
    c = GOLDEN["sigmoid_mul"]
    assert_bf16_close(K.sigmoid_mul(cu(c["x"]), cu(c["gate"])).cpu(), c["out"])
    c = GOLDEN["swiglu_gemv"]
    assert_bf16_close(K.ppu_swiglu_gemv(cu(c["x"]), cu(c["w"])).cpu(), c["out"], max_ulp=2)


def test_golden_qgkv_and_gate():
    c = GOLDEN["qgkv"]
    kw = dict(q_heads=8, kv_heads=2, dim=256, rotary_dim=64)
    q, k, v = K.qgkv_norm_rope(cu(c["packed"]), cu(c["qw"]), cu(c["kw"]), cu(c["cos"]), cu(c["sin"]), **kw)
    assert_bf16_close(q.cpu(), c["q"])
    assert_bf16_close(k.cpu(), c["k"])
    assert torch.equal(v.cpu(), c["v"])
    kc = torch.zeros(1, 2, 13, 256, dtype=BF16, device=DEV)
    vc = torch.zeros_like(kc)
    start = torch.tensor(3, device=DEV, dtype=torch.int64)
    _, k2, v2 = K.qgkv_norm_rope(cu(c["packed"]), cu(c["qw"]), cu(c["kw"]), cu(c["cos"]), cu(c["sin"]),
                                 cache_key=kc, cache_value=vc, cache_start=start, **kw)
    assert_bf16_close(k2[:, :, 3:8].cpu(), c["k"])
    assert torch.equal(v2[:, :, 3:8].cpu(), c["v"])
    assert not k2[:, :, :3].any() and not v2[:, :, 8:].any()  # prefix/suffix untouched (KAT)
    assert_bf16_close(K.attention_gate_mul(cu(c["attn_out"]), cu(c["packed"]), 256).cpu(), c["gated"])


# widths that take the 16-byte vector kernels (multiples of 8, warp-per-row norms at 256-1024)
# and widths that fall back to the scalar kernels
@pytest.mark.parametrize("rows,width", [(1024, 256), (300, 512), (33, 1024), (64, 2048), (17, 200), (9, 129)])
def test_norms_vector_and_scalar_paths(rows, width):
    x, u = randn(rows, width, seed=width), randn(rows, width, seed=width + 1)
    w = randn(width, seed=width + 2, scale=0.1)
    assert_bf16_close(K.rms_norm(cu(x), cu(w)).cpu(), O.rms_norm(x, w))
    r, n = K.residual_add_rms_norm(cu(x), cu(u), cu(w))
    ro, no = O.residual_add_rms_norm(x, u, w)
    assert torch.equal(r.cpu(), ro)
    assert_bf16_close(n.cpu(), no)
    g = randn(rows, width, seed=width + 3)
    assert_bf16_close(K.gated_rms_norm(cu(x), cu(g), cu(w)).cpu(), O.gated_rms_norm(x, g, w))


@pytest.mark.parametrize("rows,width", [(1024, 6144), (1, 6144), (3, 100)])
def test_activations_vector_and_scalar_paths(rows, width):
    packed = randn(rows, 2 * width, seed=width)
    assert_bf16_close(K.silu_and_mul(cu(packed)).cpu(), O.silu_and_mul(packed))
    x, gt = randn(rows, width, seed=width + 1), randn(rows, width, seed=width + 2)
    assert_bf16_close(K.sigmoid_mul(cu(x), cu(gt)).cpu(), O.sigmoid_mul(x, gt))
    for hidden, hd in ((2048, 256), (96, 12)):  # vector path / head_dim not a multiple of 8
        att = randn(rows, hidden, seed=hidden)
        qg = randn(rows, 2 * hidden + 64, seed=hidden + 1)
        assert_bf16_close(K.attention_gate_mul(cu(att), cu(qg), hd).cpu(), O.attention_gate_mul(att, qg, hd))


def test_golden_lm_head_and_tie():
    c = GOLDEN["lm_head"]
    assert torch.equal(K.lm_head_argmax(cu(c["h"]), cu(c["w"])).cpu(), c["out"])
    c = GOLDEN["lm_head_tie"]
    assert int(K.lm_head_argmax(cu(c["h"]), cu(c["w"]))) == 0


def test_golden_gqa_decode():
    c = GOLDEN["gqa_decode"]
    for n, expected in c["out"].items():
        length = torch.tensor([n], device=DEV, dtype=torch.int64)
        out = K.gqa_decode_attention(cu(c["q"]), cu(c["k"]), cu(c["v"]), length, 0.0625)
        assert rel_err(out, expected) < 1e-2, n


@pytest.mark.parametrize("n", [1, 17])
def test_golden_conv(n):
    c = GOLDEN[f"conv_{n}"]
    st = cu(c["state0"].clone())
    out = K.causal_conv1d_fused(cu(c["x"]), cu(c["w"]), st)
    assert_bf16_close(out.cpu(), c["out"])
    assert torch.equal(st.cpu(), c["state"])
    st = cu(c["state0"].clone())
    out = K.causal_conv1d_fused(cu(c["px"]), cu(c["w"]), st)
    assert_bf16_close(out.cpu(), c["pout"])
    assert torch.equal(st.cpu(), c["pstate"])


# the sliding-window kernel (full and partial last runs, packed rows wider than the channels) and
# the generic kernel (L < 4): outputs against the oracle, the conv state bit-exact
@pytest.mark.parametrize("length,channels,stride", [(1024, 6144, 8224), (37, 6144, 6144), (50, 100, 100),
                                                    (3, 64, 64)])
def test_causal_conv_paths(length, channels, stride):
    x = randn(1, length, stride, seed=length + channels)
    w = randn(channels, 4, seed=5, scale=0.5)
    st0 = randn(1, channels, 4, seed=6)
    st = cu(st0.clone())
    out = K.causal_conv1d_fused(cu(x), cu(w), st)
    sto = st0.clone()
    want = O.causal_conv1d(x, w, sto)
    assert_bf16_close(out.cpu(), want)
    assert torch.equal(st.cpu(), sto)


def test_golden_delta_recurrent():
    c = GOLDEN["delta"]
    st = cu(c["state0"].clone())
    out = K.delta_recurrent_fused(cu(c["qkv"]), cu(c["packed"]), cu(c["a_log"]), cu(c["dt_bias"]), st)
    assert_bf16_close(out.cpu(), c["out"], max_ulp=1, max_frac=0.02)
    assert torch.allclose(st.cpu(), c["state"], rtol=1e-4, atol=1e-5)


# ------------------------------------------------------------------ A8W8 (bit-exact)
@pytest.mark.parametrize("rows,width", [(1, 2048), (7, 6144), (64, 2048), (5, 100), (1024, 2048)])
def test_quantize_rows_bit_exact(rows, width):
    x = randn(rows, width, seed=rows + width)
    x[0, :5] = 0
    if rows > 1:
        x[1].zero_()  # all-zero row -> scale 1
    q, s = K.quantize_rows(cu(x))
    qo, so = OQ.quantize_rows(x)
    assert torch.equal(q.cpu(), qo)
    assert torch.equal(s.cpu(), so)


@pytest.mark.parametrize("rows,width", [(1, 2048), (7, 6144), (64, 2048), (5, 100), (1024, 2048)])
def test_quantize_tokens_bit_exact(rows, width):
    x = randn(rows, width, seed=rows + width + 1)
    x[0, :5] = 0
    x[0, 7] = 2.0
    x[0, 9] = 1.0  # +-amax/2: a half-way product
    x[0, 10] = -1.0
    if rows > 1:
        x[1].zero_()  # all-zero row -> codes 0, scale 0
    q, s, _ = K.scaled_int8_quant(cu(x))
    qo, so = OQ.quantize_tokens(x)
    assert torch.equal(q.cpu(), qo)
    assert torch.equal(s.cpu(), so)


@pytest.mark.parametrize("m,n,k", [(1, 512, 2048), (37, 300, 2048), (128, 256, 6144)])
def test_int8_gemm_int32_bit_exact(m, n, k):
    g = torch.Generator().manual_seed(m * n + k)
    qx = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    acc = K.int8_gemm(cu(qx), cu(qw))
    assert torch.equal(acc.cpu(), OQ.int8_matmul_exact(qx, qw))


@pytest.mark.parametrize("m", [1, 9, 256])
def test_a8w8_linear_bit_exact(m):
    x = randn(m, 2048, seed=m)
    w = randn(6144, 2048, seed=100 + m, scale=0.02)
    qw, sw = OQ.quantize_weight(w)
    out = K.a8w8_linear(cu(x), cu(qw), cu(sw.reshape(-1)))
    assert torch.equal(out.cpu(), OQ.a8w8_linear(x, qw, sw))


# ------------------------------------------------------------------ decode GEMVs
def test_swiglu_gemv_reference_shape():
    x = randn(1, 1, 2048, seed=1)
    w = randn(12288, 2048, seed=2, scale=0.02)
    assert_bf16_close(K.ppu_swiglu_gemv(cu(x), cu(w)).cpu(), O.swiglu_gemv(x, w), max_ulp=2)


@pytest.fixture(params=[L.Q35_GEMV_BULK, L.Q35_GEMV_REGISTERS], ids=["bulk", "registers"])
def gemv_variant(request):
    L.call("q35_set_gemv_variant", request.param)
    yield request.param
    L.call("q35_set_gemv_variant", L.Q35_GEMV_REGISTERS)
    assert L.load().q35_gemv_error() == 0


@pytest.mark.parametrize("int8", [False, True])
@pytest.mark.parametrize("kind", ["norm_store", "embed_store", "plain_residual", "norm_swiglu", "down_residual"])
def test_fused_gemv(kind, int8, gemv_variant):
    torch.manual_seed(0)
    H, I = 2048, 6144
    rows = {"norm_store": 8224, "embed_store": 5120, "plain_residual": H, "norm_swiglu": 2 * I,
            "down_residual": H}[kind]
    k = I if kind == "down_residual" else H
    w = randn(rows, k, seed=3, scale=0.02)
    x = randn(k, seed=4)
    nw = randn(H, seed=5, scale=0.1)
    resid = randn(H, seed=6)
    emb = randn(1000, H, seed=7, scale=0.02)
    tok = torch.tensor([123], dtype=torch.int64)
    if int8:
        qw, sw = OQ.quantize_weight(w)
        wd, swd = cu(qw), cu(sw.reshape(-1))
        lin = lambda v: OQ.a8w8_linear(v[None], qw, sw)[0]
    else:
        wd, swd = cu(w), None
        lin = lambda v: O.linear(v[None], w)[0]
    if kind == "norm_store":
        got = K.fused_gemv(wd, cu(resid), prologue=L.PRO_NORM, norm_weight=cu(nw), w_scale=swd)
        want = lin(O.rms_norm(resid, nw))
    elif kind == "embed_store":
        r = torch.zeros(H, dtype=BF16, device=DEV)
        got = K.fused_gemv(wd, None, prologue=L.PRO_EMBED, norm_weight=cu(nw), w_scale=swd, token=cu(tok),
                           embed=cu(emb), resid=r)
        want = lin(O.rms_norm(emb[123], nw))
        assert torch.equal(r.cpu(), emb[123])
    elif kind in ("plain_residual", "down_residual"):
        r = cu(resid.clone())
        K.fused_gemv(wd, cu(x), epilogue=L.EPI_RESIDUAL, resid=r, w_scale=swd)
        got = r
        want = (resid.float() + lin(x).float()).to(BF16)
    else:
        got = K.fused_gemv(wd, cu(resid), prologue=L.PRO_NORM, epilogue=L.EPI_SWIGLU, norm_weight=cu(nw),
                           w_scale=swd)
        want = O.silu_and_mul(lin(O.rms_norm(resid, nw)))
    if int8:
        assert torch.equal(got.cpu(), want), "A8W8 GEMV must be bit-exact"
    else:
        assert_bf16_close(got.cpu(), want, max_ulp=2, max_frac=0.05)


def test_lm_head_full_vocab():
    h = randn(1, 2048, seed=11)
    nw = randn(2048, seed=12, scale=0.02)
    e = randn(248320, 2048, seed=13, scale=0.02)
    hn = O.rms_norm(h, nw)
    tok = K.lm_head_argmax(cu(h), cu(e), norm_weight=cu(nw))
    want = O.lm_head_argmax(hn, e)
    if int(tok) != int(want):  # only acceptable on a BF16 tie-break of equal-rounded logits
        logits = O.linear(hn, e).float()[0]
        assert logits[int(tok)] == logits[int(want)] and int(tok) > int(want), (int(tok), int(want))
    # duplicated maximum -> lowest index wins
    e2 = e.clone()
    e2[200000] = e2[int(want)]
    assert int(K.lm_head_argmax(cu(h), cu(e2), norm_weight=cu(nw))) == min(int(want), 200000)


# ------------------------------------------------------------------ prefill GEMM
@pytest.mark.parametrize("m,n,k", [(1024, 8224, 2048), (77, 2048, 6144), (5, 5120, 2048)])
def test_gemm_bf16(m, n, k):
    a = randn(m, k, seed=m)
    w = randn(n, k, seed=n, scale=0.02)
    out = K.gemm(cu(a), cu(w))
    assert_bf16_close(out.cpu(), O.linear(a, w), max_ulp=2, max_frac=0.02)


def test_gemm_epilogues():
    a = randn(130, 2048, seed=1)
    w = randn(2 * 6144, 2048, seed=2, scale=0.02)
    got = K.gemm(cu(a), cu(w), epilogue=L.EPI_SWIGLU)
    assert_swiglu_close(got.cpu(), O.silu_and_mul(O.linear(a, w)))
    wd = randn(2048, 6144, seed=3, scale=0.02)
    act = randn(130, 6144, seed=4)
    r = randn(130, 2048, seed=5)
    rd = cu(r.clone())
    K.gemm(cu(act), cu(wd), epilogue=L.EPI_RESIDUAL, out=rd)
    assert_residual_close(rd, r, O.linear(act, wd))


# ------------------------------------------------------------------ attention
@pytest.mark.parametrize("batch,length", [(1, 1024), (8, 1024), (1, 4096), (8, 4096), (1, 16384), (8, 16384)])
def test_gqa_decode_config2(batch, length):
    """8 Q / 2 KV heads, D 256, K/V ~ N(0,1), fp32-softmax reference."""
    g = torch.Generator().manual_seed(batch * 7 + length)
    q = torch.randn(batch, 8, 1, 256, generator=g).to(BF16)
    kc = torch.randn(batch, 2, length, 256, generator=g).to(BF16)
    vc = torch.randn(batch, 2, length, 256, generator=g).to(BF16)
    valid = torch.tensor([length], dtype=torch.int64, device=DEV)
    out = K.gqa_decode_attention(cu(q), cu(kc), cu(vc), valid, 0.0625)
    want = O.gqa_decode_attention(q, kc, vc, length, 0.0625)
    assert rel_err(out, want) < 1e-2


@pytest.mark.parametrize("Lmax,p", [(600, 517), (2000, 1803)], ids=["cluster", "split-kv"])
def test_attn_decode_fused_matches_oracle(Lmax, p):
    """Whole decode attention mixer: Q/K norm + partial RoPE at the device position, K/V cache
    write at row cache_len, attention over rows [0, cache_len], sigmoid gate. Caches up to 1280
    rows take the cluster kernel, longer ones the split-KV kernel (staged blocks, current token
    from registers, ticketed combine)."""
    torch.manual_seed(0)
    packed = randn(1, 5120, seed=1)
    qw, kw = randn(256, seed=2, scale=0.1), randn(256, seed=3, scale=0.1)
    kc = randn(1, 2, Lmax, 256, seed=4)
    vc = randn(1, 2, Lmax, 256, seed=5)
    inv = O.rope_inv_freq(64, 1e7)
    pos = 530
    kcd, vcd = cu(kc.clone()), cu(vc.clone())
    out = K.attn_decode(cu(packed), cu(qw), cu(kw), cu(inv), kcd, vcd, torch.tensor([p], device=DEV),
                        torch.tensor([pos], device=DEV), q_heads=8, kv_heads=2, rotary_dim=64)
    cos, sin = O.rope_cos_sin(torch.tensor([[pos]]), inv)
    kco, vco = kc.clone(), vc.clone()
    q, _, _ = O.qgkv_norm_rope(packed[None], qw, kw, cos, sin, q_heads=8, kv_heads=2, dim=256, rotary_dim=64,
                               cache_key=kco, cache_value=vco, cache_start=p)
    att = O.gqa_decode_attention(q, kco, vco, p + 1, 0.0625)
    want = O.attention_gate_mul(att, packed[None], 256)[0]
    assert_bf16_close(kcd[:, :, p].cpu(), kco[:, :, p], max_ulp=1, max_frac=0.05)
    assert torch.equal(vcd[:, :, p].cpu(), vco[:, :, p])
    assert torch.equal(kcd[:, :, p + 1:].cpu(), kc[:, :, p + 1:])
    assert rel_err(out, want) < 1e-2


@pytest.mark.parametrize("length", [1, 70, 1024])
def test_prefill_attention(length):
    q = randn(1, 8, length, 256, seed=1)
    k = randn(1, 2, length, 256, seed=2)
    v = randn(1, 2, length, 256, seed=3)
    out = K.prefill_attention(cu(q), cu(k), cu(v), 0.0625)
    err = rel_err(out, O.causal_attention(q, k, v, 0.0625))
    assert err < 1e-2
    if length == 1024:  # probabilities kept to ~16 bits: within a few BF16 output roundings of FP32
        assert err < 3e-3, err


# every group size runs on the tensor-core kernel: G = 8 as two groups of 4 per KV head, G = 6 as
# three of 2, G = 3 and 5 as single heads; batch 2 and a query offset into a longer KV
@pytest.mark.parametrize("hq,hkv,length,kv_extra", [(16, 2, 200, 0), (12, 2, 64, 0), (3, 1, 33, 0),
                                                   (10, 2, 80, 0), (8, 2, 50, 30)])
def test_prefill_attention_group_sizes(hq, hkv, length, kv_extra):
    q = randn(2, hq, length, 256, seed=hq)
    k = randn(2, hkv, length + kv_extra, 256, seed=hq + 1)
    v = randn(2, hkv, length + kv_extra, 256, seed=hq + 2)
    out = K.prefill_attention(cu(q), cu(k), cu(v), 0.0625, q_offset=kv_extra)
    assert rel_err(out, O.causal_attention(q, k, v, 0.0625, q_offset=kv_extra)) < 1e-2


# the decoder's tcgen05 attention (4 query heads per KV head): ragged lengths around the 32-query
# blocks and 64-key tiles, batch 2, cache rows past L holding other values (masked), full 1024
@pytest.mark.parametrize("batch,length,extra", [(1, 1, 0), (1, 17, 5), (2, 64, 64), (1, 100, 28), (2, 333, 3),
                                                (1, 1024, 0)])
def test_prefill_attention_tc(batch, length, extra):
    q = randn(batch, 8, length, 256, seed=length)
    k = randn(batch, 2, length + extra, 256, seed=length + 1)
    v = randn(batch, 2, length + extra, 256, seed=length + 2)
    out = K.prefill_attention_tc(cu(q), cu(k), cu(v), 0.0625)
    err_word = int(L.load().q35_prefill_attention_tc_error())
    assert err_word == 0, f"bounded wait gave up at barrier slot {err_word - 1}"
    want = O.causal_attention(q, k[:, :, :length], v[:, :, :length], 0.0625)
    err = rel_err(out, want)
    assert err < 3e-3, err  # probabilities kept to ~16 bits, as the warp-MMA kernel
    ref = K.prefill_attention(cu(q), cu(k[:, :, :length].contiguous()), cu(v[:, :, :length].contiguous()), 0.0625)
    assert rel_err(out, ref.cpu()) < 3e-3


def test_prefill_attention_tc_workspace_reuse():
    """Blocks whose keys are split over two CTAs merge through the workspace; its ticket words
    return to zero, so back-to-back calls on one workspace give identical outputs."""
    length = 700
    q = cu(randn(1, 8, length, 256, seed=71))
    k = cu(randn(1, 2, length, 256, seed=72))
    v = cu(randn(1, 2, length, 256, seed=73))
    stride = (length + 63) // 64 * 64
    vt = torch.zeros((1, 2, 256, stride), device=DEV, dtype=BF16)
    vt[..., :length] = v.transpose(-1, -2)
    nbytes = int(L.load().q35_prefill_attention_tc_workspace_size(1, 2, length))
    ws = torch.zeros(nbytes, device=DEV, dtype=torch.uint8)
    outs = []
    for _ in range(2):
        out = torch.empty((1, length, 8 * 256), device=DEV, dtype=BF16)
        L.call("q35_prefill_attention_tc", L.ptr(q), L.ptr(k), L.ptr(vt), L.ptr(out), 1, 8, 2, length, length, stride,
               0.0625, L.ptr(ws), nbytes, 0)
        torch.cuda.synchronize()
        outs.append(out)
        assert int(L.load().q35_prefill_attention_tc_error()) == 0
    assert torch.equal(outs[0], outs[1])
    assert int(ws[: 2 * 22 * 4].view(torch.int32).abs().sum()) == 0  # the 2 x 22 ticket words
    assert rel_err(outs[0], O.causal_attention(q.cpu(), k.cpu(), v.cpu(), 0.0625)) < 3e-3


# ------------------------------------------------------------------ DeltaNet
def _delta_inputs(L_, seed=0):
    """16 heads x 128, conv K=4, alpha = exp(-softplus(N(0,1))),
    beta = sigmoid(N(0,1)) (A_log = dt_bias = 0, a/b ~ N(0,1)), inputs ~ N(0,1)."""
    H, D = 16, 128
    rows = 4 * H * D + 2 * H
    packed = randn(1, L_, rows + 32, seed=seed)
    conv_w = randn(3 * H * D, 4, seed=seed + 1, scale=0.5)
    a_log = torch.zeros(H, dtype=BF16)
    dt_bias = torch.zeros(H, dtype=BF16)
    gnorm = (1 + randn(D, seed=seed + 2, scale=0.1).float()).to(BF16)
    return packed, conv_w, a_log, dt_bias, gnorm


@pytest.mark.parametrize("length", [3, 100, 1024])
def test_delta_recurrent_prefill_scan(length):
    packed, conv_w, a_log, dt_bias, _ = _delta_inputs(length)
    st0 = torch.randn(1, 16, 128, 128, generator=torch.Generator().manual_seed(9)) * 0.01
    cst = torch.zeros(1, 3 * 16 * 128, 4, dtype=BF16)
    qkv = O.causal_conv1d(packed, conv_w, cst)
    st = st0.clone()
    want = O.delta_recurrent(qkv, packed, a_log, dt_bias, st)
    std = cu(st0.clone())
    got = K.delta_recurrent_fused(cu(qkv), cu(packed), cu(a_log), cu(dt_bias), std)
    assert rel_err(got, want) < 1e-2
    assert torch.allclose(std.cpu(), st, rtol=1e-3, atol=1e-4)


def test_delta_prefill_chunked_equivalence():
    """The sequential scan agrees with HF's chunked (chunk 64) form over 1024 tokens."""
    packed, conv_w, a_log, dt_bias, _ = _delta_inputs(1024, seed=3)
    cst = torch.zeros(1, 3 * 16 * 128, 4, dtype=BF16)
    qkv = O.causal_conv1d(packed, conv_w, cst)
    H, D = 16, 128
    q, k, v = qkv.float().reshape(1, 1024, 3, H, D).unbind(2)
    a_off = 3 * H * D + H * D
    qh, kh, _, beta, g = O.delta_factors(q, k, packed[..., a_off:a_off + H], packed[..., a_off + H:a_off + 2 * H],
                                         a_log, dt_bias, D)
    st = torch.zeros(1, H, D, D)
    want = O.chunk_gated_delta_rule(qh, kh, v, g, beta, st).to(BF16)
    std = torch.zeros(1, H, D, D, device=DEV)
    got = K.delta_recurrent_fused(cu(qkv), cu(packed), cu(a_log), cu(dt_bias), std)
    assert rel_err(got, want) < 1e-2
    assert torch.allclose(std.cpu(), st, rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("length", [4, 70, 1024])
def test_delta_chunked_conv_matches_separate_conv(length):
    """The causal conv folded into the chunk prep equals causal_conv1d_fused followed by
    delta_chunked_fused bit for bit: conv state, recurrent state and outputs (4-token minimum,
    a partial chunk with its halo from the previous chunk, the full prefill length)."""
    H, D = 16, 128
    packed = randn(1, length, 4 * H * D + 2 * H, seed=length)
    cw = randn(3 * H * D, 4, seed=11, scale=0.5)
    a_log, dt_bias = randn(H, seed=12, scale=0.5), randn(H, seed=13, scale=0.5)
    cs1 = torch.zeros(1, 3 * H * D, 4, dtype=BF16, device=DEV)
    st1 = torch.zeros(1, H, D, D, device=DEV)
    conv = K.causal_conv1d_fused(cu(packed), cu(cw), cs1)
    out1 = K.delta_chunked_fused(conv, cu(packed), cu(a_log), cu(dt_bias), st1)
    cs2 = torch.zeros_like(cs1)
    st2 = torch.zeros_like(st1)
    out2 = K.delta_chunked_conv_fused(cu(packed), cu(cw), cs2, cu(a_log), cu(dt_bias), st2)
    assert torch.equal(cs1, cs2)
    assert torch.equal(out1, out2)
    assert torch.equal(st1, st2)


def test_delta_decode_fused_matches_oracle():
    """One DeltaNet decode step: conv update + SiLU, q/k L2 norm, state update, gated norm."""
    packed, conv_w, a_log, dt_bias, gnorm = _delta_inputs(1, seed=5)
    conv_st = randn(1, 3 * 16 * 128, 4, seed=6)
    st0 = torch.randn(1, 16, 128, 128, generator=torch.Generator().manual_seed(7)) * 0.05
    # oracle
    cs, st = conv_st.clone(), st0.clone()
    qkv = O.causal_conv1d(packed, conv_w, cs)
    core = O.delta_recurrent(qkv, packed, a_log, dt_bias, st)
    z = packed[..., 3 * 2048:4 * 2048].reshape(-1, 128)
    want = O.gated_rms_norm(core.reshape(-1, 128), z, gnorm).reshape(-1)
    # kernel
    csd, std = cu(conv_st.clone()), cu(st0.clone())
    got = K.delta_decode(cu(packed[:, 0]), cu(conv_w), csd, cu(a_log), cu(dt_bias), cu(gnorm), std)
    assert torch.equal(csd.cpu(), cs)
    assert torch.allclose(std.cpu(), st, rtol=1e-4, atol=1e-5)
    assert_bf16_close(got[0].cpu(), want, max_ulp=2, max_frac=0.05)


@pytest.mark.parametrize("length", [1, 3, 64, 100, 1024])
def test_delta_chunked_prefill(length):
    """Chunked WY scan (prefill) against the oracle's sequential recurrence and, at 1024 tokens,
    against the oracle's restatement of HF's chunked rule; state updated in place."""
    packed, conv_w, a_log, dt_bias, _ = _delta_inputs(length, seed=11)
    a_log = randn(16, seed=12, scale=0.5)  # non-trivial decays as well
    dt_bias = randn(16, seed=13, scale=0.5)
    st0 = torch.randn(1, 16, 128, 128, generator=torch.Generator().manual_seed(14)) * 0.01
    qkv = O.causal_conv1d(packed, conv_w, torch.zeros(1, 3 * 16 * 128, 4, dtype=BF16))
    st = st0.clone()
    want = O.delta_recurrent(qkv, packed, a_log, dt_bias, st)
    std = cu(st0.clone())
    got = K.delta_chunked_fused(cu(qkv), cu(packed), cu(a_log), cu(dt_bias), std)
    torch.cuda.synchronize()
    assert K.tc_error() == 0
    assert rel_err(got, want) < 1e-2
    assert torch.allclose(std.cpu(), st, rtol=1e-3, atol=1e-4)
