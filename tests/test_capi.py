"""The C ABI library loads and exports every entry point of include/qwen35_b200.h (no GPU needed).

Argument validation runs on the host before any CUDA call, so invalid calls can be checked
here: they must fail with Q35_EINVAL, which the Python mirror raises as ValueError exactly
where the reference raises ValueError.
"""

import ctypes as C
import re
from pathlib import Path

import pytest

from ppu_b200 import lib as L

HEADER = Path(__file__).resolve().parents[1] / "include" / "qwen35_b200.h"


def header_symbols() -> set[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return set(re.findall(r"\b(q35_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_header_symbol():
    lib = L.load()
    syms = header_symbols()
    assert len(syms) >= 30
    for name in sorted(syms):
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert syms == set(L.EXPORTED), (syms ^ set(L.EXPORTED))
    assert lib.q35_abi_version() == 1


def test_invalid_arguments_are_rejected_on_host():
    lib = L.load()
    assert lib.q35_rms_norm(None, None, None, 1, 2048, 1e-6, None) == L.Q35_EINVAL
    assert "null" in L.last_error()
    with pytest.raises(ValueError):
        L.call("q35_rms_norm", None, None, None, 1, 2048, 1e-6, None)
    # shape checks mirror kernels.py (head dim, packed width, workspace sizes)
    assert lib.q35_delta_recurrent(8, 8, 8, 8, 8, 8, 1, 3, 16, 64, 10000, None) == L.Q35_EINVAL
    assert "dimensions" in L.last_error()
    assert lib.q35_delta_recurrent(16, 16, 16, 16, 16, 16, 1, 3, 16, 128, 100, None) == L.Q35_EINVAL
    assert lib.q35_gqa_decode_attention(16, 16, 16, 16, 0.0625, 16, 1, 8, 3, 256, 512, 16, 1, None) == L.Q35_EINVAL
    assert lib.q35_lm_head_argmax(16, None, 16, 16, 2, 257, 128, 1e-6, 16, 64, None) == L.Q35_EINVAL
    assert "batch" in L.last_error()
    d = L.GemvDesc(weight=16, input=16, out=16, n_out=10, k=100)  # k not a multiple of 8
    assert lib.q35_gemv(C.byref(d), None) == L.Q35_EINVAL


def test_vocab_shard_entry_points_validate_on_host():
    lib = L.load()
    ws = lib.q35_lm_shard_workspace_size()
    assert ws >= 8 * 8 + 4
    args = dict(hidden=16, batch=2, norm=None, weight=16, row0=0, rows=100, vocab=248320, k=2048, eps=1e-6,
                keys=16, ws=16, ws_bytes=ws, stream=None)

    def call(**kw):
        a = {**args, **kw}
        return lib.q35_lm_head_shard_keys(a["hidden"], a["batch"], a["norm"], a["weight"], a["row0"], a["rows"],
                                          a["vocab"], a["k"], a["eps"], a["keys"], a["ws"], a["ws_bytes"], a["stream"])

    assert call(hidden=None) == L.Q35_EINVAL
    assert call(batch=0) == L.Q35_EINVAL and call(batch=9) == L.Q35_EINVAL
    assert "batch" in L.last_error()
    assert call(k=1024) == L.Q35_EINVAL and "hidden size" in L.last_error()
    assert call(row0=248300, rows=100) == L.Q35_EINVAL and "outside the vocabulary" in L.last_error()
    assert call(ws_bytes=ws - 1) == L.Q35_EINVAL and "workspace" in L.last_error()
    assert call(hidden=18) == L.Q35_EINVAL and "alignment" in L.last_error()
    assert lib.q35_lm_keys_to_tokens(None, 1, 16, None) == L.Q35_EINVAL
    assert lib.q35_lm_keys_to_tokens(16, 0, 16, None) == L.Q35_EINVAL
    assert lib.q35_decoder_decode_layers(None, None) == L.Q35_EINVAL
    assert lib.q35_decoder_finish_step(None, 16, 0, None) == L.Q35_EINVAL
    assert lib.q35_decoder_hidden(None) is None


def test_workspace_size_queries():
    lib = L.load()
    assert lib.q35_lm_head_workspace_size(1) >= 12
    small = lib.q35_gqa_decode_workspace_size(1, 8, 2, 256, 512)
    big = lib.q35_gqa_decode_workspace_size(8, 8, 2, 256, 16384)
    assert 0 < small and small <= big
    assert lib.q35_a8w8_linear_workspace_size(7, 2048) >= 7 * 2048 + 7 * 4


def test_decoder_workspace_size_is_positive():
    from ppu_b200.config import Qwen35Dims

    d = Qwen35Dims()
    desc = L.DecoderDesc()
    desc.n_layers, desc.hidden, desc.intermediate, desc.vocab = d.layers, d.hidden, d.intermediate, d.vocab
    desc.q_heads, desc.kv_heads, desc.head_dim, desc.rotary_dim = d.q_heads, d.kv_heads, d.head_dim, d.rotary_dim
    desc.lin_heads, desc.lin_dk, desc.lin_dv, desc.conv_kernel = d.lin_heads, d.lin_dk, d.lin_dv, d.conv_kernel
    desc.delta_rows, desc.max_len, desc.max_prefill = d.delta_rows, 1152, 1024
    size = L.load().q35_decoder_workspace_size(C.byref(desc))
    assert 50 << 20 < size < 400 << 20


def test_python_mirror_rejects_cpu_tensors_like_the_reference():
    import torch

    from ppu_b200 import kernels as K

    x = torch.zeros(2, 2048, dtype=torch.bfloat16)
    w = torch.zeros(2048, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        K.rms_norm(x, w)
    with pytest.raises(ValueError):
        K.ppu_swiglu_gemv(torch.zeros(1, 2, 64, dtype=torch.bfloat16), torch.zeros(128, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        K.lm_head_argmax(torch.zeros(2, 128, dtype=torch.bfloat16), torch.zeros(10, 128, dtype=torch.bfloat16))
