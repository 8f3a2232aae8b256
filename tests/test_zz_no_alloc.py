"""The allocation-free decode attention entry point, through the C ABI.

Some callers cannot allocate device memory at the moment they call in (a locked or pool-only
allocator, a host thread that must not touch the CUDA allocator, a runtime that hands over only
its inputs and outputs). ``q35_gqa_decode_attention_noalloc`` serves them with scratch in a static
device array. This file is collected last on purpose: it must pass both alone and after the rest
of the suite, and its output must match the workspace-taking entry point on consecutive calls.
"""

import ctypes as C

import pytest
import torch

from ppu_b200 import lib as L

pytestmark = pytest.mark.gpu


def _workspace_call(q, k, v, n_valid, out):
    lib = L.load()
    b, h, _, d = q.shape
    kvh, cache_len = k.shape[1], k.shape[2]
    size = lib.q35_gqa_decode_workspace_size(b, h, kvh, d, cache_len)
    ws = torch.zeros(size, device=q.device, dtype=torch.uint8)
    L.call("q35_gqa_decode_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), n_valid.data_ptr(), 0.0625,
           out.data_ptr(), b, h, kvh, d, cache_len, ws.data_ptr(), size, L.stream_of(q.device))


def _noalloc_call(q, k, v, n_valid, out):
    b, h, _, d = q.shape
    return L.load().q35_gqa_decode_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), n_valid.data_ptr(),
                                                      C.c_float(0.0625), out.data_ptr(), b, h, k.shape[1], d,
                                                      k.shape[2], L.stream_of(q.device))


@pytest.mark.parametrize("batch,cache_len,kv_heads", [(1, 1152, 2), (8, 4096, 2), (2, 2048, 8), (4, 1024, 4)],
                         ids=["b1-g4", "b8-g4", "b2-g1", "b4-g2"])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(batch, cache_len, kv_heads):
    g = torch.Generator(device="cuda").manual_seed(batch * 131 + cache_len + kv_heads)
    q = torch.randn(batch, 8, 1, 256, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(batch, kv_heads, cache_len, 256, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(batch, kv_heads, cache_len, 256, device="cuda", generator=g).to(torch.bfloat16)
    for n in (cache_len - 5, 37):  # two calls in a row; the array keeps the previous call's contents
        n_valid = torch.tensor([n], device="cuda", dtype=torch.int64)
        want = torch.empty(batch, 1, 8 * 256, device="cuda", dtype=torch.bfloat16)
        got = torch.full_like(want, float("nan"))
        _workspace_call(q, k, v, n_valid, want)
        assert _noalloc_call(q, k, v, n_valid, got) == L.Q35_OK, L.last_error()
        torch.cuda.synchronize()
        # same kernel and split plan on the same inputs: identical results (tolerance 0)
        assert torch.equal(got, want)


def test_noalloc_rejects_shapes_beyond_its_static_scratch():
    lib = L.load()
    limit = lib.q35_gqa_decode_noalloc_max_bytes()
    assert limit == 2 << 20
    b, h, kvh, n = 64, 64, 64, 1024  # 64 x 64 split partials of 1 KB: 4 MiB of scratch
    assert lib.q35_gqa_decode_workspace_size(b, h, kvh, 256, n) > limit
    q = torch.zeros(b, h, 1, 256, device="cuda", dtype=torch.bfloat16)
    n_valid = torch.ones(1, device="cuda", dtype=torch.int64)
    out = torch.empty(b, 1, h * 256, device="cuda", dtype=torch.bfloat16)
    # the size check fails on the host before any launch
    rc = lib.q35_gqa_decode_attention_noalloc(q.data_ptr(), q.data_ptr(), q.data_ptr(), n_valid.data_ptr(),
                                              C.c_float(0.0625), out.data_ptr(), b, h, kvh, 256, n,
                                              L.stream_of(q.device))
    assert rc == L.Q35_EINVAL and "static maximum" in L.last_error()


def test_noalloc_rejects_more_split_tickets_than_its_scratch_holds():
    lib = L.load()
    b, h, kvh, n = 64, 5, 5, 64  # 320 (batch x kv_heads) tickets, 256 fit; the scratch itself is small
    assert lib.q35_gqa_decode_workspace_size(b, h, kvh, 256, n) <= lib.q35_gqa_decode_noalloc_max_bytes()
    q = torch.zeros(b, h, 1, 256, device="cuda", dtype=torch.bfloat16)
    kv = torch.zeros(b, kvh, n, 256, device="cuda", dtype=torch.bfloat16)
    n_valid = torch.ones(1, device="cuda", dtype=torch.int64)
    out = torch.empty(b, 1, h * 256, device="cuda", dtype=torch.bfloat16)
    rc = lib.q35_gqa_decode_attention_noalloc(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), n_valid.data_ptr(),
                                              C.c_float(0.0625), out.data_ptr(), b, h, kvh, 256, n,
                                              L.stream_of(q.device))
    assert rc == L.Q35_EINVAL and "ticket" in L.last_error()
