"""Vocab-sharded LM head on the GPU, through the C ABI.

* ``q35_lm_head_shard_keys`` over the full 248320 x 2048 table, split into 1, 2, 3 and 8 shards
  for 1-8 hiddens: the reduced keys give exactly the single-GPU head's token
  (``q35_lm_head_argmax``), and the logit a key carries is bit-identical to the decode GEMV's
  BF16 logit for that row; the tokens match the oracle up to a BF16 tie;
* ties planted across shard boundaries go to the lowest index; empty shards give INT64_MIN;
* the decoder's split step (``decode_layers`` + shard keys + ``finish_step``) emits the tokens of
  ``decode_step`` and advances the counters the same way;
* lock-step decode of two requests, emulated on one GPU (two engines, the exchange done with
  ``torch.stack`` / ``max``), emits each request's solo tokens;
* with two or more GPUs: the same over NCCL (``ShardedDecode``, eager and CUDA-graph steps).
"""

import os
import socket
import struct

import pytest
import torch
import torch.multiprocessing as mp

from oracle import ops as O
from ppu_b200 import kernels as K
from ppu_b200 import lib as L
from ppu_b200 import vocab_shard as VS
from ppu_b200.config import Qwen35Dims
from ppu_b200.engine import Qwen35Engine
from ppu_b200.synthetic import make_prompt, make_weights

from .helpers import randn

pytestmark = pytest.mark.gpu
DEV = "cuda"
VOCAB, HID = 248320, 2048
SMALL = Qwen35Dims(layers=4, vocab=8192)


def cu(t):
    return t.to(DEV)


def key_logit(key: int) -> float:
    """The FP32 logit a shard key carries (inverse of the order-preserving map)."""
    order = ((key + (1 << 63)) >> 32) & 0xFFFFFFFF
    bits = order & 0x7FFFFFFF if order & 0x80000000 else (~order) & 0xFFFFFFFF
    return struct.unpack("<f", struct.pack("<I", bits))[0]


def sharded_keys(h, e, nw, world):
    keys = []
    for r in range(world):
        a, b = VS.shard_range(e.shape[0], world, r)
        keys.append(K.lm_head_shard_keys(h, e[a:b], a, e.shape[0], norm_weight=nw))
    return torch.stack(keys)


@pytest.fixture(scope="module")
def table():
    h = randn(8, HID, seed=21)
    nw = randn(HID, seed=22, scale=0.02)
    e = randn(VOCAB, HID, seed=23, scale=0.02)
    return h, nw, e, cu(h), cu(nw), cu(e)


@pytest.mark.parametrize("n", [1, 2, 3, 8])
def test_shard_keys_give_the_single_gpu_token(table, n):
    h, nw, e, hd, nwd, ed = table
    single = [int(K.lm_head_argmax(hd[b:b + 1].contiguous(), ed, norm_weight=nwd)) for b in range(n)]
    for world in (1, 2, 3, 8):
        keys = sharded_keys(hd[:n].contiguous(), ed, nwd, world)
        tokens = K.lm_keys_to_tokens(keys.max(0).values.contiguous()).cpu().tolist()
        assert tokens == single, (world, tokens, single)
    hn = O.rms_norm(h[:n], nw)
    want = O.lm_head_argmax(hn, e).reshape(-1).tolist()
    logits = O.linear(hn, e).float()
    for b in range(n):  # the oracle's top-1, or an equal BF16 logit at a higher index
        if single[b] != want[b]:
            assert logits[b, single[b]] == logits[b, want[b]] and single[b] > want[b]


def test_key_logits_are_the_decode_gemv_logits(table):
    _, _, _, hd, nwd, ed = table
    n = 4
    keys = sharded_keys(hd[:n].contiguous(), ed, nwd, 8)
    for b in range(n):
        logits = K.fused_gemv(ed, hd[b], prologue=L.PRO_NORM, epilogue=L.EPI_STORE, norm_weight=nwd).float().cpu()
        for r in range(8):
            a, z = VS.shard_range(VOCAB, 8, r)
            part = logits[a:z]
            best = int(torch.nonzero(part == part.max())[0, 0])
            key = int(keys[r, b])
            assert 0xFFFFFFFF - ((key + (1 << 63)) & 0xFFFFFFFF) == a + best
            assert key_logit(key) == float(part[best])


def test_ties_across_shards_and_empty_shards(table):
    _, _, _, hd, nwd, ed = table
    tok = int(K.lm_head_argmax(hd[:1].contiguous(), ed, norm_weight=nwd))
    e2 = ed.clone()
    e2[VOCAB - 1] = e2[tok]
    e2[5] = e2[tok]
    for world in (2, 8):
        keys = sharded_keys(hd[:2].contiguous(), e2, nwd, world).max(0).values.contiguous()
        assert int(K.lm_keys_to_tokens(keys)[0]) == min(5, tok)
    empty = K.lm_head_shard_keys(hd[:3].contiguous(), ed[:0], 0, VOCAB, norm_weight=nwd)
    assert empty.cpu().tolist() == [O.INT64_MIN] * 3
    assert int(K.lm_keys_to_tokens(empty)[0]) == 0
    with pytest.raises(ValueError):
        K.lm_head_shard_keys(hd[:1].contiguous(), ed[:10], VOCAB - 5, VOCAB)  # shard past the vocabulary
    with pytest.raises(ValueError):
        K.lm_head_shard_keys(hd.repeat(2, 1).contiguous(), ed[:10], 0, VOCAB)  # 16 hiddens > 8


def _engine(seed=0):
    w = make_weights(SMALL, seed=seed, device=DEV)
    return Qwen35Engine(w, SMALL, max_len=256, max_prefill=64, device=DEV)


def _solo_tokens(eng, steps):
    out = []
    for _ in range(steps):
        eng.decode_step()
        out.append(int(eng.token))
    return out


def test_decoder_split_step_matches_decode_step():
    eng = _engine()
    eng.prefill(make_prompt(SMALL, 40, seed=3)[0].to(DEV))
    snap = eng.snapshot()
    log0 = int(eng.log_pos)
    want = _solo_tokens(eng, 12)
    counters = (int(eng.cache_len), int(eng.rope_pos), int(eng.log_pos) - log0)
    eng.restore(snap)
    eng.log_pos.fill_(log0)
    ws = torch.zeros(L.load().q35_lm_shard_workspace_size(), device=DEV, dtype=torch.uint8)
    got = []
    for step in range(12):
        eng.decode_layers()
        h = eng.hidden_view().reshape(1, -1)
        world = 1 + step % 3  # 1, 2 and 3 shards
        keys = []
        for r in range(world):
            a, b = VS.shard_range(SMALL.vocab, world, r)
            keys.append(K.lm_head_shard_keys(h, eng.embed[a:b], a, SMALL.vocab, norm_weight=eng.final_norm,
                                             eps=SMALL.eps, workspace=ws))
        eng.finish_step(torch.stack(keys).max(0).values.contiguous(), 0)
        got.append(int(eng.token))
    assert got == want
    assert (int(eng.cache_len), int(eng.rope_pos), int(eng.log_pos) - log0) == counters
    assert eng.token_log[log0:log0 + 12].cpu().tolist() == want


def test_two_requests_lockstep_on_one_gpu():
    engs = [_engine(), _engine()]
    for i, eng in enumerate(engs):
        eng.prefill(make_prompt(SMALL, 33 + 9 * i, seed=100 + i)[0].to(DEV))
    snaps = [e.snapshot() for e in engs]
    solo = [_solo_tokens(e, 10) for e in engs]
    for e, s in zip(engs, snaps):
        e.restore(s)
    got = [[], []]
    for _ in range(10):
        for e in engs:
            e.decode_layers()
        gathered = torch.stack([e.hidden_view() for e in engs])
        keys = []
        for r in range(2):
            a, b = VS.shard_range(SMALL.vocab, 2, r)
            keys.append(K.lm_head_shard_keys(gathered, engs[r].embed[a:b], a, SMALL.vocab,
                                             norm_weight=engs[r].final_norm, eps=SMALL.eps))
        reduced = torch.stack(keys).max(0).values.contiguous()
        for i, e in enumerate(engs):
            e.finish_step(reduced, i)
            got[i].append(int(e.token))
    assert got == solo


# ------------------------------------------------------------------ NCCL, two or more GPUs
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank: int, world: int, port: int, out) -> None:
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "NCCL_NVLS_ENABLE": "0"})
    from datetime import timedelta

    import torch.distributed as dist

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
        w = make_weights(SMALL, seed=0, device=dev)
        eng = Qwen35Engine(w, SMALL, max_len=256, max_prefill=64, device=dev)
        sd = VS.ShardedDecode(eng)
        eng.prefill(make_prompt(SMALL, 30 + 7 * rank, seed=200 + rank)[0].to(dev))
        snap = eng.snapshot()
        solo = []
        for _ in range(8):
            eng.decode_step()
            solo.append(int(eng.token))
        eng.restore(snap)
        eager = []
        for _ in range(4):
            sd.step()
            eager.append(int(eng.token))
        g = sd.capture(1)
        for _ in range(4):
            g.replay()
            eager.append(int(eng.token))
        toks, _, _ = sd.generate(make_prompt(SMALL, 30 + 7 * rank, seed=200 + rank)[0], 9)
        torch.cuda.synchronize()
        sd.release()
        del g
        dist.barrier()
        dist.destroy_process_group()
        out.put((rank, solo, eager, toks[1:]))
    except Exception as e:  # reported to the parent instead of leaving it waiting
        out.put((rank, "error", repr(e), None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_lockstep_two_ranks():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((out.get(timeout=300) for _ in range(2)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, solo, eager, gen in res:
        assert solo != "error", (rank, eager)
        assert eager == solo, (rank, eager, solo)
        assert gen == solo, (rank, gen, solo)
