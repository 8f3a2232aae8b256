"""Host logic of the vocab-sharded LM head (lock-step decode), on CPU: the shard partition, the
64-bit key packing of the oracle restatement reduced to the full-vocabulary top-1 (ties across
shard boundaries, negative and signed-zero logits, empty shards), and the exchange step itself
(``reduce_keys``, an int64 MAX all-reduce) across gloo ranks at world sizes 2 and 3."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import ops as O
from ppu_b200 import vocab_shard as VS


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(n=3, vocab=1000, k=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(n, k, generator=g).to(torch.bfloat16)
    w = torch.randn(vocab, k, generator=g).to(torch.bfloat16)
    return h, w


def _sharded_tokens(h, w, world):
    keys = []
    for r in range(world):
        a, b = VS.shard_range(w.shape[0], world, r)
        keys.append(O.lm_shard_keys(h, w[a:b], a))
    return O.lm_keys_to_tokens(torch.stack(keys).max(0).values)


@pytest.mark.parametrize("vocab,world", [(248320, 8), (248320, 2), (1000, 3), (7, 8), (0, 2), (5, 1)])
def test_shard_range_partitions_the_vocabulary(vocab, world):
    ranges = [VS.shard_range(vocab, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == vocab
    for (a0, b0), (a1, b1) in zip(ranges, ranges[1:]):
        assert b0 == a1 and b0 - a0 >= b1 - a1
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1
    if vocab == 248320 and world == 8:
        assert sizes == [31040] * 8
    with pytest.raises(ValueError):
        VS.shard_range(vocab, world, world)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_keys_reduce_to_full_top1(world):
    h, w = _case()
    assert torch.equal(_sharded_tokens(h, w, world), O.lm_head_argmax(h, w).reshape(-1))


def test_ties_across_shards_take_the_lowest_index():
    h, w = _case(n=2)
    want = O.lm_head_argmax(h, w).reshape(-1)
    for b in range(2):
        w2 = w.clone()
        w2[990] = w2[int(want[b])]  # same logit in the last shard
        w2[3] = w2[int(want[b])]    # ... and in the first
        for world in (2, 4, 8):
            assert int(_sharded_tokens(h, w2, world)[b]) == 3


def test_negative_zero_and_empty_shards():
    k = 64
    h = torch.ones(1, k, dtype=torch.bfloat16)
    w = -torch.ones(5, k, dtype=torch.bfloat16)  # all logits negative: -64
    w[3] = -0.5
    assert int(_sharded_tokens(h, w, 8)[0]) == 3  # 3 of the 8 shards are empty
    z = torch.zeros(4, k, dtype=torch.bfloat16)
    z[2, 0], z[2, 1] = 1.0, -1.0  # +0 logits everywhere (row 2 sums to +0 exactly)
    assert int(_sharded_tokens(h, z, 2)[0]) == 0
    assert int(O.lm_keys_to_tokens(torch.tensor([O.INT64_MIN]))[0]) == 0
    assert O.float_order_key(-0.0) == O.float_order_key(0.0)
    assert O.float_order_key(-1.0) < O.float_order_key(-0.5) < O.float_order_key(0.0) < O.float_order_key(1e-30)


def _worker(rank: int, world: int, port: int, out) -> None:
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import torch.distributed as dist
    from datetime import timedelta

    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    h, w = _case(n=world, vocab=997, seed=5)
    w[996] = w[int(O.lm_head_argmax(h[:1], w)[0, 0])]  # a tie for request 0 in the last shard
    a, b = VS.shard_range(w.shape[0], world, rank)
    keys = O.lm_shard_keys(h, w[a:b], a)
    VS.reduce_keys(keys)
    out.put((rank, O.lm_keys_to_tokens(keys).tolist(), O.lm_head_argmax(h, w).reshape(-1).tolist()))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_reduce_keys_across_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((out.get(timeout=120) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for _, got, want in res:
        assert got == want  # every rank holds every request's token after the exchange


def test_reduce_keys_single_process_and_dtype_guard():
    k = torch.tensor([5, -3], dtype=torch.int64)
    assert VS.reduce_keys(k) is k and k.tolist() == [5, -3]
    with pytest.raises(ValueError):
        VS.reduce_keys(torch.zeros(2, dtype=torch.int32))


def test_sharded_decode_needs_a_process_group():
    with pytest.raises(RuntimeError):
        VS.ShardedDecode(object())
