"""Vocab-sharded LM head for lock-step greedy decode, one request per rank.

The LM head is the largest single read of a decode step: the tied ``[248320, 2048]`` embedding,
1017 MB, streamed once per token (kernels.py:1093-1185 has it as one batch-1 GEMV with a fused
top-1). With N ranks decoding in lock step, rank r streams only rows ``shard_range(V, N, r)`` and
serves every rank's request from that read:

1. ``decode_layers``: the 24 layers of its own request; the final residual stays on the device;
2. ``all_gather`` (NCCL) of the N final residuals, 4 KB each;
3. ``q35_lm_head_shard_keys``: the final RMSNorm and the GEMV of all N hiddens against the shard,
   one signed 64-bit key per request, ``(order(bf16 logit) << 32 | (0xFFFFFFFF - index)) - 2^63``;
4. ``all_reduce`` with MAX (NCCL, int64) of the N keys: the largest logit, lowest index on ties;
5. ``finish_step``: the token its own key encodes goes to the decoder's token slot; the step
   counters advance.

The logits are bit-identical to the single-GPU head's, so every rank emits exactly the tokens it
would emit alone. All ranks take the same collective steps in the same order: a rank whose
request has ended keeps stepping until the others are done (``generate`` runs a fixed count).
Data moves only through NCCL into local buffers (no peer loads, no multicast).
"""

from __future__ import annotations

import time

import torch
import torch.distributed as dist

from . import kernels as K
from . import lib as L

MAX_RANKS = 8  # the shard kernel serves at most 8 hiddens per launch


def shard_range(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """Rows ``[start, stop)`` of the vocabulary owned by ``rank``: contiguous, sizes differing by
    at most one row, the larger shards first (248320 rows over 8 ranks: 31040 each)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if vocab < 0:
        raise ValueError("vocab must be non-negative")
    base, extra = divmod(vocab, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def reduce_keys(keys: torch.Tensor, group=None) -> torch.Tensor:
    """In-place maximum of the int64 shard keys over the ranks of ``group`` (the exchange step)."""
    if keys.dtype != torch.int64:
        raise ValueError("shard keys are int64")
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
    return keys


class ShardedDecode:
    """Lock-step decode of one request per rank over ``engine`` with the LM head vocab-sharded.
    Constructing it is a collective (every rank of ``group`` constructs one).

    ``step()`` replaces ``engine.decode_step()``; ``capture()`` records steps, collectives included,
    into a CUDA graph (release it before the process group is destroyed)."""

    def __init__(self, engine, group=None):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("ShardedDecode needs an initialised process group")
        if engine.persistent:
            raise ValueError("the vocab-sharded step runs on the per-op decode path (persistent=False)")
        self.engine = engine
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks share one shard launch (got {self.world})")
        vocab, hidden = engine.embed.shape
        self.vocab = vocab
        self.row0, self.row1 = shard_range(vocab, self.world, self.rank)
        self.shard = engine.embed[self.row0:self.row1]
        dev = engine.device
        self.hidden = engine.hidden_view()
        self.gathered = torch.empty(self.world, hidden, device=dev, dtype=torch.bfloat16)
        self.keys = torch.empty(self.world, device=dev, dtype=torch.int64)
        self.workspace = torch.zeros(max(L.load().q35_lm_shard_workspace_size(), 16), device=dev,
                                     dtype=torch.uint8)
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        # collective: every rank constructs its ShardedDecode; the communicator is set up here,
        # before any step is captured into a CUDA graph
        reduce_keys(torch.zeros(self.world, device=dev, dtype=torch.int64), group)
        torch.cuda.synchronize(dev)

    def step(self) -> torch.Tensor:
        """One lock-step decode step (every rank must call it); returns the engine's token slot."""
        eng = self.engine
        eng.decode_layers()
        dist.all_gather_into_tensor(self.gathered, self.hidden, group=self.group)
        K.lm_head_shard_keys(self.gathered, self.shard, self.row0, self.vocab, norm_weight=eng.final_norm,
                             eps=eng.dims.eps, workspace=self.workspace, out=self.keys)
        reduce_keys(self.keys, self.group)
        return eng.finish_step(self.keys, self.rank)

    def capture(self, steps: int = 1) -> torch.cuda.CUDAGraph:
        """CUDA graph of ``steps`` lock-step decode steps (all ranks capture the same count)."""
        if steps in self._graphs:
            return self._graphs[steps]
        dev = self.engine.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                for _ in range(steps):
                    self.step()
        torch.cuda.current_stream(dev).wait_stream(side)
        self._graphs[steps] = g
        return g

    def release(self) -> None:
        """Drops the captured graphs (they hold NCCL work: release before destroy_process_group)."""
        self._graphs.clear()

    def generate(self, prompt_ids, max_new_tokens: int, *, eos_ids=(), use_graph: bool = True):
        """``Qwen35Engine.generate`` in lock step: host prompt, local prefill, first token read on
        the host (TTFT), then ``max_new_tokens - 1`` sharded steps on every rank with a host read of
        each token; tokens after this rank's EOS are stepped but not returned. Returns
        ``(tokens, ttft_s, elapsed_s)``."""
        eng = self.engine
        eos = set(int(e) for e in eos_ids)
        host = torch.as_tensor(prompt_ids, dtype=torch.int64).reshape(-1)
        if not host.is_pinned():
            host = host.pin_memory()
        start = time.perf_counter()
        eng.prefill(host.to(eng.device, non_blocking=True))
        tokens = [int(eng.token.item())]
        first_at = time.perf_counter()
        graph = self.capture(1) if (use_graph and max_new_tokens > 1) else None
        done = tokens[-1] in eos
        for _ in range(max_new_tokens - 1):
            if graph is not None:
                graph.replay()
            else:
                self.step()
            t = int(eng.token.item())
            if not done:
                tokens.append(t)
                done = t in eos
        end = time.perf_counter()
        return tokens, first_at - start, end - start
