"""Device-resident Qwen3.5 text decoder driven through the C ABI decoder loop.

``Qwen35Engine`` packs a Hugging Face-named weight dict the way qwen35_fused/integration.py
packs the model (integration.py:69-140: [qkv|z|a|b] for DeltaNet, [Q|gate..|K|V] for attention,
[gate; up] for the MLP), optionally quantises the M/F/L projection groups to A8W8 with the CUDA
quantiser, allocates the static KV cache, DeltaNet conv/recurrent states and one workspace, and
creates a ``q35_decoder``. Prefill and each greedy decode step are single C calls on the current
stream; ``capture`` records decode steps into a CUDA graph (qwen35_fused/graph.py). The decode
step is the per-op step (5 kernels per layer + LM head), or with ``persistent=True`` the
one-kernel persistent step (bf16, 2B shapes).
"""

from __future__ import annotations

import ctypes as C
import time

import torch

from . import lib as L
from .config import Qwen35Dims

BF16 = torch.bfloat16


def rope_inv_freq(rotary_dim: int, theta: float) -> torch.Tensor:
    """HF Qwen3_5TextRotaryEmbedding.compute_default_rope_parameters, in FP32."""
    exponent = torch.arange(0, rotary_dim, 2, dtype=torch.int64).to(torch.float32) / rotary_dim
    return 1.0 / (theta ** exponent)


def cache_bucket(input_len: int, max_new_tokens: int) -> int:
    """Static-cache length bucket of evaluation_wrapper.py:340-341."""
    need = input_len + max_new_tokens + 1
    return max(512, (need + 127) // 128 * 128)


class Qwen35Engine:
    def __init__(self, weights: dict, dims: Qwen35Dims = Qwen35Dims(), *, a8w8: bool = False,
                 max_len: int = 2048, max_prefill: int = 1024, device="cuda", use_pdl: bool = True,
                 prefill_tc: bool = True, prefill_chunked: bool = True, log_len: int = 4096, release_source: bool = False,
                 persistent: bool | None = None, batch: int = 1):
        L.load()
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("Qwen35Engine runs on a CUDA device only")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if not 1 <= batch <= 8:
            raise ValueError("batch must be within [1, 8]")
        if batch > 1 and a8w8:
            raise ValueError("batched decoding runs bf16 weights (the A8W8 decode path is batch 1)")
        self.dims = dims
        self.device = dev
        self.a8w8 = a8w8
        self.batch = batch
        self.max_len = max_len
        # prefill rows: one prompt shorter than the cache, or (batched) one per slot
        self.max_prefill = min(max_prefill, (max_len - 1) * batch)
        self._keep: list[torch.Tensor] = []

        def w(name):
            t = weights[name]
            if release_source:
                weights[name] = None
            return t.to(device=dev, dtype=BF16).contiguous()

        d = dims
        self.layer_descs = (L.LayerDesc * d.layers)()
        self.conv_states, self.rec_states, self.k_caches, self.v_caches = [], [], [], []
        self.layer_tensors = []
        for i, kind in enumerate(d.layer_types):
            p = f"model.layers.{i}."
            T: dict[str, torch.Tensor] = {
                "in_ln": w(p + "input_layernorm.weight"),
                "post_ln": w(p + "post_attention_layernorm.weight"),
                "gate_up": torch.cat((w(p + "mlp.gate_proj.weight"), w(p + "mlp.up_proj.weight")), 0).contiguous(),
                "down": w(p + "mlp.down_proj.weight"),
            }
            ld = self.layer_descs[i]
            if kind == "linear_attention":
                la = p + "linear_attn."
                packed = torch.cat((w(la + "in_proj_qkv.weight"), w(la + "in_proj_z.weight"),
                                    w(la + "in_proj_a.weight"), w(la + "in_proj_b.weight")), 0)
                pad = d.delta_rows - packed.shape[0]
                if pad:
                    packed = torch.cat((packed, packed.new_zeros(pad, packed.shape[1])), 0)
                T["mix_in"] = packed.contiguous()
                T["mix_out"] = w(la + "out_proj.weight")
                T["conv_w"] = w(la + "conv1d.weight").reshape(d.conv_dim, d.conv_kernel).contiguous()
                T["a_log"] = w(la + "A_log")
                T["dt_bias"] = w(la + "dt_bias")
                T["gnorm"] = w(la + "norm.weight")
                T["conv_state"] = torch.zeros(batch, d.conv_dim, d.conv_kernel, device=dev, dtype=BF16)
                T["rec_state"] = torch.zeros(batch, d.lin_heads, d.lin_dk, d.lin_dv, device=dev, dtype=torch.float32)
                self.conv_states.append(T["conv_state"])
                self.rec_states.append(T["rec_state"])
                ld.kind = 0
            else:
                sa = p + "self_attn."
                T["mix_in"] = torch.cat((w(sa + "q_proj.weight"), w(sa + "k_proj.weight"),
                                         w(sa + "v_proj.weight")), 0).contiguous()
                T["mix_out"] = w(sa + "o_proj.weight")
                T["q_norm"] = w(sa + "q_norm.weight")
                T["k_norm"] = w(sa + "k_norm.weight")
                T["k_cache"] = torch.zeros(batch, d.kv_heads, max_len, d.head_dim, device=dev, dtype=BF16)
                T["v_cache"] = torch.zeros_like(T["k_cache"])
                self.k_caches.append(T["k_cache"])
                self.v_caches.append(T["v_cache"])
                ld.kind = 1
            if a8w8:
                for key in ("mix_in", "mix_out", "gate_up", "down"):
                    q, s = self._quantize(T[key])
                    T[key] = q
                    T[key + "_scale"] = s
            for key in ("in_ln", "post_ln", "mix_in", "mix_out", "gate_up", "down", "conv_w", "a_log", "dt_bias",
                        "gnorm", "conv_state", "rec_state", "q_norm", "k_norm", "k_cache", "v_cache",
                        "mix_in_scale", "mix_out_scale", "gate_up_scale", "down_scale"):
                if key in T:
                    setattr(ld, key, T[key].data_ptr())
            self.layer_tensors.append(T)
        self.embed = w("model.embed_tokens.weight")
        self.final_norm = w("model.norm.weight")
        self.inv_freq = rope_inv_freq(d.rotary_dim, d.rope_theta).to(dev)
        self.token = torch.zeros(batch, device=dev, dtype=torch.int64)
        self.cache_len = torch.zeros(1, device=dev, dtype=torch.int64)
        self.rope_pos = torch.zeros(1, device=dev, dtype=torch.int64)
        self.log_len = log_len
        self.token_log = torch.zeros(max(log_len, 1), device=dev, dtype=torch.int64)
        self.log_pos = torch.zeros(1, device=dev, dtype=torch.int64)

        desc = L.DecoderDesc()
        desc.n_layers, desc.hidden, desc.intermediate, desc.vocab = d.layers, d.hidden, d.intermediate, d.vocab
        desc.q_heads, desc.kv_heads, desc.head_dim, desc.rotary_dim = d.q_heads, d.kv_heads, d.head_dim, d.rotary_dim
        desc.lin_heads, desc.lin_dk, desc.lin_dv = d.lin_heads, d.lin_dk, d.lin_dv
        desc.conv_kernel, desc.delta_rows = d.conv_kernel, d.delta_rows
        desc.max_len, desc.max_prefill, desc.a8w8, desc.eps = max_len, self.max_prefill, int(a8w8), d.eps
        desc.layers = self.layer_descs
        desc.embed, desc.final_norm, desc.inv_freq = self.embed.data_ptr(), self.final_norm.data_ptr(), \
            self.inv_freq.data_ptr()
        desc.token, desc.cache_len, desc.rope_pos = self.token.data_ptr(), self.cache_len.data_ptr(), \
            self.rope_pos.data_ptr()
        desc.token_log = self.token_log.data_ptr() if log_len > 0 else None
        desc.log_pos = self.log_pos.data_ptr()
        desc.log_len = log_len
        desc.use_pdl = int(use_pdl)
        desc.prefill_tc = int(prefill_tc)
        desc.prefill_delta = 0 if prefill_chunked else 1
        for i, sec in enumerate(d.mrope_section):
            desc.mrope_section[i] = sec
        desc.batch = batch
        size = L.load().q35_decoder_workspace_size(C.byref(desc))
        self.workspace = torch.zeros(size, device=dev, dtype=torch.uint8)
        desc.workspace, desc.workspace_bytes = self.workspace.data_ptr(), size
        self.desc = desc
        handle = C.c_void_p()
        L.check(L.load().q35_decoder_create(C.byref(desc), C.byref(handle)), "q35_decoder_create")
        self.handle = handle
        self.has_persistent = bool(L.load().q35_decoder_has_persistent(handle))
        if persistent and not self.has_persistent:
            raise ValueError("persistent decode step unavailable for this model (A8W8, shapes or device)")
        self.persistent = False if persistent is None else bool(persistent)
        self.kernels_per_step = 1 if self.persistent else L.load().q35_decoder_kernels_per_step(handle)
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                L.load().q35_decoder_destroy(h)
            except Exception:
                pass

    def _quantize(self, w: torch.Tensor):
        q = torch.empty(w.shape, device=w.device, dtype=torch.int8)
        s = torch.empty(w.shape[0], device=w.device, dtype=torch.float32)
        L.call("q35_quantize_rows", w.data_ptr(), q.data_ptr(), s.data_ptr(), w.shape[0], w.shape[1],
               L.stream_of(w.device))
        return q, s

    # ------------------------------------------------------------------ steps
    def prefill(self, ids: torch.Tensor, slot: int = 0) -> torch.Tensor:
        """Prefill device token ids ``[L]`` from an empty cache; the greedy first token lands in
        ``self.token`` (returned, on device). Batched engines: request slot ``slot``; every slot of a
        batch is prefilled with the same length before the batch decodes."""
        ids = ids.reshape(-1)
        if not ids.is_cuda or ids.dtype != torch.int64:
            raise ValueError("prefill expects int64 token ids on a CUDA device")
        if ids.device != self.device:
            ids = ids.to(self.device)
        n = ids.numel()
        if n > min(self.max_prefill, self.max_len - 1):
            raise ValueError(f"prompt of {n} tokens exceeds max_prefill={self.max_prefill} or the cache")
        L.check(L.load().q35_decoder_prefill_slot(self.handle, ids.data_ptr(), n, int(slot), L.stream_of(self.device)),
                "q35_decoder_prefill_slot")
        return self.token

    def prefill_multimodal(self, ids: torch.Tensor, image_embeds: torch.Tensor, image_rows: torch.Tensor,
                           positions3: torch.Tensor, rope_next: int, slot: int = 0) -> torch.Tensor:
        """Prefill an image + text prompt from an empty cache: device ids ``[L]`` (the image rows'
        ids are ignored), ``image_embeds`` bf16 ``[n, hidden]`` placed at rows ``image_rows``
        (int64 ``[n]``), 3-axis M-RoPE ``positions3`` int64 ``[3, L]``; afterwards the decode
        steps continue at RoPE position ``rope_next``. The greedy first token lands in
        ``self.token``."""
        ids = ids.reshape(-1)
        n = ids.numel()
        if not (ids.is_cuda and ids.dtype == torch.int64 and image_rows.dtype == torch.int64
                and positions3.dtype == torch.int64):
            raise ValueError("prefill_multimodal expects int64 ids, image rows and positions on the GPU")
        if n > min(self.max_prefill, self.max_len - 1):
            raise ValueError(f"prompt of {n} tokens exceeds max_prefill={self.max_prefill} or the cache")
        if positions3.shape != (3, n) or image_embeds.dim() != 2 or image_embeds.shape[1] != self.dims.hidden:
            raise ValueError("positions3 must be [3, L] and image_embeds [n, hidden]")
        if image_rows.numel() != image_embeds.shape[0] or image_embeds.dtype != BF16:
            raise ValueError("one image row per bf16 image embedding")
        dev = self.device
        ids, image_rows = ids.to(dev), image_rows.to(dev).contiguous()
        image_embeds, positions3 = image_embeds.to(dev).contiguous(), positions3.to(dev).contiguous()
        L.check(L.load().q35_decoder_prefill_mm(self.handle, ids.data_ptr(), n, image_embeds.data_ptr(),
                                                image_rows.data_ptr(), image_rows.numel(), positions3.data_ptr(),
                                                int(rope_next), int(slot), L.stream_of(dev)), "q35_decoder_prefill_mm")
        return self.token

    def prefill_batch(self, ids: torch.Tensor, *, image_embeds: torch.Tensor | None = None,
                      image_rows: torch.Tensor | None = None, positions3: torch.Tensor | None = None,
                      rope_next: int = -1, slot: int = 0) -> torch.Tensor:
        """Batched engines: prefill ``n`` requests of one length in one pass, device ids
        ``[n, L]`` into slots ``slot .. slot + n - 1`` (``n * L <= max_prefill``). Optional image
        rows as in ``prefill_multimodal``, with ``image_rows`` indexing the ``n * L`` rows and
        ``positions3`` int64 ``[3, n, L]``. The first tokens land in ``self.token[slot:slot + n]``."""
        if ids.dim() != 2 or not ids.is_cuda or ids.dtype != torch.int64:
            raise ValueError("prefill_batch expects int64 token ids [n, L] on a CUDA device")
        nseq, n = ids.shape
        if nseq * n > self.max_prefill:
            raise ValueError(f"{nseq} x {n} prompt tokens exceed max_prefill={self.max_prefill}")
        dev = self.device
        ids = ids.to(dev).contiguous()
        emb_p = rows_p = pos_p = None
        n_img = 0
        if image_embeds is not None:
            if image_rows is None or image_rows.numel() != image_embeds.shape[0] or image_embeds.dtype != BF16 \
                    or image_embeds.dim() != 2 or image_embeds.shape[1] != self.dims.hidden:
                raise ValueError("one int64 image row per bf16 image embedding [n, hidden]")
            image_embeds, image_rows = image_embeds.to(dev).contiguous(), image_rows.to(dev).contiguous()
            emb_p, rows_p, n_img = image_embeds.data_ptr(), image_rows.data_ptr(), image_rows.numel()
        if positions3 is not None:
            if positions3.shape != (3, nseq, n) or positions3.dtype != torch.int64:
                raise ValueError("positions3 must be int64 [3, n, L]")
            positions3 = positions3.to(dev).contiguous()
            pos_p = positions3.data_ptr()
        L.check(L.load().q35_decoder_prefill_batch(self.handle, ids.data_ptr(), n, nseq, emb_p, rows_p, n_img, pos_p,
                                                   int(rope_next), int(slot), L.stream_of(dev)),
                "q35_decoder_prefill_batch")
        return self.token

    def decode_step(self) -> torch.Tensor:
        """One greedy decode step on the current stream (reads/writes ``self.token``)."""
        if self.persistent:
            L.check(L.load().q35_decoder_decode_step_persistent(self.handle, L.stream_of(self.device)),
                    "q35_decoder_decode_step_persistent")
        else:
            L.check(L.load().q35_decoder_decode_step(self.handle, L.stream_of(self.device)),
                    "q35_decoder_decode_step")
        return self.token

    # ---- the step split for a vocab-sharded LM head (ppu_b200.vocab_shard)
    def decode_layers(self) -> None:
        """The decode step's layers only: the final residual lands in ``hidden_view()``; no token
        is written and the step counters stay put until ``finish_step``."""
        L.check(L.load().q35_decoder_decode_layers(self.handle, L.stream_of(self.device)),
                "q35_decoder_decode_layers")

    def hidden_view(self) -> torch.Tensor:
        """The decoder's final-residual buffer (``[hidden]`` BF16, pre final norm) as a tensor view."""
        ptr = L.load().q35_decoder_hidden(self.handle)
        off = (ptr or 0) - self.workspace.data_ptr()
        nbytes = 2 * self.dims.hidden
        if ptr is None or off < 0 or off + nbytes > self.workspace.numel():
            raise RuntimeError("decoder hidden buffer lies outside the engine workspace")
        return self.workspace[off:off + nbytes].view(BF16)

    def finish_step(self, keys: torch.Tensor, index: int) -> torch.Tensor:
        """Completes a ``decode_layers`` step from reduced shard keys: the token ``keys[index]``
        encodes goes to ``self.token`` (and the token log), and the counters advance."""
        if keys.dtype != torch.int64 or keys.device != self.device or not keys.is_contiguous():
            raise ValueError("keys must be a contiguous int64 tensor on the engine's device")
        if not 0 <= index < keys.numel():
            raise ValueError(f"key index {index} outside [0, {keys.numel()})")
        L.check(L.load().q35_decoder_finish_step(self.handle, keys.data_ptr(), index, L.stream_of(self.device)),
                "q35_decoder_finish_step")
        return self.token

    def capture(self, steps: int = 1) -> torch.cuda.CUDAGraph:
        """CUDA graph of ``steps`` consecutive decode steps (graph.py:50-79)."""
        if steps in self._graphs:
            return self._graphs[steps]
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                for _ in range(steps):
                    self.decode_step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        self._graphs[steps] = g
        return g

    def _persistent_op_labels(self) -> list[str]:
        labels = []
        for kind in self.dims.layer_types:
            if kind == "linear_attention":
                labels += ["in_proj+conv", "delta_step", "out_proj(gated norm)", "gate_up", "down"]
            else:
                labels += ["qgkv_proj", "attn_partials", "attn_combine", "o_proj", "gate_up", "down"]
        return labels + ["lm_head"]

    def trace_step(self) -> dict:
        """Runs one persistent decode step with barrier tracing (``q35_decoder_set_trace``) and
        returns, per op, the CTAs' mean / max work time and mean wait at the following grid
        barrier (microseconds), plus the step's wall time on the device. Advances the decoder by
        one token like ``decode_step``."""
        if not self.has_persistent:
            raise ValueError("persistent decode step unavailable for this model")
        n_sm = 148
        n_ops = L.load().q35_decoder_trace_ops(self.handle)
        buf = torch.zeros((n_ops + 1) * n_sm * 2, device=self.device, dtype=torch.int64)
        L.check(L.load().q35_decoder_set_trace(self.handle, buf.data_ptr(), buf.numel()), "q35_decoder_set_trace")
        persistent, self.persistent = self.persistent, True
        try:
            self.decode_step()
            torch.cuda.synchronize(self.device)
        finally:
            self.persistent = persistent
            L.load().q35_decoder_set_trace(self.handle, None, 0)
        t = buf.view(n_ops + 1, n_sm, 2).double().cpu() / 1000.0
        start, end = t[n_ops, :, 0], t[n_ops, :, 1]
        labels = self._persistent_op_labels()
        ops = []
        prev = start
        for j in range(n_ops):
            work = t[j, :, 0] - prev
            wait = t[j, :, 1] - t[j, :, 0]
            ops.append({"op": labels[j] if j < len(labels) else f"op{j}", "work_mean_us": float(work.mean()),
                        "work_max_us": float(work.max()), "wait_mean_us": float(wait.mean())})
            prev = t[j, :, 1]
        return {"step_us": float(end.max() - start.min()), "ops": ops}

    def prefill_probe(self, ids: torch.Tensor) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """A8W8 diagnostic: prefills ``ids`` like ``prefill`` and returns, per A8W8 projection in
        call order (per layer: in-projection, out-projection, gate/up, down), the per-token int8
        codes ``[L, k]`` and FP32 scales ``[L, 1]`` its input was quantised to."""
        if not self.a8w8:
            raise ValueError("prefill_probe needs an A8W8 engine")
        n = ids.numel()
        d = self.dims
        ks = []
        for kind in d.layer_types:
            ks += [d.hidden, d.value_dim if kind == "linear_attention" else d.attn_width, d.hidden, d.intermediate]
        total = sum(n * k + 4 * n for k in ks)
        buf = torch.zeros(total, device=self.device, dtype=torch.uint8)
        lib = L.load()
        L.check(lib.q35_decoder_set_probe(self.handle, buf.data_ptr(), total), "q35_decoder_set_probe")
        try:
            self.prefill(ids)
            torch.cuda.synchronize(self.device)
        finally:
            lib.q35_decoder_set_probe(self.handle, None, 0)
        if lib.q35_decoder_probe_bytes(self.handle) != total:
            raise RuntimeError("prefill probe: unexpected record size")
        out, off = [], 0
        host = buf.cpu()
        for k in ks:
            codes = host[off:off + n * k].view(torch.int8).reshape(n, k)
            off += n * k
            scale = host[off:off + 4 * n].view(torch.float32).reshape(n, 1)
            off += 4 * n
            out.append((codes, scale))
        return out

    # ------------------------------------------------------------------ state
    def snapshot(self) -> dict:
        """Copies of every piece of mutable decoding state (for restoring after warm-up)."""
        return {"conv": [t.clone() for t in self.conv_states], "rec": [t.clone() for t in self.rec_states],
                "k": [t.clone() for t in self.k_caches], "v": [t.clone() for t in self.v_caches],
                "token": self.token.clone(), "cache_len": self.cache_len.clone(), "rope_pos": self.rope_pos.clone()}

    def restore(self, snap: dict) -> None:
        for dst, src in zip(self.conv_states, snap["conv"]):
            dst.copy_(src)
        for dst, src in zip(self.rec_states, snap["rec"]):
            dst.copy_(src)
        for dst, src in zip(self.k_caches, snap["k"]):
            dst.copy_(src)
        for dst, src in zip(self.v_caches, snap["v"]):
            dst.copy_(src)
        self.token.copy_(snap["token"])
        self.cache_len.copy_(snap["cache_len"])
        self.rope_pos.copy_(snap["rope_pos"])

    # ------------------------------------------------------------------ generation
    def generate_batch(self, prompts, max_new_tokens: int):
        """Greedy generation of ``batch`` requests in lock step from host prompts of one length:
        H2D copy, one batched prefill of all requests (one per slot when they exceed
        ``max_prefill`` together), the first tokens read on the host (TTFT), then one
        graph-replayed batched step per token with a host read of the ``batch`` tokens. Returns
        ``(tokens per request, ttft_s, elapsed_s)``."""
        if len(prompts) != self.batch:
            raise ValueError(f"expected {self.batch} prompts")
        hosts = [torch.as_tensor(p, dtype=torch.int64).reshape(-1) for p in prompts]
        if len({h.numel() for h in hosts}) != 1:
            raise ValueError("the prompts of one batch share a length (one cache position for all)")
        host = torch.stack(hosts).pin_memory()
        start = time.perf_counter()
        ids = host.to(self.device, non_blocking=True)
        if ids.numel() <= self.max_prefill:
            self.prefill_batch(ids)
        else:
            for slot in range(self.batch):
                self.prefill(ids[slot], slot)
        out = [[t] for t in self.token.tolist()]
        first_at = time.perf_counter()
        graph = self.capture(1) if max_new_tokens > 1 else None
        for _ in range(max_new_tokens - 1):
            graph.replay()
            for seq, t in zip(out, self.token.tolist()):
                seq.append(t)
        return out, first_at - start, time.perf_counter() - start

    def generate(self, prompt_ids, max_new_tokens: int, *, eos_ids=(), use_graph: bool = True,
                 graph_steps: int = 1):
        """Greedy generation from host token ids, mirroring evaluation_wrapper.py:307-441:
        H2D copy of the prompt, prefill, first token read on the host (TTFT), then one decode
        step per token with a host read of each token (EOS check). Returns
        ``(tokens, ttft_s, elapsed_s)``."""
        eos = set(int(e) for e in eos_ids)
        host = torch.as_tensor(prompt_ids, dtype=torch.int64).reshape(-1)
        if not host.is_pinned():
            host = host.pin_memory()
        start = time.perf_counter()
        ids = host.to(self.device, non_blocking=True)
        self.prefill(ids)
        tokens = [int(self.token.item())]
        first_at = time.perf_counter()
        graph = self.capture(graph_steps) if (use_graph and max_new_tokens > 1) else None
        while len(tokens) < max_new_tokens and tokens[-1] not in eos:
            if graph is not None:
                graph.replay()
                if graph_steps == 1:
                    new = [int(self.token.item())]
                else:
                    pos = int(self.log_pos.item())
                    idx = [(pos - graph_steps + j) % self.log_len for j in range(graph_steps)]
                    new = [int(v) for v in self.token_log[idx].tolist()]
            else:
                self.decode_step()
                new = [int(self.token.item())]
            for t in new:
                if len(tokens) >= max_new_tokens:
                    break
                tokens.append(t)
                if t in eos:
                    break
        end = time.perf_counter()
        return tokens, first_at - start, end - start
