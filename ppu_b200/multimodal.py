"""Image + text requests: the vision tower and the text decoder on one GPU.

The reference serves MMBench-style requests through ``VLMModel.generate_with_metrics``: the
processor patches the image, the (patched) vision tower encodes it, the image features replace the
image placeholder tokens of the prompt (Transformers' masked_scatter), the text model prefills
with 3-axis M-RoPE positions, and the greedy decode runs from the graph cache
(evaluation_wrapper.py:307-441, integration.py:509-736). ``MultimodalEngine`` does the same with
this package's engines: ``VisionEngine`` (one CUDA graph per image size) and ``Qwen35Engine``
(``prefill_multimodal`` + the captured decode step).

Prompt layout: the merged image tokens first, then the text tokens (config 5: 196 image tokens
before 300 text tokens). Positions follow Transformers' get_rope_index: the image tokens take
(t, h, w) = (0, merged row, merged column), the text continues at max(merged rows, merged
columns) on all three axes, and decoding continues after the last text position.
"""

from __future__ import annotations

import time

import torch

from .config import Qwen35Dims, VisionDims
from .engine import Qwen35Engine, cache_bucket
from .vision import VisionEngine, vision_positions

IMAGE_TOKEN_ID = 248056  # Qwen3_5Config.image_token_id (the placeholder the image features replace)


def prompt_layout(vd: VisionDims, image_hw: tuple[int, int], n_text: int):
    """(image_rows int64 [n_img], positions3 int64 [3, n_img + n_text], rope_next) of an image
    prepended to ``n_text`` text tokens."""
    n_img = vd.merged_tokens(*image_hw)
    img_pos = vision_positions(vd, *image_hw, start=0)
    gh, gw = vd.grid(*image_hw)
    text_start = max(gh, gw) // vd.merge
    text_pos = torch.arange(text_start, text_start + n_text, dtype=torch.int64).view(1, -1).expand(3, -1)
    positions = torch.cat((img_pos, text_pos), 1).contiguous()
    return torch.arange(n_img, dtype=torch.int64), positions, text_start + n_text


class MultimodalEngine:
    def __init__(self, text_weights: dict | None, vision_weights: dict | None, dims: Qwen35Dims = Qwen35Dims(),
                 vd: VisionDims = VisionDims(), *, image_hw=(448, 448), max_text: int = 512, max_new_tokens: int = 16,
                 a8w8: bool = False, device="cuda", text_engine: Qwen35Engine | None = None,
                 vision_engine: VisionEngine | None = None, decode_graph=None):
        """Builds both engines from Hugging Face-named weight dicts, or takes existing ones
        (``text_engine`` must hold a prompt of ``n_image + max_text`` tokens plus the decode steps;
        ``decode_graph`` replaces the text engine's captured decode step, e.g. a lock-step graph)."""
        self.dims, self.vd, self.image_hw = dims, vd, tuple(image_hw)
        self.vision = vision_engine or VisionEngine(vision_weights, vd, max_image=self.image_hw, device=device)
        self.device = self.vision.device
        self.n_img = vd.merged_tokens(*self.image_hw)
        max_prompt = self.n_img + max_text
        if text_engine is None:
            text_engine = Qwen35Engine(text_weights, dims, a8w8=a8w8,
                                       max_len=cache_bucket(max_prompt, max_new_tokens), max_prefill=max_prompt,
                                       device=self.device)
        elif text_engine.max_prefill < max_prompt or text_engine.max_len <= max_prompt + max_new_tokens:
            raise ValueError("the text engine's cache is too short for the multimodal prompt")
        self.text = text_engine
        self._vgraph = self.vision.capture(*self.image_hw)
        self._dgraph = decode_graph if decode_graph is not None else self.text.capture(1)
        self._layouts: dict[int, tuple[torch.Tensor, torch.Tensor, int]] = {}
        self._group_layouts: dict[tuple[int, int], tuple[torch.Tensor, torch.Tensor, torch.Tensor, int]] = {}
        # a batched text engine takes a group of requests per prefill; the vision tower takes the
        # group's images in one encode when its workspace holds them all
        self.batch = getattr(self.text, "batch", 1)
        n_patch = vd.merge * vd.merge * self.n_img
        self.group_images = max(1, min(self.batch, self.vision.max_patches // n_patch))
        self.group_prefill = self.batch > 1 and self.batch * max_prompt <= self.text.max_prefill

    def _layout(self, n_text: int):
        if n_text not in self._layouts:
            rows, pos, nxt = prompt_layout(self.vd, self.image_hw, n_text)
            self._layouts[n_text] = (rows.to(self.device), pos.to(self.device), nxt)
        return self._layouts[n_text]

    def encode_image(self, pixels: torch.Tensor) -> torch.Tensor:
        """Device pixels fp32 [3, H, W] -> the merged image tokens (the vision graph's output
        buffer, valid until the next encode)."""
        g, pix, tokens = self._vgraph
        pix.copy_(pixels, non_blocking=True)
        g.replay()
        return tokens

    def prefill(self, pixels: torch.Tensor, text_ids: torch.Tensor, slot: int = 0) -> torch.Tensor:
        """Device pixels fp32 [3, H, W] and text ids int64 [n]: vision graph, then the multimodal
        prefill (into request slot ``slot`` of a batched text engine); the first greedy token lands
        in ``text.token[slot]``."""
        return self.prefill_prompt(self.encode_image(pixels), text_ids, slot)

    def prefill_prompt(self, tokens: torch.Tensor, text_ids: torch.Tensor, slot: int = 0) -> torch.Tensor:
        """The text model's prefill of [image tokens, text ids] (image first)."""
        n_text = text_ids.numel()
        rows, pos, nxt = self._layout(n_text)
        ids = torch.cat((torch.full((self.n_img,), IMAGE_TOKEN_ID, device=self.device, dtype=torch.int64),
                         text_ids.reshape(-1)))
        return self.text.prefill_multimodal(ids, tokens, rows, pos, nxt, slot)

    def encode_images(self, pixels: torch.Tensor) -> torch.Tensor:
        """Device pixels fp32 ``[n, 3, H, W]`` -> merged tokens ``[n * n_image, out_width]`` (image
        order): one vision-graph replay per ``group_images`` images."""
        n = pixels.shape[0]
        outs = []
        for j in range(0, n, self.group_images):
            k = min(self.group_images, n - j)
            if k == 1:
                outs.append(self.encode_image(pixels[j]).clone() if n > 1 else self.encode_image(pixels[j]))
                continue
            g, pix, tokens = self.vision.capture(*self.image_hw, images=k)
            pix.copy_(pixels[j:j + k], non_blocking=True)
            g.replay()
            outs.append(tokens if n <= self.group_images else tokens.clone())
        return outs[0] if len(outs) == 1 else torch.cat(outs)

    def _group_layout(self, nseq: int, n_text: int):
        key = (nseq, n_text)
        if key not in self._group_layouts:
            rows, pos, nxt = self._layout(n_text)
            length = self.n_img + n_text
            all_rows = (rows.view(1, -1) + length * torch.arange(nseq, device=self.device).view(-1, 1)).reshape(-1)
            pos3 = pos.view(3, 1, length).expand(3, nseq, length).contiguous()
            img_ids = torch.full((nseq, self.n_img), IMAGE_TOKEN_ID, device=self.device, dtype=torch.int64)
            self._group_layouts[key] = (all_rows, pos3, img_ids, nxt)
        return self._group_layouts[key]

    def prefill_group(self, tokens: torch.Tensor, text_ids: torch.Tensor, slot: int = 0) -> torch.Tensor:
        """Batched text engines: ``n`` requests at once, merged image tokens ``[n * n_image,
        hidden]`` (``encode_images``) and text ids int64 ``[n, T]`` (one length), prefilled in one
        pass into slots ``slot .. slot + n - 1``; the first tokens land in ``text.token``."""
        nseq, n_text = text_ids.shape
        if not self.group_prefill or slot + nseq > self.batch:
            raise ValueError("group prefill needs a batched text engine whose max_prefill holds the group")
        rows, pos3, img_ids, nxt = self._group_layout(nseq, n_text)
        ids = torch.cat((img_ids, text_ids), 1)
        return self.text.prefill_batch(ids, image_embeds=tokens, image_rows=rows, positions3=pos3, rope_next=nxt,
                                       slot=slot)

    def decode_step(self) -> None:
        self._dgraph.replay()

    def generate(self, pixels, text_ids, max_new_tokens: int, *, eos_ids=()):
        """One request from host tensors (the image fp32 [3, H, W], text ids int64 [n]): H2D copies,
        vision + prefill, the first token read on the host (TTFT), then graph-replayed decode steps
        with a host read of each token. Returns ``(tokens, ttft_s, elapsed_s)``."""
        eos = set(int(e) for e in eos_ids)
        pix_h = torch.as_tensor(pixels, dtype=torch.float32)
        ids_h = torch.as_tensor(text_ids, dtype=torch.int64).reshape(-1)
        if not pix_h.is_pinned():
            pix_h = pix_h.pin_memory()
        if not ids_h.is_pinned():
            ids_h = ids_h.pin_memory()
        start = time.perf_counter()
        self.prefill(pix_h.to(self.device, non_blocking=True), ids_h.to(self.device, non_blocking=True))
        tokens = [int(self.text.token.item())]
        first = time.perf_counter()
        while len(tokens) < max_new_tokens and tokens[-1] not in eos:
            self.decode_step()
            tokens.append(int(self.text.token.item()))
        return tokens, first - start, time.perf_counter() - start
