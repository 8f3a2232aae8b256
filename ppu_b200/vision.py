"""Device-resident Qwen3.5 vision tower driven through the C ABI ViT runner.

``VisionEngine`` holds a Hugging Face-named vision weight dict (``model.visual.*`` of
``Qwen3_5ForConditionalGeneration``) on the GPU, flattens the Conv3d patch embedding into a
``[width, C*T*P*P]`` GEMM weight, and creates a ``q35_vit`` (``q35_vit_encode``: patchify, patch
embedding on tcgen05, position embedding, 24 blocks of 8 launches, 2x2 merger). ``encode`` maps one
image (fp32 ``[3, H, W]`` rescaled to [0, 1)) to the merged visual tokens ``[H*W/(P*M)^2,
out_width]`` bf16 that the text model consumes; ``capture`` records an encode of a fixed image
size into a CUDA graph (the reference caches one vision graph per patch count,
integration.py:586-637).
"""

from __future__ import annotations

import ctypes as C

import torch

from . import lib as L
from .config import VisionDims

BF16 = torch.bfloat16


def vision_rope_inv_freq(head_dim: int, theta: float = 10000.0) -> torch.Tensor:
    """Qwen3_5VisionRotaryEmbedding(head_dim // 2).inv_freq in FP32."""
    dim = head_dim // 2
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))


def vision_positions(vd: VisionDims, height: int, width: int, start: int = 0) -> torch.Tensor:
    """3-axis M-RoPE positions ``[3, n_merged]`` of an image's merged tokens in the text model
    (Transformers get_vision_position_ids): temporal = start, height = start + merged row,
    width = start + merged column; the text after the image continues at
    ``start + max(merged rows, merged cols)``."""
    gh, gw = vd.grid(height, width)
    mh, mw = gh // vd.merge, gw // vd.merge
    t = torch.full((mh * mw,), start, dtype=torch.int64)
    h = torch.arange(start, start + mh, dtype=torch.int64).repeat_interleave(mw)
    w = torch.arange(start, start + mw, dtype=torch.int64).repeat(mh)
    return torch.stack([t, h, w])


class VisionEngine:
    def __init__(self, weights: dict, vd: VisionDims = VisionDims(), *, max_image=(448, 448), device="cuda",
                 prefix: str = "model.visual.", max_patches: int | None = None):
        L.load()
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("VisionEngine runs on a CUDA device only")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if vd.head_dim != 64:
            raise ValueError("the vision kernels are built for head dim 64")
        self.vd, self.device = vd, dev

        def w(name):
            return weights[prefix + name].to(device=dev, dtype=BF16).contiguous()

        self._keep: list[torch.Tensor] = []

        def keep(t):
            self._keep.append(t)
            return t.data_ptr()

        self.blocks = (L.VitBlockDesc * vd.depth)()
        for i in range(vd.depth):
            b, p = self.blocks[i], f"blocks.{i}."
            b.norm1_w, b.norm1_b = keep(w(p + "norm1.weight")), keep(w(p + "norm1.bias"))
            b.norm2_w, b.norm2_b = keep(w(p + "norm2.weight")), keep(w(p + "norm2.bias"))
            b.qkv_w, b.qkv_b = keep(w(p + "attn.qkv.weight")), keep(w(p + "attn.qkv.bias"))
            b.proj_w, b.proj_b = keep(w(p + "attn.proj.weight")), keep(w(p + "attn.proj.bias"))
            b.fc1_w, b.fc1_b = keep(w(p + "mlp.linear_fc1.weight")), keep(w(p + "mlp.linear_fc1.bias"))
            b.fc2_w, b.fc2_b = keep(w(p + "mlp.linear_fc2.weight")), keep(w(p + "mlp.linear_fc2.bias"))
        self.inv_freq = vision_rope_inv_freq(vd.head_dim, vd.rope_theta).to(dev)
        gh, gw = vd.grid(*max_image)
        self.max_patches = max(gh * gw, max_patches or 0)
        d = L.VitDesc()
        d.depth, d.width, d.heads, d.intermediate = vd.depth, vd.width, vd.heads, vd.intermediate
        d.in_channels, d.patch, d.temporal_patch, d.merge = vd.in_channels, vd.patch, vd.temporal_patch, vd.merge
        d.out_width, d.pos_side, d.max_patches, d.eps = vd.out_width, vd.pos_side, self.max_patches, vd.eps
        d.pixel_mean, d.pixel_std = vd.pixel_mean, vd.pixel_std
        d.blocks = self.blocks
        d.patch_w = keep(w("patch_embed.proj.weight").reshape(vd.width, -1).contiguous())
        d.patch_b = keep(w("patch_embed.proj.bias"))
        d.pos_table = keep(w("pos_embed.weight"))
        d.rope_inv_freq = self.inv_freq.data_ptr()
        d.merger_norm_w, d.merger_norm_b = keep(w("merger.norm.weight")), keep(w("merger.norm.bias"))
        d.merger_fc1_w, d.merger_fc1_b = keep(w("merger.linear_fc1.weight")), keep(w("merger.linear_fc1.bias"))
        d.merger_fc2_w, d.merger_fc2_b = keep(w("merger.linear_fc2.weight")), keep(w("merger.linear_fc2.bias"))
        size = L.load().q35_vit_workspace_size(C.byref(d))
        self.workspace = torch.zeros(size, device=dev, dtype=torch.uint8)
        d.workspace, d.workspace_bytes = self.workspace.data_ptr(), size
        self.desc = d
        handle = C.c_void_p()
        L.check(L.load().q35_vit_create(C.byref(d), C.byref(handle)), "q35_vit_create")
        self.handle = handle
        self._graphs: dict[tuple[int, int, int], tuple[torch.cuda.CUDAGraph, torch.Tensor, torch.Tensor]] = {}

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                L.load().q35_vit_destroy(h)
            except Exception:
                pass

    def kernels_per_encode(self) -> int:
        return 4 + 8 * self.vd.depth + 2

    def encode(self, pixels: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """One image, fp32 ``[C, H, W]`` on this device -> merged visual tokens bf16 ``[n, out_width]``
        (current stream)."""
        if pixels.dim() != 3 or pixels.dtype != torch.float32 or pixels.device != self.device:
            raise ValueError("pixels must be an fp32 [C, H, W] tensor on the engine's device")
        pixels = pixels.contiguous()
        _, h, wd = pixels.shape
        n = self.vd.merged_tokens(h, wd)
        if out is None:
            out = torch.empty((n, self.vd.out_width), device=self.device, dtype=BF16)
        L.check(L.load().q35_vit_encode(self.handle, pixels.data_ptr(), h, wd, out.data_ptr(),
                                        L.stream_of(self.device)), "q35_vit_encode")
        return out

    def encode_batch(self, pixels: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Images of one size, fp32 ``[n, C, H, W]`` on this device -> merged tokens bf16
        ``[n * tokens, out_width]`` (image order), one launch sequence for the whole batch."""
        if pixels.dim() != 4 or pixels.dtype != torch.float32 or pixels.device != self.device:
            raise ValueError("pixels must be an fp32 [n, C, H, W] tensor on the engine's device")
        pixels = pixels.contiguous()
        n_img, _, h, wd = pixels.shape
        n = n_img * self.vd.merged_tokens(h, wd)
        if out is None:
            out = torch.empty((n, self.vd.out_width), device=self.device, dtype=BF16)
        L.check(L.load().q35_vit_encode_batch(self.handle, pixels.data_ptr(), n_img, h, wd, out.data_ptr(),
                                              L.stream_of(self.device)), "q35_vit_encode_batch")
        return out

    def encode_patches(self, patches: torch.Tensor, grid_h: int, grid_w: int,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """One image from the processor's patches (fp32 ``[grid_h*grid_w, C*T*P*P]``, the
        ``pixel_values`` Transformers feeds Qwen3_5VisionModel) -> merged tokens bf16."""
        n = grid_h * grid_w
        if patches.shape != (n, self.vd.patch_features) or patches.device != self.device:
            raise ValueError(f"patches must be [{n}, {self.vd.patch_features}] on the engine's device")
        if patches.dtype != torch.float32:
            raise ValueError("patches must be fp32 (the processor's pixel_values)")
        patches = patches.contiguous()
        if out is None:
            m2 = self.vd.merge * self.vd.merge
            out = torch.empty((n // m2, self.vd.out_width), device=self.device, dtype=BF16)
        L.check(L.load().q35_vit_encode_patches(self.handle, patches.data_ptr(), grid_h, grid_w, out.data_ptr(),
                                                L.stream_of(self.device)), "q35_vit_encode_patches")
        return out

    def hidden(self, n_patches: int) -> torch.Tensor:
        """The last encode's final patch states ``[n_patches, width]`` (pre-merger), a view."""
        ptr = L.load().q35_vit_hidden(self.handle)
        off = ptr - self.workspace.data_ptr()
        nbytes = 2 * n_patches * self.vd.width
        return self.workspace[off:off + nbytes].view(BF16).view(n_patches, self.vd.width)

    def capture(self, height: int, width: int, images: int = 1):
        """CUDA graph of one encode at a fixed image size (of ``images`` images at once); returns
        ``(graph, pixels_in, tokens_out)``: copy the image(s) into ``pixels_in`` (``[C, H, W]``, or
        ``[images, C, H, W]`` when ``images > 1``), replay, read ``tokens_out``."""
        key = (height, width, images)
        if key in self._graphs:
            return self._graphs[key]
        shape = (self.vd.in_channels, height, width)
        pix = torch.zeros(shape if images == 1 else (images, *shape), device=self.device, dtype=torch.float32)
        out = torch.empty((images * self.vd.merged_tokens(height, width), self.vd.out_width), device=self.device,
                          dtype=BF16)
        run = self.encode if images == 1 else self.encode_batch
        run(pix, out)  # warm-up: first-use kernel attributes are set outside the capture
        torch.cuda.synchronize(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
            run(pix, out)
        torch.cuda.current_stream(self.device).wait_stream(side)
        self._graphs[key] = (g, pix, out)
        return self._graphs[key]
