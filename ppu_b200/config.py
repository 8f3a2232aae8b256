"""Model dimensions and fusion switches for the Qwen3.5 text decoder hot path."""

from __future__ import annotations

from dataclasses import dataclass, field


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass(frozen=True)
class Qwen35Dims:
    """Shape of a Qwen3.5 text decoder (defaults: the 2B checkpoint's language model).

    Values follow the Hugging Face ``Qwen3_5TextConfig`` of the 2B checkpoint: hidden 2048,
    SwiGLU 6144, 24 layers in a 3 x Gated-DeltaNet : 1 x gated-GQA pattern, 8 query / 2 KV
    heads of width 256 with RoPE on the first 64 dims (theta 1e7), 16 linear-attention heads
    of key/value width 128, causal conv kernel 4, tied embedding of 248320 rows.
    """

    vocab: int = 248320
    hidden: int = 2048
    intermediate: int = 6144
    layers: int = 24
    full_attention_interval: int = 4
    q_heads: int = 8
    kv_heads: int = 2
    head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 1.0e7
    mrope_section: tuple = (11, 11, 10)
    lin_heads: int = 16
    lin_dk: int = 128
    lin_dv: int = 128
    conv_kernel: int = 4
    eps: float = 1e-6
    # The reference pads the packed DeltaNet rows to 128 for Triton tiles (integration.py:90-93);
    # the CUDA GEMV needs no padding, so rows are only rounded to 16 (8224 rows, no dead rows).
    delta_padding: int = 16

    @property
    def layer_types(self) -> list[str]:
        """integration.py iterates ``layer.block_type``; HF builds this list the same way."""
        return [
            "linear_attention" if (i + 1) % self.full_attention_interval else "full_attention"
            for i in range(self.layers)
        ]

    @property
    def n_delta(self) -> int:
        return sum(t == "linear_attention" for t in self.layer_types)

    @property
    def n_attn(self) -> int:
        return self.layers - self.n_delta

    @property
    def key_dim(self) -> int:
        return self.lin_heads * self.lin_dk

    @property
    def value_dim(self) -> int:
        return self.lin_heads * self.lin_dv

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def delta_rows(self) -> int:
        """Rows of the packed DeltaNet projection ``[qkv | z | a | b | pad]`` (integration.py:81-93)."""
        raw = self.conv_dim + self.value_dim + 2 * self.lin_heads
        return _round_up(raw, self.delta_padding) if self.delta_padding else raw

    @property
    def qgkv_rows(self) -> int:
        return 2 * self.q_heads * self.head_dim + 2 * self.kv_heads * self.head_dim

    @property
    def attn_width(self) -> int:
        return self.q_heads * self.head_dim

    def weight_bytes_per_token(self, a8w8: bool = False) -> int:
        """Algorithmic HBM bytes one batch-1 decode step must read (weights + DeltaNet state
        read/write + conv state), excluding the KV cache."""
        h = self.hidden
        per_delta = self.delta_rows * h + h * self.value_dim
        per_attn = self.qgkv_rows * h + h * self.attn_width
        mlp = 3 * self.intermediate * h
        lin_params = self.n_delta * per_delta + self.n_attn * per_attn + self.layers * mlp
        if a8w8:
            lin = lin_params + 4 * (
                self.n_delta * (self.delta_rows + h) + self.n_attn * (self.qgkv_rows + h)
                + self.layers * (2 * self.intermediate + h)
            )
        else:
            lin = 2 * lin_params
        lm_head = 2 * self.vocab * h
        state = self.n_delta * (2 * 4 * self.lin_heads * self.lin_dk * self.lin_dv
                                + 2 * 2 * self.conv_dim * self.conv_kernel
                                + 2 * self.conv_dim * self.conv_kernel)
        return lin + lm_head + state


@dataclass(frozen=True)
class FusionConfig:
    """Switches mirroring qwen35_fused/integration.py:32-48 (``FusionConfig``).

    Triton tile knobs of the reference (``delta_block_v``, ``ppu_swiglu_block_n``) are accepted
    and ignored: tile shapes here are compile-time constants of the CUDA kernels.
    ``a8w8`` selects int8 weights with per-token int8 activations for the M/F/L projection
    groups (explore_runtime_quantization.py:66-84); the LM head stays BF16.
    """

    delta: bool = True
    rms_norm: bool = True
    residual_norm: bool = True
    swiglu: bool = True
    attention: bool = True
    vision: bool = True
    release_original_weights: bool = True
    delta_projection_padding: int = 128
    delta_block_v: int = 8
    delta_precompute_factors: bool = True
    ppu_swiglu_gemv: bool = True
    ppu_swiglu_block_n: int = 8
    gqa_decode_attention: bool = True
    vision_graph: bool = False
    vision_graph_max_entries: int = 48
    a8w8: bool = False
    # The reference's patched forwards hand inputs that are not BF16 CUDA tensors (and padded
    # batches, which need a 4D mask) back to the Transformers implementation. Off by default
    # here: such inputs raise ValueError, so nothing silently leaves the B200 kernels.
    eager_fallback: bool = False
    extra: dict = field(default_factory=dict, compare=False, hash=False)


@dataclass(frozen=True)
class VisionDims:
    """Vision tower shape (defaults: BASELINE config 5's ViT: 24 layers, width 1024, 16 heads of 64,
    SwiGLU-free GELU(tanh) MLP 4096, patch 16 over 2 temporal slots, 2 x 2 merge to the text model's
    hidden 2048, a 48 x 48 learned position table; the Qwen2-VL processor's mean = std = 0.5)."""

    depth: int = 24
    width: int = 1024
    heads: int = 16
    intermediate: int = 4096
    in_channels: int = 3
    patch: int = 16
    temporal_patch: int = 2
    merge: int = 2
    out_width: int = 2048
    pos_side: int = 48
    eps: float = 1e-6
    rope_theta: float = 10000.0
    pixel_mean: float = 0.5
    pixel_std: float = 0.5

    @property
    def head_dim(self) -> int:
        return self.width // self.heads

    @property
    def patch_features(self) -> int:
        return self.in_channels * self.temporal_patch * self.patch * self.patch

    def grid(self, height: int, width: int) -> tuple[int, int]:
        """Patch grid (rows, cols) of an image; both must be multiples of patch x merge."""
        step = self.patch * self.merge
        if height % step or width % step:
            raise ValueError(f"image {height}x{width} is not a multiple of {step}")
        return height // self.patch, width // self.patch

    def merged_tokens(self, height: int, width: int) -> int:
        gh, gw = self.grid(height, width)
        return gh * gw // (self.merge * self.merge)

    def linear_flops(self, height: int, width: int) -> int:
        """Dense FLOPs of one image: patch embedding, per block QKV / proj / fc1 / fc2 and the
        bidirectional attention, and the merger."""
        gh, gw = self.grid(height, width)
        n = gh * gw
        w, i = self.width, self.intermediate
        per_block = 2 * n * (3 * w * w + w * w + 2 * w * i) + 4 * n * n * w
        mw = w * self.merge * self.merge
        nm = n // (self.merge * self.merge)
        return 2 * n * self.patch_features * w + self.depth * per_block + 2 * nm * (mw * mw + mw * self.out_width)
