"""Static shapes of the two encoders on the hot path.

`TowerConfig` is the moondream2 SigLIP-style vision tower that `FastMD2._vision` runs
(moondream/gpu/md2fast.py:25-28 for the 378 / 14 / 27 / 729 geometry, md2fast.py:89-103 for
the weight set, md2fast.py:147-160 for the forward).  `TapNextConfig` is the TAPNext-style
per-frame step: a ViT block followed by an RG-LRU recurrence, 12 deep, 1280 tokens of width 768
(the token layout of tapnext/npu/step8.py:251-267, the RG-LRU of tapnext/npu/r9/cpuemu.py:33-47).
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class TowerConfig:
    width: int = 1152          # enc_dim
    heads: int = 16            # enc_n_heads
    head_dim: int = 72
    ff: int = 4304             # MLP hidden
    n_blocks: int = 27
    img: int = 378
    patch: int = 14
    in_ch: int = 3
    proj_hidden: int = 8192    # projection MLP 2304 -> 8192 -> 2048
    proj_out: int = 2048
    eps: float = 1e-6          # LayerNorm eps the configs specify (the reference's _ln uses torch's 1e-5)

    @property
    def grid(self) -> int:
        return self.img // self.patch            # 27

    @property
    def ntok(self) -> int:
        return self.grid * self.grid             # 729

    @property
    def patch_k(self) -> int:
        return self.in_ch * self.patch * self.patch  # 588

    @property
    def qkv_dim(self) -> int:
        return 3 * self.heads * self.head_dim    # 3456

    def flops_per_crop(self) -> dict:
        """Algorithmic FLOPs of one crop through patch-embed + blocks (no padding counted)."""
        T, W = self.ntok, self.width
        blk_gemm = 2 * T * W * (self.qkv_dim + W + 2 * self.ff)
        blk_attn = 4 * T * T * self.head_dim * self.heads
        pe = 2 * T * self.patch_k * W
        return {"gemm": self.n_blocks * blk_gemm + pe, "attn": self.n_blocks * blk_attn,
                "total": self.n_blocks * (blk_gemm + blk_attn) + pe}


@dataclass(frozen=True)
class TapNextConfig:
    width: int = 768
    heads: int = 12
    head_dim: int = 64
    ff: int = 3072
    n_blocks: int = 12
    img: int = 256
    patch: int = 8
    in_ch: int = 3
    n_queries: int = 256
    eps: float = 1e-6
    lru_c: float = 8.0          # a = sigmoid(-a_param) ** (c * r_t)
    # tracking heads on the query tokens (the reference's model.coordinate_head / visible_head, run on the
    # host by tapnext/npu/step8.py:327-362): Linear width -> head_hidden, LN, GELU, Linear, LN, GELU, Linear
    # -> 2 x track_bins coordinate logits (y bins | x bins) or 1 visibility logit; soft-argmax window +-20
    head_hidden: int = 256
    track_bins: int = 256
    track_window: int = 20
    track_temperature: float = 0.5
    head_eps: float = 1e-6

    @property
    def grid(self) -> int:
        return self.img // self.patch            # 32

    @property
    def n_img_tok(self) -> int:
        return self.grid * self.grid             # 1024

    @property
    def ntok(self) -> int:
        return self.n_img_tok + self.n_queries   # 1280

    @property
    def patch_k(self) -> int:
        return self.in_ch * self.patch * self.patch  # 192

    def flops_per_frame(self) -> int:
        T, W = self.ntok, self.width
        vit = 2 * T * W * (3 * W + W + 2 * self.ff) + 4 * T * T * self.head_dim * self.heads
        gates = 2 * T * W * (2 * W)
        pe = 2 * self.n_img_tok * self.patch_k * W
        return self.n_blocks * (vit + gates) + pe


@dataclass(frozen=True)
class TextConfig:
    """The moondream2 text decoder that consumes the tower's features (FastMD2._text_layers / _encode /
    _query, moondream/gpu/md2fast.py:162-212; dims as moondream/gpu/gemm_bench.py:14): 24 parallel
    attention + MLP blocks of width 2048, 32 heads x 64 with rotary embedding on the first 32 dims of each
    head (md2fast.py:29, 162-167), a 730-token prefix (bos + 729 image tokens) and a 32-token question
    whose yes / no logits are read at its last real token."""
    dim: int = 2048
    heads: int = 32
    head_dim: int = 64
    ff: int = 8192
    n_layers: int = 24
    rot: int = 32
    theta: float = 10000.0
    prefix: int = 730
    q_len: int = 32
    vocab: int = 1024           # synthetic embedding rows (the tokenizer and 51200-row table are not needed)
    n_yn: int = 4               # yes / no rows of the lm head (lm_small, md2fast.py:139-143)
    eps: float = 1e-5           # torch's layer_norm default, as _ln (md2fast.py:43-44)

    @property
    def ctx(self) -> int:
        return self.prefix + self.q_len

    def flops(self, n) -> int:
        """GEMM FLOPs of n tokens through all layers (attention excluded)."""
        D, Fh = self.dim, self.ff
        return self.n_layers * 2 * n * D * (3 * D + D + 2 * Fh)


TOWER = TowerConfig()
TAPNEXT = TapNextConfig()
TEXT = TextConfig()
