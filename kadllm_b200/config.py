"""Architecture description of the hybrid Gated-DeltaNet / full-attention stack.

The fields mirror Transformers' ``Qwen3_5TextConfig`` (the model that Kadllm's
``Qwen35GRBeamAdapter`` wraps, ``src/kadllm/adapters/qwen3_5.py:40-96``) so a
config can be taken from a loaded model (:meth:`HybridConfig.from_hf`) or built
directly for synthetic benchmarks.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace

LINEAR = "linear_attention"
FULL = "full_attention"


@dataclass(frozen=True)
class HybridConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    layer_types: tuple[str, ...]
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int = 4
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    partial_rotary_factor: float = 0.25
    tie_word_embeddings: bool = True
    extra: dict = field(default_factory=dict, compare=False)

    # ---- derived sizes -------------------------------------------------
    @property
    def num_layers(self) -> int:
        return len(self.layer_types)

    @property
    def key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def gdn_in_dim(self) -> int:
        """Width of the packed GDN input projection: qkv | z | b | a."""
        return self.conv_dim + self.value_dim + 2 * self.linear_num_value_heads

    @property
    def attn_in_dim(self) -> int:
        """Width of the packed attention input projection: (q|gate) per head | k | v."""
        return (2 * self.num_attention_heads + 2 * self.num_key_value_heads) * self.head_dim

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def validate(self) -> None:
        if any(kind not in (LINEAR, FULL) for kind in self.layer_types):
            raise ValueError("unsupported layer type")
        if self.linear_conv_kernel_dim != 4:
            raise ValueError("only width-4 short convolutions are supported")
        if self.linear_num_value_heads % self.linear_num_key_heads:
            raise ValueError("linear value heads must be a multiple of key heads")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("attention heads must be a multiple of kv heads")
        if self.linear_key_head_dim not in (32, 64, 128) or self.linear_value_head_dim not in (32, 64, 128):
            raise ValueError("GDN head dims must be 32, 64 or 128")
        if self.head_dim not in (32, 64, 128, 256):
            raise ValueError("attention head_dim must be 32, 64, 128 or 256")
        if self.rotary_dim % 2 or self.rotary_dim > self.head_dim:
            raise ValueError("rotary dim must be even and at most head_dim")
        if self.hidden_size not in (128, 256, 512, 1024, 2048):
            raise ValueError("hidden size must be one of 128, 256, 512, 1024, 2048")
        if self.intermediate_size % 8:
            raise ValueError("intermediate size must be a multiple of 8")

    # ---- conversions -----------------------------------------------------
    @classmethod
    def from_hf(cls, cfg) -> "HybridConfig":
        """Build from a Transformers ``Qwen3_5TextConfig``."""
        rope = dict(cfg.rope_parameters or {})
        if rope.get("rope_type", "default") != "default":
            raise ValueError("only default RoPE is supported")
        return cls(
            vocab_size=cfg.vocab_size,
            hidden_size=cfg.hidden_size,
            intermediate_size=cfg.intermediate_size,
            layer_types=tuple(cfg.layer_types),
            num_attention_heads=cfg.num_attention_heads,
            num_key_value_heads=cfg.num_key_value_heads,
            head_dim=cfg.head_dim,
            linear_num_key_heads=cfg.linear_num_key_heads,
            linear_num_value_heads=cfg.linear_num_value_heads,
            linear_key_head_dim=cfg.linear_key_head_dim,
            linear_value_head_dim=cfg.linear_value_head_dim,
            linear_conv_kernel_dim=cfg.linear_conv_kernel_dim,
            rms_norm_eps=cfg.rms_norm_eps,
            rope_theta=float(rope.get("rope_theta", 10000.0)),
            partial_rotary_factor=float(rope.get("partial_rotary_factor", 0.25)),
            tie_word_embeddings=bool(getattr(cfg, "tie_word_embeddings", False)),
        )

    def to_hf_kwargs(self) -> dict:
        """Keyword arguments for ``transformers.Qwen3_5TextConfig``."""
        return dict(
            vocab_size=self.vocab_size,
            hidden_size=self.hidden_size,
            intermediate_size=self.intermediate_size,
            num_hidden_layers=self.num_layers,
            layer_types=list(self.layer_types),
            num_attention_heads=self.num_attention_heads,
            num_key_value_heads=self.num_key_value_heads,
            head_dim=self.head_dim,
            linear_num_key_heads=self.linear_num_key_heads,
            linear_num_value_heads=self.linear_num_value_heads,
            linear_key_head_dim=self.linear_key_head_dim,
            linear_value_head_dim=self.linear_value_head_dim,
            linear_conv_kernel_dim=self.linear_conv_kernel_dim,
            rms_norm_eps=self.rms_norm_eps,
            rope_parameters=dict(
                rope_type="default",
                rope_theta=self.rope_theta,
                partial_rotary_factor=self.partial_rotary_factor,
            ),
            tie_word_embeddings=self.tie_word_embeddings,
        )

    def with_(self, **kw) -> "HybridConfig":
        return replace(self, **kw)


_PATTERN = (LINEAR, LINEAR, LINEAR, FULL)

#: Config 1: the tiny CPU-plumbing hybrid (3 GDN layers, then one GQA layer).
TINY = HybridConfig(
    vocab_size=4096,
    hidden_size=128,
    intermediate_size=384,
    layer_types=_PATTERN,
    num_attention_heads=4,
    num_key_value_heads=2,
    head_dim=32,
    linear_num_key_heads=4,
    linear_num_value_heads=4,
    linear_key_head_dim=32,
    linear_value_head_dim=32,
)

#: Qwen3.5-0.8B text dims: 24 layers in a 3:1 GDN/attention pattern, 16x128 GDN
#: heads, 8 q / 2 kv attention heads of 256, partial RoPE 0.25, tied embeddings.
QWEN35_08B = HybridConfig(
    vocab_size=248320,
    hidden_size=1024,
    intermediate_size=3584,
    layer_types=_PATTERN * 6,
    num_attention_heads=8,
    num_key_value_heads=2,
    head_dim=256,
    linear_num_key_heads=16,
    linear_num_value_heads=16,
    linear_key_head_dim=128,
    linear_value_head_dim=128,
    rope_theta=10_000_000.0,
)

PRESETS = {"tiny": TINY, "qwen3.5-0.8b": QWEN35_08B}
