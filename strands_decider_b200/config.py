"""Model and workload specifications for the B200 scoring-prefill backend.

A `ModelSpec` describes the hybrid decider torso the reference runs through transformers'
Qwen3.5 text model (`Qwen3_5TextConfig`; layer pattern, GDN and attention shapes, RoPE,
RMSNorm eps, tied embeddings) plus the packed weight format of its linears.

The device keeps each layer's linears fused so one GEMM launch covers what the reference
runs as several `nn.Linear`s:
  GDN in-projection   rows [in_proj_qkv | in_proj_z | in_proj_b | in_proj_a]
                      (TF:417-420), padded to a multiple of 256 rows
  attention qkv       rows [q_proj (query and gate, per head) | k_proj | v_proj]
                      (TF:632-640)
  MLP gate/up         rows interleaved in blocks of 64: gate[64j:64j+64], up[64j:64j+64]
                      (TF:701-702), so a 128-column accumulator tile holds matching
                      gate and up columns and the SwiGLU runs in the GEMM epilogue
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace

GDN = "linear_attention"
ATTN = "full_attention"

WEIGHT_FORMATS = ("bf16", "int4", "nvfp4", "ternary")
ROW_PAD = 256          # fused weights are padded to this many rows (the GEMM's widest N tile)
SWIGLU_BLOCK = 64      # gate/up interleave block


def _pad(n: int, m: int = ROW_PAD) -> int:
    return (n + m - 1) // m * m


@dataclass(frozen=True)
class ModelSpec:
    name: str
    vocab: int
    hidden: int
    inter: int
    layer_types: tuple[str, ...]
    gdn_heads: int
    gdn_dk: int = 128
    gdn_dv: int = 128
    conv_width: int = 4
    attn_heads: int = 8
    attn_kv_heads: int = 2
    head_dim: int = 128
    rope_theta: float = 1e7
    partial_rotary: float = 0.25
    eps: float = 1e-6
    weight_format: str = "int4"
    max_positions: int = 4096

    # ---- derived shapes
    @property
    def n_layers(self) -> int:
        return len(self.layer_types)

    @property
    def key_dim(self) -> int:
        return self.gdn_heads * self.gdn_dk

    @property
    def value_dim(self) -> int:
        return self.gdn_heads * self.gdn_dv

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def rope_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)

    @property
    def gdn_in_rows(self) -> int:
        return self.conv_dim + self.value_dim + 2 * self.gdn_heads

    @property
    def gdn_in_rows_padded(self) -> int:
        return _pad(self.gdn_in_rows)

    @property
    def gdn_f32_split(self) -> int:
        """First fused in-projection row written as fp32 (the b and a rows)."""
        return self.conv_dim + self.value_dim

    @property
    def attn_q_rows(self) -> int:
        return 2 * self.attn_heads * self.head_dim

    @property
    def attn_qkv_rows(self) -> int:
        return self.attn_q_rows + 2 * self.attn_kv_heads * self.head_dim

    @property
    def attn_o_in(self) -> int:
        return self.attn_heads * self.head_dim

    def linear_params(self) -> int:
        n = 0
        for lt in self.layer_types:
            if lt == GDN:
                n += self.hidden * self.gdn_in_rows + self.value_dim * self.hidden
            else:
                n += self.hidden * self.attn_qkv_rows + self.attn_o_in * self.hidden
            n += 3 * self.hidden * self.inter
        return n

    def logical_linears(self, li: int) -> list[tuple[str, int, int]]:
        """(name, out_features, in_features) of layer li's linears, reference naming."""
        H = self.hidden
        if self.layer_types[li] == GDN:
            mix = [("linear_attn.in_proj_qkv", self.conv_dim, H),
                   ("linear_attn.in_proj_z", self.value_dim, H),
                   ("linear_attn.in_proj_b", self.gdn_heads, H),
                   ("linear_attn.in_proj_a", self.gdn_heads, H),
                   ("linear_attn.out_proj", H, self.value_dim)]
        else:
            mix = [("self_attn.q_proj", self.attn_q_rows, H),
                   ("self_attn.k_proj", self.attn_kv_heads * self.head_dim, H),
                   ("self_attn.v_proj", self.attn_kv_heads * self.head_dim, H),
                   ("self_attn.o_proj", H, self.attn_o_in)]
        return mix + [("mlp.gate_proj", self.inter, H), ("mlp.up_proj", self.inter, H),
                      ("mlp.down_proj", H, self.inter)]

    def with_format(self, fmt: str) -> ModelSpec:
        assert fmt in WEIGHT_FORMATS
        return replace(self, weight_format=fmt)

    @classmethod
    def from_hf_config(cls, cfg, weight_format: str = "nvfp4", name: str | None = None,
                       max_positions: int = 32768) -> ModelSpec:
        """The spec of a transformers `Qwen3_5TextConfig` (the torso strands-decider loads,
        src/strands_decider/modeling.py:293-303). Raises ValueError for shapes the kernels
        do not take."""
        rp = getattr(cfg, "rope_parameters", None) or {}
        spec = cls(
            name=name or f"qwen3_5-h{cfg.hidden_size}-l{cfg.num_hidden_layers}", vocab=cfg.vocab_size,
            hidden=cfg.hidden_size, inter=cfg.intermediate_size, layer_types=tuple(cfg.layer_types),
            gdn_heads=cfg.linear_num_key_heads, gdn_dk=cfg.linear_key_head_dim, gdn_dv=cfg.linear_value_head_dim,
            conv_width=cfg.linear_conv_kernel_dim, attn_heads=cfg.num_attention_heads,
            attn_kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
            rope_theta=float(rp.get("rope_theta", getattr(cfg, "rope_theta", 1e7))),
            partial_rotary=float(rp.get("partial_rotary_factor", getattr(cfg, "partial_rotary_factor", 0.25))),
            eps=cfg.rms_norm_eps, weight_format=weight_format,
            max_positions=min(int(getattr(cfg, "max_position_embeddings", max_positions)), max_positions))
        if cfg.linear_num_value_heads != cfg.linear_num_key_heads:
            raise ValueError("GDN layers with different key and value head counts are not supported")
        if not getattr(cfg, "tie_word_embeddings", True):
            raise ValueError("the option-token head reads the tied embedding; untied checkpoints are not supported")
        spec.validate()
        return spec

    def validate(self) -> None:
        """The shapes the kernels take (raises ValueError otherwise)."""
        problems = []
        if self.gdn_dk != 128 or self.gdn_dv != 128:
            problems.append("GDN head dims must be 128")
        if self.head_dim not in (64, 128, 256):
            problems.append("attention head_dim must be 64, 128 or 256")
        if self.hidden % 128 or self.inter % 128 or self.hidden > 4096:
            problems.append("hidden and intermediate sizes must be multiples of 128 (hidden <= 4096)")
        if self.conv_width != 4:
            problems.append("the depthwise conv width must be 4")
        if self.attn_heads % self.attn_kv_heads:
            problems.append("query heads must be a multiple of kv heads")
        if any(t not in (GDN, ATTN) for t in self.layer_types):
            problems.append("layer types must be linear_attention or full_attention")
        if self.weight_format not in WEIGHT_FORMATS:
            problems.append(f"weight format must be one of {WEIGHT_FORMATS}")
        if problems:
            raise ValueError("; ".join(problems))


def hybrid_pattern(n_layers: int) -> tuple[str, ...]:
    """[GDN, GDN, GDN, attention] repeated (Qwen3.5's full_attention_interval 4)."""
    return tuple(ATTN if (i + 1) % 4 == 0 else GDN for i in range(n_layers))


# Reduced fp32 CPU decider: hidden 1024, 8 layers [GDN x3, attn] x2, GDN 8 heads x 128,
# attention 8q/2kv x 128, FFN 3072, vocab 32768 tied; int4 group-128 weights.
REDUCED_1024 = ModelSpec(
    name="reduced-hybrid-h1024-l8", vocab=32768, hidden=1024, inter=3072,
    layer_types=hybrid_pattern(8), gdn_heads=8, attn_heads=8, attn_kv_heads=2,
    head_dim=128, weight_format="int4")

# 2B-shape hybrid: hidden 2048, 24 layers at 3:1 GDN:attention, GDN 16 heads x 128,
# attention 8q/2kv x 256, FFN 6144, vocab 248320 tied; NVFP4 weights.
HYBRID_2B = ModelSpec(
    name="hybrid-2b", vocab=248320, hidden=2048, inter=6144,
    layer_types=hybrid_pattern(24), gdn_heads=16, attn_heads=8, attn_kv_heads=2,
    head_dim=256, weight_format="nvfp4")

# A tiny spec with the same structure, for fast unit tests.
TINY = ModelSpec(
    name="tiny-hybrid", vocab=512, hidden=256, inter=512,
    layer_types=hybrid_pattern(4), gdn_heads=2, attn_heads=4, attn_kv_heads=2,
    head_dim=64, weight_format="int4")

SPECS = {s.name: s for s in (REDUCED_1024, HYBRID_2B, TINY)}


@dataclass(frozen=True)
class Workload:
    """A batch of scoring requests: each has a shared state and some questions."""

    name: str
    n_requests: int
    state_len: tuple[int, int]        # inclusive range; (L, L) for fixed length
    n_questions: int
    question_len: int
    options: tuple[int, ...] = field(default=(3, 2, 3))  # option count per question, cycled with kinds
    kinds: tuple[int, ...] = (1, 0, 2)                    # choice, noul, score
    seed: int = 0
    option_range: tuple[int, int] | None = None          # if set, option counts ~ U{lo..hi}, all choice


# 1024 prompts of 512 uniform-random tokens, 3 questions each (3-way choice, yes/no noul,
# 3-level score), each question a 32-token suffix ending at the decision position.
HYBRID_2B_WORKLOAD = Workload("hybrid-2b-nvfp4-1024x512x3", 1024, (512, 512), 3, 32)

# 512 requests with shared states of U[64, 2048] tokens, 32 questions of 48 tokens each,
# scoring 2-5 single-token options.
PREFIX_CACHE_WORKLOAD = Workload("hybrid-2b-nvfp4-prefix-512x32q", 512, (64, 2048), 32, 48, kinds=(1,),
                                 options=(2,), option_range=(2, 5))

# one request of 96 tokens with a single 3-way choice (the latency workload), and its batch
LATENCY_WORKLOAD = Workload("hybrid-2b-ternary-1x96", 1, (93, 93), 1, 3, kinds=(1,), options=(3,))
