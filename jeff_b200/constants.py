"""The model layout and the batching constants of the decision hot path.

The layout is the Qwen3.5-0.8B hybrid the reference's fast path is built for (reference
runtime/python/src/jeff_runtime/engine/fast_path.py:58-69 and the checks at :386-395): 24 decoder layers in
blocks of three Gated DeltaNet layers and one gated full-attention layer, hidden 1024, SwiGLU 3584, Gated DeltaNet
16 heads of 128 (keys and values), attention 8 query heads and 2 key/value heads of 256, partial RoPE on the
first 64 dimensions of each head, RMSNorm epsilon 1e-6 with (1 + weight) scaling.

Batching (reference engine/batched_path.py:97-100, engine/prepare.py:355): a pass holds B rows of N new tokens each,
N from NEW_BUCKETS, B from BATCH_BUCKETS, B * N <= MAX_PASS_TOKENS."""

from __future__ import annotations

EPS = 1e-6
HIDDEN = 1024
INTER = 3584
LAYERS = 24
NK, DK, NV, DV = 16, 128, 16, 128          # Gated DeltaNet heads (keys and values share the head count here)
NQ, NKV, HD, ROT = 8, 2, 256, 64           # attention heads, head dim, rotary dims
CONV = 4                                   # causal depthwise convolution width
QKV_DIM = NK * DK * 2 + NV * DV            # 6144: the convolved q | k | v channels
Z_DIM = NV * DV                            # 2048: the output gate z of the gated norm
GDN_PROJ = QKV_DIM + Z_DIM + 2 * NV        # 8224: in_proj_qkv | in_proj_z | in_proj_b | in_proj_a
ATTN_PROJ = NQ * 2 * HD + 2 * NKV * HD     # 5120: q_proj (query and gate interleaved per head) | k_proj | v_proj
READOUT_ROWS = 255
VOCAB = 151936
ROPE_THETA = 1e7
LAYER_KINDS = tuple(("full_attention" if i % 4 == 3 else "linear_attention") for i in range(LAYERS))
GDN_LAYERS = sum(1 for k in LAYER_KINDS if k == "linear_attention")   # 18
ATTN_LAYERS = LAYERS - GDN_LAYERS                                       # 6

# The ten matrices an adapter adapts (reference fast_path.py:68-69).
LORA_TARGETS = ("in_proj_qkv", "in_proj_z", "out_proj", "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj",
                "up_proj", "down_proj")
LORA_RANK = 16

NEW_BUCKETS = (32, 64, 128, 256, 512, 1024)
BATCH_BUCKETS = (1, 2, 4, 8, 16, 32, 64)
MAX_PASS_TOKENS = 16384
PREFIX_BUCKETS = (64, 128, 256, 512, 768, 1024, 1536, 2048, 3072, 4096, 6144, 8192)
LONGEST_PREFIX_TOKENS = 8192
META = 5   # per-row numbers of a decision pass's packed input: slot, adapter, prefix length, last, count

KERNEL_COLUMNS = 64   # a fused group's outputs are padded to a multiple of this in the int4 kernel layout
WORD = 8              # 4-bit integers per int32 word of the kernel layout
