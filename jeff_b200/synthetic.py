"""Seeded synthetic weights, adapters and passes for the decision hot path (no checkpoint or tokenizer exists offline).

Every tensor is drawn from its own CPU generator, seeded from (spec seed, tensor name), so the same spec gives the
same bits on any machine with the same torch build; GPU code receives copies of these CPU tensors, so the oracle and
the kernels read identical inputs.

Weights follow the reference benchmark configuration (random init as transformers initialises Qwen3.5: matrices
N(0, 0.02), RMSNorm weights 0, A_log = log U(0, 16), dt_bias = 1; transformers Qwen3_5PreTrainedModel._init_weights),
quantised to int4 ("g128z": group 128 with bf16 scale and zero; "g64": the reference's symmetric int4-g64).
`norm_noise` > 0 perturbs the norm weights (tests use it so that a kernel that ignores a norm weight fails).

Fused groups (the reference's `Lin`, fast_path.py:301-349): matrices reading the same input, concatenated along the
output. Each adapter's LoRA update of a group is block diagonal: rank 16 per adapted matrix, ranks stacked
(R = 16 x adapted matrices; the reference pads R to a power of two with zero rows, which adds zeros)."""

from __future__ import annotations

import zlib
from dataclasses import dataclass, field

import torch

from jeff_b200 import constants as C
from jeff_b200.int4 import PackedInt4, quantize_pack

DT = torch.bfloat16


def generator(seed: int, name: str) -> torch.Generator:
    """The CPU generator of one named tensor under a spec seed."""
    return torch.Generator().manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) % (2**63))


def normal(seed: int, name: str, shape: tuple[int, ...], std: float, mean: float = 0.0) -> torch.Tensor:
    return torch.randn(*shape, generator=generator(seed, name)) * std + mean


def uniform(seed: int, name: str, shape: tuple[int, ...], lo: float, hi: float) -> torch.Tensor:
    return torch.rand(*shape, generator=generator(seed, name)) * (hi - lo) + lo


@dataclass
class FusedGroup:
    """Matrices that read the same input, concatenated along the output (module docstring)."""
    names: list[str]
    sizes: list[int]
    k: int
    packed: PackedInt4
    W: torch.Tensor            # (out, k) bf16: the dequantised weights, as the standard path multiplies by them
    adapted: list[bool]        # which matrices an adapter adapts
    rank: int                  # R = 16 x adapted matrices (0: no LoRA on this group)

    @property
    def out(self) -> int:
        return sum(self.sizes)


@dataclass
class LayerWeights:
    kind: str
    norm_in: torch.Tensor      # (1024,) float32: the RMSNorm weight w (the kernels scale by 1 + w)
    norm_post: torch.Tensor
    groups: dict[str, FusedGroup]
    conv: torch.Tensor | None = None      # (6144, 4) bf16 depthwise weights
    A_log: torch.Tensor | None = None     # (16,) float32
    dt_bias: torch.Tensor | None = None   # (16,) float32
    gnorm: torch.Tensor | None = None     # (128,) bf16, plain weight (no 1 +)
    q_norm: torch.Tensor | None = None    # (256,) float32 w (1 + w applied)
    k_norm: torch.Tensor | None = None


@dataclass
class ModelSpec:
    layers: int = C.LAYERS
    vocab: int = C.VOCAB
    fmt: str = "g128z"
    seed: int = 4
    norm_noise: float = 0.0


@dataclass
class ModelWeights:
    spec: ModelSpec
    kinds: list[str]
    embed: torch.Tensor        # (vocab, 1024) bf16
    final_norm: torch.Tensor   # (1024,) float32 w
    layers: list[LayerWeights] = field(default_factory=list)


def _skeleton_pack(out: int, k: int, fmt: str) -> PackedInt4:
    """Correctly shaped placeholders of a packed group (filled later, e.g. by a broadcast from another rank)."""
    group = 64 if fmt == "g64" else 128
    columns = -(-out // C.KERNEL_COLUMNS) * C.KERNEL_COLUMNS
    zeros = None if fmt == "g64" else torch.zeros(k // group, columns, dtype=DT)
    return PackedInt4(torch.zeros(k // C.WORD, columns, dtype=torch.int32), torch.zeros(k // group, columns, dtype=DT),
                      zeros, group, out)


def _group(seed: int, prefix: str, names: list[str], sizes: list[int], k: int, fmt: str,
           skeleton: bool = False) -> FusedGroup:
    adapted = [n.rsplit(".", 1)[-1] in C.LORA_TARGETS for n in names]
    if skeleton:
        return FusedGroup([prefix + n for n in names], sizes, k, _skeleton_pack(sum(sizes), k, fmt),
                          torch.empty(0, dtype=DT), adapted, C.LORA_RANK * sum(adapted))
    ws = [normal(seed, prefix + n, (s, k), 0.02) for n, s in zip(names, sizes, strict=True)]
    packed, deq = quantize_pack(torch.cat(ws), fmt)
    return FusedGroup([prefix + n for n in names], sizes, k, packed, deq, adapted, C.LORA_RANK * sum(adapted))


def make_model(spec: ModelSpec, skeleton: bool = False) -> ModelWeights:
    """The synthetic base of `spec` (module docstring). The layer kinds repeat (GDN, GDN, GDN, attention).
    skeleton=True: the same shapes with placeholder values, for a replica whose weights arrive by broadcast."""
    s = spec.seed
    kinds = [C.LAYER_KINDS[i % 4] for i in range(spec.layers)]
    embed = (torch.zeros(spec.vocab, C.HIDDEN, dtype=DT) if skeleton
             else normal(s, "embed_tokens", (spec.vocab, C.HIDDEN), 0.02).to(DT))

    def norm(name: str, n: int) -> torch.Tensor:
        if spec.norm_noise:
            return normal(s, name, (n,), spec.norm_noise)
        return torch.zeros(n)

    model = ModelWeights(spec, kinds, embed, norm("norm", C.HIDDEN))
    for i, kind in enumerate(kinds):
        p = f"layers.{i}."
        groups = {
            "mlp_in": _group(s, p, ["mlp.gate_proj", "mlp.up_proj"], [C.INTER, C.INTER], C.HIDDEN, spec.fmt, skeleton),
            "mlp_down": _group(s, p, ["mlp.down_proj"], [C.HIDDEN], C.INTER, spec.fmt, skeleton),
        }
        layer = LayerWeights(kind, norm(p + "input_layernorm", C.HIDDEN), norm(p + "post_attention_layernorm", C.HIDDEN),
                             groups)
        if kind == "linear_attention":
            la = "linear_attn."
            groups["proj"] = _group(s, p, [la + "in_proj_qkv", la + "in_proj_z", la + "in_proj_b", la + "in_proj_a"],
                                    [C.QKV_DIM, C.Z_DIM, C.NV, C.NV], C.HIDDEN, spec.fmt, skeleton)
            groups["out"] = _group(s, p, [la + "out_proj"], [C.HIDDEN], C.NV * C.DV, spec.fmt, skeleton)
            layer.conv = uniform(s, p + la + "conv1d", (C.QKV_DIM, C.CONV), -0.5, 0.5).to(DT)
            layer.A_log = torch.log(uniform(s, p + la + "A_log", (C.NV,), 0.0, 16.0).clamp_min(1e-3))
            layer.dt_bias = torch.ones(C.NV) + (normal(s, p + la + "dt_bias", (C.NV,), spec.norm_noise)
                                                if spec.norm_noise else 0.0)
            g = torch.ones(C.DV) + (normal(s, p + la + "norm", (C.DV,), spec.norm_noise) if spec.norm_noise else 0.0)
            layer.gnorm = g.to(DT)
        else:
            sa = "self_attn."
            groups["proj"] = _group(s, p, [sa + "q_proj", sa + "k_proj", sa + "v_proj"],
                                    [C.NQ * 2 * C.HD, C.NKV * C.HD, C.NKV * C.HD], C.HIDDEN, spec.fmt, skeleton)
            groups["out"] = _group(s, p, [sa + "o_proj"], [C.HIDDEN], C.NQ * C.HD, spec.fmt, skeleton)
            layer.q_norm = norm(p + sa + "q_norm", C.HD)
            layer.k_norm = norm(p + sa + "k_norm", C.HD)
        model.layers.append(layer)
    return model


@dataclass
class AdapterWeights:
    """One adapter: per fused group (layer, group key) the stacked A (R, k) and block-diagonal B (out, R), both bf16
    with the scale alpha / r folded into B (the reference LoraLinear's "model" precision, lora.py:204-210); its
    readout (255, 1024) bf16 and temperature."""
    name: str
    lora: dict[tuple[int, str], tuple[torch.Tensor, torch.Tensor]]
    readout: torch.Tensor
    temperature: float
    matrices: dict[str, tuple[torch.Tensor, torch.Tensor]] = field(default_factory=dict)  # per matrix (A, sB)


def make_adapter(model: ModelWeights, index: int, seed: int, alpha: float = 32.0,
                 skeleton: bool = False) -> AdapterWeights:
    """A rank-16 adapter of every LoRA target: A ~ N(0, 0.02), B ~ N(0, 0.01), scale alpha / 16; readout
    N(0, 0.02); temperature U(0.5, 2). skeleton=True: zeros of the same shapes (filled by a broadcast)."""
    name = f"adapter-{index}"
    scale = alpha / C.LORA_RANK
    lora: dict[tuple[int, str], tuple[torch.Tensor, torch.Tensor]] = {}
    matrices: dict[str, tuple[torch.Tensor, torch.Tensor]] = {}
    for i, layer in enumerate(model.layers):
        for key, grp in layer.groups.items():
            if not grp.rank:
                continue
            a_all = torch.zeros(grp.rank, grp.k, dtype=DT)
            b_all = torch.zeros(grp.out, grp.rank, dtype=DT)
            r0 = o0 = 0
            for mname, size, adapted in zip(grp.names, grp.sizes, grp.adapted, strict=True):
                if adapted and skeleton:
                    r0 += C.LORA_RANK
                elif adapted:
                    a = normal(seed, f"{name}/{mname}/A", (C.LORA_RANK, grp.k), 0.02).to(DT)
                    b = (normal(seed, f"{name}/{mname}/B", (size, C.LORA_RANK), 0.01) * scale).to(DT)
                    a_all[r0:r0 + C.LORA_RANK] = a
                    b_all[o0:o0 + size, r0:r0 + C.LORA_RANK] = b
                    matrices[mname] = (a, b)
                    r0 += C.LORA_RANK
                o0 += size
            lora[(i, key)] = (a_all, b_all)
    if skeleton:
        return AdapterWeights(name, lora, torch.zeros(C.READOUT_ROWS, C.HIDDEN, dtype=DT), 1.0, matrices)
    readout = normal(seed, f"{name}/readout", (C.READOUT_ROWS, C.HIDDEN), 0.02).to(DT)
    temperature = float(uniform(seed, f"{name}/temperature", (1,), 0.5, 2.0)[0])
    return AdapterWeights(name, lora, readout, temperature, matrices)


def base_head(model: ModelWeights) -> tuple[torch.Tensor, float]:
    """The base's own readout (adapter row 0) and temperature."""
    return normal(model.spec.seed, "readout", (C.READOUT_ROWS, C.HIDDEN), 0.02).to(DT), 1.0


@dataclass
class PassRows:
    """One decision pass's rows: adapter index (0 the base, i the i-th adapter), prefix token ids, new token ids,
    option count."""
    adapters: list[int]
    prefixes: list[list[int]]
    new_ids: list[list[int]]
    counts: list[int]


def make_cfg4_rows(seed: int, calls: int = 64, new_tokens: int = 128, prefix_tokens: int = 512, adapters: int = 16,
                   vocab: int = C.VOCAB) -> PassRows:
    """The reference benchmark configuration 4: `calls` calls of `new_tokens` tokens, each on its adapter's shared
    `prefix_tokens`-token prefix (one prefix per adapter), adapters uniform over 1..adapters, option counts
    U{2..32}, token ids uniform over the vocabulary."""
    g = generator(seed, "cfg4/rows")
    prefix_of = {a: torch.randint(0, vocab, (prefix_tokens,), generator=generator(seed, f"cfg4/prefix/{a}")).tolist()
                 for a in range(1, adapters + 1)}
    chosen = torch.randint(1, adapters + 1, (calls,), generator=g).tolist()
    new = torch.randint(0, vocab, (calls, new_tokens), generator=g).tolist()
    counts = torch.randint(2, 33, (calls,), generator=g).tolist()
    return PassRows(chosen, [prefix_of[a] for a in chosen], new, counts)


# ---------------------------------------------------------------- configuration 2: the projection sweep

# one decoder layer's projections (name, k, n): q/k/v/o, gate/up/down, and the attention input as the reference runs
# it (q with its output gate, 1024 -> 4096)
CFG2_SHAPES = (("q", 1024, 2048), ("k", 1024, 512), ("v", 1024, 512), ("o", 2048, 1024), ("gate", 1024, 3584),
               ("up", 1024, 3584), ("down", 3584, 1024), ("q_gate", 1024, 4096))


def cfg2_lengths(seed: int = 2, requests: int = 64, total: int = 4096, lo: int = 32, hi: int = 128) -> list[int]:
    """The reference benchmark configuration 2's request lengths: `requests` draws from U{lo..hi}, then moved by one
    token at a time, round robin over the requests and staying inside [lo, hi], until they sum to `total`."""
    if not requests * lo <= total <= requests * hi:
        raise ValueError(f"{requests} lengths in [{lo}, {hi}] cannot sum to {total}")
    lengths = torch.randint(lo, hi + 1, (requests,), generator=generator(seed, "cfg2/lengths")).tolist()
    i = 0
    while (gap := total - sum(lengths)) != 0:
        step = 1 if gap > 0 else -1
        if lo <= lengths[i] + step <= hi:
            lengths[i] += step
        i = (i + 1) % requests
    return lengths


def cfg2_adapters(seed: int = 2, requests: int = 64, adapters: int = 8) -> list[int]:
    """Each request's adapter: pool rows 1..adapters uniformly at random (row 0 is the base, no update)."""
    return torch.randint(1, adapters + 1, (requests,), generator=generator(seed, "cfg2/adapters")).tolist()


@dataclass
class Cfg2Projection:
    """One projection of the sweep: packed int4 weights (group 128 with bf16 scale and zero), the LoRA pools with
    row 0 zeros and rows 1..8 rank-16 adapters (A ~ N(0, 0.02), B ~ N(0, 0.01) with alpha / r = 2 folded in), and
    the packed pass's input x (tokens, k) ~ N(0, 1), bf16."""
    name: str
    k: int
    n: int
    packed: PackedInt4
    W: torch.Tensor
    lora_a: torch.Tensor     # (9, 16, k)
    lora_b: torch.Tensor     # (9, columns, 16)
    x: torch.Tensor


def cfg2_projection(name: str, k: int, n: int, tokens: int = 4096, seed: int = 2, adapters: int = 8,
                    rank: int = C.LORA_RANK, alpha: float = 32.0) -> Cfg2Projection:
    w = normal(seed, f"cfg2/{name}/W", (n, k), 0.02)
    packed, W = quantize_pack(w, "g128z")
    lora_a = torch.zeros(adapters + 1, rank, k, dtype=DT)
    lora_b = torch.zeros(adapters + 1, packed.columns, rank, dtype=DT)
    lora_a[1:] = normal(seed, f"cfg2/{name}/A", (adapters, rank, k), 0.02).to(DT)
    lora_b[1:, :n] = (normal(seed, f"cfg2/{name}/B", (adapters, n, rank), 0.01) * (alpha / rank)).to(DT)
    x = normal(seed, f"cfg2/{name}/x", (tokens, k), 1.0).to(DT)
    return Cfg2Projection(name, k, n, packed, W, lora_a, lora_b, x)
