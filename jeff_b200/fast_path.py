"""The hot path's weights, stacked adapter pools and prefix pool on one GPU (the reference's engine/fast_path.py
FastPath, :366-570, and Lin, :301-349), for the B200 kernels.

- DeviceLin: one fused group (matrices reading the same input, concatenated along the output) as packed int4
  (the reference's kernel word layout, int4.KernelInt4) with its LoRA pools: lora_a (rows, R, k) and
  lora_b (rows, columns, R) bf16, row 0 the base (zeros, which leave the product unchanged), rows 1.. the loaded
  adapters. R = 16 per adapted matrix of the group, block diagonal.
- FastPath: every layer's groups and small weights (norm weights as 1 + w in float32, the depthwise convolution as
  (4, 6144) float32, -exp(A_log), dt_bias, the gated norm weight, q/k norm weights), the embedding, the readout and
  temperature pools (rows, 255, 1024) / (rows,), and the PrefixPool. Adapters are added into the lowest free row
  and removed by freeing it; either forgets that row's cached prefixes (fast_path.py:492-540)."""

from __future__ import annotations

import bisect

import torch

from jeff_b200 import constants as C
from jeff_b200 import kernels
from jeff_b200.prefix_pool import PrefixPool, pool_pages
from jeff_b200.synthetic import AdapterWeights, FusedGroup, ModelWeights

DT = torch.bfloat16
MAX_ADAPTERS = 255   # pool rows (adapters + the base's row 0) the product's gathered LoRA expand can hold: 256


def swiglu_order(inter: int, block: int = 64) -> torch.Tensor:
    """Column order of a [gate | up] group for the fused SwiGLU epilogue: gate block j (64 columns), then up block
    j, for j = 0 .. inter / 64 - 1, so every 128-column tile of the product holds matching gate and up columns."""
    idx = []
    for j in range(inter // block):
        idx += list(range(j * block, (j + 1) * block)) + list(range(inter + j * block, inter + (j + 1) * block))
    return torch.tensor(idx, dtype=torch.long)


class DeviceLin:
    def __init__(self, grp: FusedGroup, pool_rows: int, device: torch.device, swiglu: bool = False) -> None:
        p = grp.packed
        self.names = grp.names
        self.k = grp.k
        self.out = grp.out
        self.group = p.group
        self.columns = p.columns
        self.swiglu = swiglu
        words, scales, zeros = p.words, p.scales, p.zeros
        self.order: torch.Tensor | None = None
        if swiglu:
            if len(grp.sizes) != 2 or grp.sizes[0] != grp.sizes[1] or grp.sizes[0] % 64 or p.columns != grp.out:
                raise ValueError(f"{', '.join(grp.names)}: the SwiGLU epilogue needs a [gate | up] group of equal "
                                 "halves, a multiple of 64 wide")
            self.order = swiglu_order(grp.sizes[0])
            words, scales = words[:, self.order], scales[:, self.order]
            zeros = zeros[:, self.order] if zeros is not None else None
        self.words = kernels.int4_repack(words.contiguous().to(device))     # the kernels' word layout
        self.scales = scales.contiguous().to(device)
        self.zeros = zeros.contiguous().to(device) if zeros is not None else None
        self.rank = grp.rank
        self.lora_a = torch.zeros(pool_rows, self.rank, self.k, dtype=DT, device=device) if self.rank else None
        self.lora_b = torch.zeros(pool_rows, self.columns, self.rank, dtype=DT, device=device) if self.rank else None

    def write(self, row: int, a: torch.Tensor, b: torch.Tensor) -> None:
        """Adapter row `row` := (A (R, k), B (out, R)); padding columns of B stay zero."""
        if not self.rank:
            return
        assert self.lora_a is not None and self.lora_b is not None
        if tuple(a.shape) != (self.rank, self.k) or tuple(b.shape) != (self.out, self.rank):
            raise ValueError(f"{', '.join(self.names)}: LoRA shapes {tuple(a.shape)} and {tuple(b.shape)} do not fit "
                             f"rank {self.rank}, {self.k} inputs, {self.out} outputs")
        self.lora_a[row].copy_(a)
        self.lora_b[row].zero_()
        if self.order is not None:
            b = b[self.order.to(b.device)]
        self.lora_b[row, :self.out].copy_(b)

    def clear(self, row: int) -> None:
        if self.rank:
            assert self.lora_a is not None and self.lora_b is not None
            self.lora_a[row].zero_()
            self.lora_b[row].zero_()

    def __call__(self, x: torch.Tensor, adapters: torch.Tensor, row_len: int, mid: torch.Tensor | None,
                 y: torch.Tensor | None = None, split: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
        """y = the group's product of x with each token's adapter; `split` (fp32 slices, int32 counters): the
        split-K scratch that lets a pass too small to fill the GPU spread each tile's K over several CTAs."""
        m = x.shape[0]
        mid_v = mid[:m * self.rank].view(m, self.rank) if (mid is not None and self.rank) else None
        return kernels.int4_product(x, self.words, self.scales, self.zeros, self.group, self.out, self.lora_a,
                                    self.lora_b, adapters, row_len, mid_v, y, swiglu=self.swiglu, split=split)

    def nbytes(self) -> int:
        n = self.words.numel() * 4 + self.scales.numel() * 2 + (self.zeros.numel() * 2 if self.zeros is not None else 0)
        return n


class FastPath:
    def __init__(self, model: ModelWeights, max_adapters: int, prefix_pool_mb: int | None = None,
                 pool_pages_count: int | None = None, device: str | torch.device = "cuda",
                 base_readout: tuple[torch.Tensor, float] | None = None) -> None:
        if max_adapters < 1:
            raise ValueError(f"max_adapters={max_adapters}: the fast path needs room for at least one adapter")
        if max_adapters > MAX_ADAPTERS:
            raise ValueError(f"max_adapters={max_adapters}: the fast path holds at most {MAX_ADAPTERS} adapters (the "
                             "product gathers a pass's LoRA updates from at most 256 pool rows, the base's included)")
        self.device = torch.device(device)
        self.model = model
        self.max_adapters = max_adapters
        rows = max_adapters + 1
        dev = self.device
        self.embed = model.embed.to(dev)
        self.final_w1 = (1.0 + model.final_norm.float()).to(dev)
        self.kinds = list(model.kinds)
        self.layers: list[dict] = []
        self.lins: list[DeviceLin] = []
        for lw in model.layers:
            layer: dict = {"kind": lw.kind, "norm_in": (1.0 + lw.norm_in.float()).to(dev),
                           "norm_post": (1.0 + lw.norm_post.float()).to(dev)}
            for key, grp in lw.groups.items():
                lin = DeviceLin(grp, rows, dev, swiglu=(key == "mlp_in"))
                layer[key] = lin
                self.lins.append(lin)
            if lw.kind == "linear_attention":
                layer["conv"] = lw.conv.float().T.contiguous().to(dev)          # (4, 6144)
                layer["a_neg"] = (-torch.exp(lw.A_log.float())).to(dev)
                layer["dt_bias"] = lw.dt_bias.float().to(dev)
                layer["gnorm"] = lw.gnorm.to(DT).to(dev)
            else:
                layer["q_w1"] = (1.0 + lw.q_norm.float()).to(dev)
                layer["k_w1"] = (1.0 + lw.k_norm.float()).to(dev)
            self.layers.append(layer)
        self.gdn_layers = [i for i, k in enumerate(self.kinds) if k == "linear_attention"]
        self.attn_layers = [i for i, k in enumerate(self.kinds) if k == "full_attention"]
        self.inv_freq = (1.0 / (C.ROPE_THETA ** (torch.arange(0, C.ROT, 2, dtype=torch.float32) / C.ROT))).to(dev)
        self.readout_pool = torch.zeros(rows, C.READOUT_ROWS, C.HIDDEN, dtype=DT, device=dev)
        self.temp_pool = torch.ones(rows, dtype=torch.float32, device=dev)
        if base_readout is not None:
            self.readout_pool[0].copy_(base_readout[0])
            self.temp_pool[0] = float(base_readout[1])
        self.adapter_index: dict[str | None, int] = {None: 0}
        self.free_rows = list(range(1, rows))
        if pool_pages_count is None:
            if prefix_pool_mb is None:
                raise ValueError("FastPath needs prefix_pool_mb or pool_pages_count")
            pool_pages_count = pool_pages(prefix_pool_mb)
        self.prefixes = PrefixPool(pool_pages_count, dev)
        self.max_rank = max(lin.rank for lin in self.lins)

    # ------------------------------------------------------------ adapters

    def add_adapter(self, adapter: AdapterWeights) -> int:
        """Pack an adapter (LoRA matrices, readout, temperature) into the lowest free row; returns the row."""
        if adapter.name in self.adapter_index:
            raise ValueError(f"Adapter {adapter.name} is already in the fast path")
        if not self.free_rows:
            raise ValueError(f"The fast path holds at most {self.max_adapters} adapters (--max-adapters "
                             f"{self.max_adapters}) and all {len(self.adapter_index) - 1} are loaded; remove one first, "
                             "or restart the engine with a larger --max-adapters")
        index = self.free_rows[0]
        for li, layer in enumerate(self.layers):
            for key in ("proj", "out", "mlp_in", "mlp_down"):
                lin: DeviceLin = layer[key]
                pair = adapter.lora.get((li, key))
                if pair is None:
                    lin.clear(index)
                else:
                    lin.write(index, pair[0].to(self.device), pair[1].to(self.device))
        self.readout_pool[index].copy_(adapter.readout)
        self.temp_pool[index] = float(adapter.temperature)
        self.free_rows.pop(0)
        self.adapter_index[adapter.name] = index
        self.prefixes.forget_adapter(index)
        return index

    def remove_adapter(self, name: str) -> None:
        index = self.adapter_index.pop(name)
        bisect.insort(self.free_rows, index)
        self.prefixes.forget_adapter(index)

    def index(self, adapter: str | None) -> int:
        if adapter not in self.adapter_index:
            raise ValueError(f"Adapter {adapter!r} is not loaded in the fast path "
                             f"(loaded: {sorted(str(a) for a in self.adapter_index)})")
        return self.adapter_index[adapter]

    def weight_bytes(self) -> int:
        return sum(lin.nbytes() for lin in self.lins)

    def adapter_tensors(self, index: int) -> list[torch.Tensor]:
        """The device memory of one adapter row, as views in a fixed order: every group's LoRA A and B rows, its
        readout rows and its temperature (what an adapter add changes, so what the replicas re-broadcast)."""
        if not 0 <= index <= self.max_adapters:
            raise ValueError(f"Adapter row {index} is outside the pools' rows 0..{self.max_adapters}")
        out = [self.readout_pool[index], self.temp_pool[index:index + 1]]
        for lin in self.lins:
            if lin.rank:
                assert lin.lora_a is not None and lin.lora_b is not None
                out += [lin.lora_a[index], lin.lora_b[index]]
        return out

    def tensors(self) -> list[torch.Tensor]:
        """Every device tensor of the weights and adapter pools, in a fixed order (the NCCL broadcast at load)."""
        out = [self.embed, self.final_w1, self.readout_pool, self.temp_pool, self.inv_freq]
        for layer in self.layers:
            for key in sorted(layer):
                value = layer[key]
                if isinstance(value, torch.Tensor):
                    out.append(value)
                elif isinstance(value, DeviceLin):
                    out += [t for t in (value.words, value.scales, value.zeros, value.lora_a, value.lora_b)
                            if t is not None]
        return out
