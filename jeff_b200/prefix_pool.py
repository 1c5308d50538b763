"""The paged prefix-state pool: every cached prefix's state in device memory at fixed addresses, read in place by
the decision kernels through per-row block tables.

Mirrors the reference's engine/prefix_pool.py (PrefixShapes :55-98, PrefixPool :150-322) in behaviour, numbers and
error wording, so the engine above it behaves the same:
- uniform pages of `page_bytes` (what PAGE_TOKENS tokens of attention keys and values take over all attention layers;
  393,216 B for the 0.8B layout), three typed views of one allocation: kv[page, attn layer, K|V, token, head, dim]
  (bf16), state[page, head, key dim, value dim] (fp32, a whole number of Gated DeltaNet heads per page) and
  conv[page, layer, 3, channels] (bf16);
- a prefix of p tokens takes state_pages + conv_pages + ceil(p / PAGE_TOKENS) pages, listed in its block table in
  that order; slot 0 is the empty prefix (its fixed entries all name page 1, all zeros, never written), page 0 is a
  sink the prefix pass writes padding to and nothing reads;
- prefixes are keyed by (adapter row, prefix text); least recently used first out, never a pinned one.

Host bookkeeping is plain Python on the engine's GPU thread (nothing here is thread safe). The page memory is one
device allocation made at start; the block tables live on the host and in a device copy (`tables`)."""

from __future__ import annotations

import heapq
from collections import OrderedDict
from collections.abc import Iterable
from dataclasses import dataclass

import torch

from jeff_b200 import constants as C

PAGE_TOKENS = 32
SINK_PAGE, ZERO_PAGE = 0, 1
RESERVED_PAGES = 2


class EngineError(RuntimeError):
    """A request the engine cannot serve as configured (the reference's jeff.errors.EngineError role)."""


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


@dataclass(frozen=True)
class PrefixShapes:
    gdn_layers: int
    conv: tuple[int, int]
    state: tuple[int, int, int]
    attn_layers: int
    kv: tuple[int, int]
    page_tokens: int = PAGE_TOKENS

    @property
    def page_bytes(self) -> int:
        return self.attn_layers * 2 * self.page_tokens * self.kv[0] * self.kv[1] * 2

    @property
    def state_pages(self) -> int:
        heads = self.gdn_layers * self.state[0]
        return _cdiv(heads, self.page_bytes // (self.state[1] * self.state[2] * 4))

    @property
    def heads_per_page(self) -> int:
        return self.gdn_layers * self.state[0] // self.state_pages

    @property
    def conv_pages(self) -> int:
        return _cdiv(self.gdn_layers, self.page_bytes // (self.conv[0] * self.conv[1] * 2))

    @property
    def layers_per_conv_page(self) -> int:
        return self.gdn_layers // self.conv_pages

    @property
    def fixed_pages(self) -> int:
        return self.state_pages + self.conv_pages

    def pages_per_prefix(self, tokens: int) -> int:
        return self.fixed_pages + _cdiv(tokens, self.page_tokens)

    def check(self) -> None:
        heads = self.gdn_layers * self.state[0]
        if self.page_bytes % 4 or heads % self.state_pages or self.gdn_layers % self.conv_pages:
            raise ValueError(f"{self}: the states and convolution tails do not split evenly into pages")


FAST_PATH_SHAPES = PrefixShapes(gdn_layers=C.GDN_LAYERS, conv=(C.CONV - 1, C.QKV_DIM), state=(C.NV, C.DK, C.DV),
                                attn_layers=C.ATTN_LAYERS, kv=(C.NKV, C.HD))


def pool_pages(prefix_pool_mb: int, shapes: PrefixShapes = FAST_PATH_SHAPES) -> int:
    return prefix_pool_mb * 2**20 // shapes.page_bytes


def prefixes_held(prefix_pool_mb: int, tokens: int, shapes: PrefixShapes = FAST_PATH_SHAPES) -> int:
    return max(0, pool_pages(prefix_pool_mb, shapes) - RESERVED_PAGES) // shapes.pages_per_prefix(tokens)


def prefix_pool_mb_for(rows: int, shapes: PrefixShapes = FAST_PATH_SHAPES) -> int:
    pages = rows * shapes.pages_per_prefix(C.LONGEST_PREFIX_TOKENS) + RESERVED_PAGES
    return _cdiv(pages * shapes.page_bytes, 2**20)


def check_pool_size(prefix_pool_mb: object) -> int:
    smallest = prefix_pool_mb_for(1)
    if isinstance(prefix_pool_mb, bool) or not isinstance(prefix_pool_mb, int) or prefix_pool_mb < smallest:
        raise EngineError(f"--prefix-pool-mb {prefix_pool_mb!r}: give a whole number of megabytes, at least {smallest} "
                          f"(one prefix of {C.LONGEST_PREFIX_TOKENS} tokens); for example 2048 holds "
                          f"{prefixes_held(2048, 1000)} prefixes of 1,000 tokens")
    return prefix_pool_mb


def check_pool_holds(prefix_pool_mb: int, max_batch_rows: int) -> None:
    needed = prefix_pool_mb_for(max_batch_rows)
    if prefix_pool_mb < needed:
        raise EngineError(
            f"--prefix-pool-mb {prefix_pool_mb} cannot hold --max-batch-rows {max_batch_rows} prefixes of "
            f"{C.LONGEST_PREFIX_TOKENS} tokens (the longest prefix) at once, as one pass of {max_batch_rows} rows may "
            f"need; give --prefix-pool-mb at least {needed}, or lower --max-batch-rows.")


@dataclass
class _Entry:
    key: tuple[int, str]
    length: int
    pages: list[int]


class PrefixPool:
    """Pages allocated once on `device`, and which prefix holds which (module docstring)."""

    def __init__(self, pages: int, device: str | torch.device = "cuda", *,
                 shapes: PrefixShapes = FAST_PATH_SHAPES, max_prefix_tokens: int = C.LONGEST_PREFIX_TOKENS) -> None:
        shapes.check()
        if pages < RESERVED_PAGES + shapes.fixed_pages:
            raise ValueError(f"A prefix pool of {pages} pages cannot hold a single prefix ({shapes.fixed_pages} pages "
                             "and the 2 reserved)")
        self.shapes, self.pages, self.page_tokens = shapes, pages, shapes.page_tokens
        self.fixed_pages = shapes.fixed_pages
        self.slots = 1 + (pages - RESERVED_PAGES) // self.fixed_pages
        words = shapes.page_bytes // 4
        self.data = torch.zeros(pages, words, device=device, dtype=torch.int32)
        halves = self.data.view(torch.bfloat16)
        self.kv = halves.view(pages, shapes.attn_layers, 2, self.page_tokens, *shapes.kv)
        heads = shapes.heads_per_page
        self.state = self.data.view(torch.float32)[:, :heads * shapes.state[1] * shapes.state[2]].view(
            pages, heads, shapes.state[1], shapes.state[2])
        layers = shapes.layers_per_conv_page
        self.conv = halves[:, :layers * shapes.conv[0] * shapes.conv[1]].view(pages, layers, *shapes.conv)
        self.max_prefix_tokens = max_prefix_tokens
        self.max_kv_pages = _cdiv(max_prefix_tokens, self.page_tokens)
        self.width = self.fixed_pages + self.max_kv_pages
        self.tables = torch.zeros(self.slots, self.width, device=device, dtype=torch.int32)
        self.tables[0, :self.fixed_pages] = ZERO_PAGE
        self._entries: OrderedDict[tuple[int, str], int] = OrderedDict()
        self._slot: dict[int, _Entry] = {}
        self._pinned: dict[int, int] = {}
        self._free_slots = list(range(1, self.slots))
        self._free_pages = list(range(pages - 1, RESERVED_PAGES - 1, -1))

    @property
    def nbytes(self) -> int:
        return self.data.numel() * self.data.element_size()

    def __len__(self) -> int:
        return len(self._entries)

    def free_slot_count(self) -> int:
        return len(self._free_slots)

    def free_page_count(self) -> int:
        return len(self._free_pages)

    def lookup(self, adapter_index: int, text: str) -> int | None:
        key = (adapter_index, text)
        slot = self._entries.get(key)
        if slot is not None:
            self._entries.move_to_end(key)
        return slot

    def reserve(self, adapter_index: int, text: str, tokens: int) -> int:
        key = (adapter_index, text)
        if key in self._entries:
            raise ValueError(f"Prefix of adapter row {adapter_index} is already in the pool "
                             f"(slot {self._entries[key]})")
        if tokens > self.max_prefix_tokens:
            raise ValueError(f"A prefix of {tokens} tokens is longer than the longest prefix ({self.max_prefix_tokens})")
        wanted = self.shapes.pages_per_prefix(tokens)
        if wanted > self.pages - RESERVED_PAGES:
            raise EngineError(f"A prefix of {tokens} tokens needs {wanted} pages; the prefix pool has "
                              f"{self.pages - RESERVED_PAGES} in all (raise --prefix-pool-mb)")
        evictable = [slot for slot in self._entries.values() if slot not in self._pinned]
        if (len(self._free_slots) + len(evictable) < 1
                or len(self._free_pages) + sum(len(self._slot[s].pages) for s in evictable) < wanted):
            raise EngineError(f"No room in the prefix pool for a prefix of {tokens} tokens ({wanted} pages): "
                              f"{len(self._pinned)} prefixes are pinned by the pass being formed, and the others free "
                              f"too few pages. Lower --max-batch-rows or raise --prefix-pool-mb.")
        for slot in evictable:
            if self._free_slots and len(self._free_pages) >= wanted:
                break
            self._free(slot)
        slot = heapq.heappop(self._free_slots)
        pages = [self._free_pages.pop() for _ in range(wanted)]
        self.tables[slot, :wanted] = torch.tensor(pages, dtype=torch.int32)
        self._slot[slot] = _Entry(key, tokens, pages)
        self._entries[key] = slot
        return slot

    def release(self, slot: int) -> None:
        if slot in self._pinned:
            raise ValueError(f"Prefix slot {slot} is pinned")
        self._in_use(slot)
        self._free(slot)

    def block_table(self, slot: int) -> list[int]:
        return [ZERO_PAGE] * self.fixed_pages if slot == 0 else list(self._in_use(slot).pages)

    def key(self, slot: int) -> tuple[int, str]:
        return self._in_use(slot).key

    def length(self, slot: int) -> int:
        return 0 if slot == 0 else self._in_use(slot).length

    def pin(self, slots: Iterable[int]) -> None:
        slots = list(slots)
        for slot in slots:
            self._in_use(slot)
        for slot in slots:
            self._pinned[slot] = self._pinned.get(slot, 0) + 1

    def unpin(self, slots: Iterable[int]) -> None:
        for slot in slots:
            count = self._pinned.get(slot)
            if count is None:
                raise ValueError(f"Prefix slot {slot} is not pinned")
            if count == 1:
                del self._pinned[slot]
            else:
                self._pinned[slot] = count - 1

    def forget_adapter(self, adapter_index: int) -> None:
        slots = [slot for (index, _), slot in self._entries.items() if index == adapter_index]
        pinned = [slot for slot in slots if slot in self._pinned]
        if pinned:
            raise ValueError(f"Adapter row {adapter_index} has pinned prefix slots {pinned}: an adapter changes only "
                             "between passes")
        for slot in slots:
            self._free(slot)

    def gather(self, slot: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """A prefix's state copied out of its pages: conv (layers, 3, channels), state (layers, heads, key dim,
        value dim), kv (attention layers, 2, prefix length, heads, dim). For tests and inspection."""
        shapes = self.shapes
        s, c = shapes.state_pages, shapes.conv_pages
        table = self.tables[slot].long()
        state = self.state.index_select(0, table[:s]).reshape(shapes.gdn_layers, *shapes.state)
        conv = self.conv.index_select(0, table[s:s + c]).reshape(shapes.gdn_layers, *shapes.conv)
        p = self.length(slot)
        n = _cdiv(p, self.page_tokens)
        kv = self.kv.index_select(0, table[s + c:s + c + n]).permute(1, 2, 0, 3, 4, 5)
        return conv, state, kv.reshape(shapes.attn_layers, 2, n * self.page_tokens, *shapes.kv)[:, :, :p]

    def write(self, slot: int, conv: torch.Tensor, state: torch.Tensor, kv: torch.Tensor) -> None:
        """Write one prefix's state into its slot's pages (tests and tools; the prefix pass writes in its kernels).
        conv (layers, 3, channels), state (layers, heads, kd, vd), kv (attention layers, 2, tokens, heads, dim)."""
        shapes = self.shapes
        s, c = shapes.state_pages, shapes.conv_pages
        table = self.tables[slot].long()
        self.state.index_copy_(0, table[:s], state.reshape(s, *self.state.shape[1:]).to(self.state))
        self.conv.index_copy_(0, table[s:s + c], conv.reshape(c, *self.conv.shape[1:]).to(self.conv))
        p = kv.shape[2]
        n = _cdiv(p, self.page_tokens)
        if n:
            padded = torch.zeros(shapes.attn_layers, 2, n * self.page_tokens, *shapes.kv, dtype=self.kv.dtype,
                                 device=self.kv.device)
            padded[:, :, :p] = kv.to(self.kv)
            self.kv.index_copy_(0, table[s + c:s + c + n],
                                padded.view(shapes.attn_layers, 2, n, self.page_tokens, *shapes.kv)
                                .permute(2, 0, 1, 3, 4, 5).contiguous())

    def _in_use(self, slot: int) -> _Entry:
        entry = self._slot.get(slot)
        if entry is None:
            raise ValueError(f"Prefix slot {slot} holds no prefix")
        return entry

    def _free(self, slot: int) -> None:
        entry = self._slot.pop(slot)
        del self._entries[entry.key]
        self._free_pages.extend(reversed(entry.pages))
        heapq.heappush(self._free_slots, slot)
