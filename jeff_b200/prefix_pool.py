"""The paged prefix-state pool: every cached prefix's state in device memory at fixed addresses, read in place by
the decision kernels through per-slot block tables.

The contract kept from the reference's engine/prefix_pool.py (so an engine above it behaves the same): pages of one
size (the bytes of PAGE_TOKENS tokens of attention keys and values over all attention layers: 393,216 B for the
0.8B layout) viewed three ways (kv[page, attn layer, K|V, token, head, dim] bf16; state[page, head, key dim, value
dim] fp32 with a whole number of Gated DeltaNet heads per page; conv[page, layer, 3, channels] bf16); a prefix of p
tokens takes its state pages, its convolution pages and ceil(p / PAGE_TOKENS) key/value pages, in that order in its
block table; slot 0 is the empty prefix (its fixed entries name page 1, zeros, never written), page 0 is the sink
the prefix pass writes padding to; prefixes are keyed by (adapter row, prefix text), least recently used out first,
never a pinned one; the capacity arithmetic and the error messages.

The bookkeeping is this module's own, built for one engine thread that reserves many prefixes per pass:
- per-slot state lives in flat numpy arrays (pages held, tokens, pin count, recency stamp), not in per-prefix
  objects; recency is a global clock stamped on a slot when it is reserved or looked up, and eviction takes the
  unpinned slots in stamp order (one argsort when a reservation has to evict, no reordering on every lookup);
- free pages are one numpy stack (a reservation takes a slice off its top, a freed prefix pushes its pages back),
  free slots a plain stack;
- block tables are written into a host mirror and reach the device table in one copy of the changed row range when
  the device table is next used (`tables`, `sync()`), not one copy per reservation.

Nothing here is thread safe: it runs on the engine's GPU thread between passes."""

from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass

import numpy as np
import torch

from jeff_b200 import constants as C
from jeff_b200.errors import EngineError

PAGE_TOKENS = 32
SINK_PAGE, ZERO_PAGE = 0, 1
RESERVED_PAGES = 2

__all__ = ["EngineError", "FAST_PATH_SHAPES", "PAGE_TOKENS", "PrefixPool", "PrefixShapes", "RESERVED_PAGES",
           "SINK_PAGE", "ZERO_PAGE", "check_pool_holds", "check_pool_size", "pool_pages", "prefix_pool_mb_for",
           "prefixes_held"]


def _ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


@dataclass(frozen=True)
class PrefixShapes:
    """One prefix's state: per Gated DeltaNet layer a conv tail (3, channels) and a recurrent state (heads, key dim,
    value dim); per attention layer and token, keys and values (heads, dim)."""
    gdn_layers: int
    conv: tuple[int, int]
    state: tuple[int, int, int]
    attn_layers: int
    kv: tuple[int, int]
    page_tokens: int = PAGE_TOKENS

    @property
    def page_bytes(self) -> int:
        heads, dim = self.kv
        return 2 * self.attn_layers * self.page_tokens * heads * dim * 2      # K and V, bf16

    def _per_page(self, unit_bytes: int) -> int:
        return self.page_bytes // unit_bytes

    @property
    def _heads(self) -> int:
        return self.gdn_layers * self.state[0]

    @property
    def state_pages(self) -> int:
        _, kd, vd = self.state
        return _ceil_div(self._heads, self._per_page(kd * vd * 4))

    @property
    def heads_per_page(self) -> int:
        return self._heads // self.state_pages

    @property
    def conv_pages(self) -> int:
        taps, channels = self.conv
        return _ceil_div(self.gdn_layers, self._per_page(taps * channels * 2))

    @property
    def layers_per_conv_page(self) -> int:
        return self.gdn_layers // self.conv_pages

    @property
    def fixed_pages(self) -> int:
        """Pages a prefix takes whatever its length."""
        return self.state_pages + self.conv_pages

    def pages_per_prefix(self, tokens: int) -> int:
        return self.fixed_pages + _ceil_div(tokens, self.page_tokens)

    def check(self) -> None:
        even = (self.page_bytes % 4 == 0 and self._heads % self.state_pages == 0
                and self.gdn_layers % self.conv_pages == 0)
        if not even:
            raise ValueError(f"{self}: the states and convolution tails do not split evenly into pages")


FAST_PATH_SHAPES = PrefixShapes(gdn_layers=C.GDN_LAYERS, conv=(C.CONV - 1, C.QKV_DIM), state=(C.NV, C.DK, C.DV),
                                attn_layers=C.ATTN_LAYERS, kv=(C.NKV, C.HD))


def pool_pages(prefix_pool_mb: int, shapes: PrefixShapes = FAST_PATH_SHAPES) -> int:
    """Pages in a pool of `prefix_pool_mb` MB, the reserved two included."""
    return (prefix_pool_mb << 20) // shapes.page_bytes


def prefixes_held(prefix_pool_mb: int, tokens: int, shapes: PrefixShapes = FAST_PATH_SHAPES) -> int:
    """How many prefixes of `tokens` tokens such a pool holds at once."""
    usable = pool_pages(prefix_pool_mb, shapes) - RESERVED_PAGES
    return usable // shapes.pages_per_prefix(tokens) if usable > 0 else 0


def prefix_pool_mb_for(rows: int, shapes: PrefixShapes = FAST_PATH_SHAPES) -> int:
    """The smallest pool (MB) holding `rows` prefixes of the longest prefix at once."""
    need = RESERVED_PAGES + rows * shapes.pages_per_prefix(C.LONGEST_PREFIX_TOKENS)
    return _ceil_div(need * shapes.page_bytes, 1 << 20)


def check_pool_size(prefix_pool_mb: object) -> int:
    smallest = prefix_pool_mb_for(1)
    valid = type(prefix_pool_mb) is int and prefix_pool_mb >= smallest
    if not valid:
        raise EngineError(f"--prefix-pool-mb {prefix_pool_mb!r}: give a whole number of megabytes, at least {smallest} "
                          f"(one prefix of {C.LONGEST_PREFIX_TOKENS} tokens); for example 2048 holds "
                          f"{prefixes_held(2048, 1000)} prefixes of 1,000 tokens")
    return prefix_pool_mb  # type: ignore[return-value]


def check_pool_holds(prefix_pool_mb: int, max_batch_rows: int) -> None:
    needed = prefix_pool_mb_for(max_batch_rows)
    if prefix_pool_mb >= needed:
        return
    raise EngineError(
        f"--prefix-pool-mb {prefix_pool_mb} cannot hold --max-batch-rows {max_batch_rows} prefixes of "
        f"{C.LONGEST_PREFIX_TOKENS} tokens (the longest prefix) at once, as one pass of {max_batch_rows} rows may "
        f"need; give --prefix-pool-mb at least {needed}, or lower --max-batch-rows.")


class PrefixPool:
    """Page memory allocated once on `device`, and the host bookkeeping of which prefix holds which pages."""

    def __init__(self, pages: int, device: str | torch.device = "cuda", *,
                 shapes: PrefixShapes = FAST_PATH_SHAPES, max_prefix_tokens: int = C.LONGEST_PREFIX_TOKENS) -> None:
        shapes.check()
        fixed = shapes.fixed_pages
        if pages < RESERVED_PAGES + fixed:
            raise ValueError(f"A prefix pool of {pages} pages cannot hold a single prefix ({fixed} pages "
                             "and the 2 reserved)")
        self.shapes, self.pages, self.page_tokens, self.fixed_pages = shapes, pages, shapes.page_tokens, fixed
        self.slots = 1 + (pages - RESERVED_PAGES) // fixed
        self.max_prefix_tokens = max_prefix_tokens
        self.max_kv_pages = _ceil_div(max_prefix_tokens, self.page_tokens)
        self.width = fixed + self.max_kv_pages

        # device memory: one int32 allocation and its three typed views
        self.data = torch.zeros(pages, shapes.page_bytes // 4, device=device, dtype=torch.int32)
        bf16 = self.data.view(torch.bfloat16)
        self.kv = bf16.view(pages, shapes.attn_layers, 2, self.page_tokens, *shapes.kv)
        state_words = shapes.heads_per_page * shapes.state[1] * shapes.state[2]
        self.state = self.data.view(torch.float32)[:, :state_words].view(pages, shapes.heads_per_page,
                                                                         shapes.state[1], shapes.state[2])
        conv_halves = shapes.layers_per_conv_page * shapes.conv[0] * shapes.conv[1]
        self.conv = bf16[:, :conv_halves].view(pages, shapes.layers_per_conv_page, *shapes.conv)

        # block tables: host mirror, device copy, and the host rows not yet copied
        self._host_tables = np.zeros((self.slots, self.width), dtype=np.int32)
        self._host_tables[0, :fixed] = ZERO_PAGE
        self._dev_tables = torch.from_numpy(self._host_tables).to(device)
        self._stale_lo, self._stale_hi = self.slots, 0

        # per-slot bookkeeping (slot 0, the empty prefix, is never held)
        self._held = np.zeros(self.slots, dtype=bool)
        self._npages = np.zeros(self.slots, dtype=np.int32)
        self._tokens = np.zeros(self.slots, dtype=np.int64)
        self._pins = np.zeros(self.slots, dtype=np.int32)
        self._stamp = np.zeros(self.slots, dtype=np.int64)
        self._clock = 0
        self._key_of: list[tuple[int, str] | None] = [None] * self.slots
        self._slot_of: dict[tuple[int, str], int] = {}
        self._free_slots = list(range(self.slots - 1, 0, -1))        # lowest slot on top
        self._page_stack = np.arange(pages - 1, RESERVED_PAGES - 1, -1, dtype=np.int32)   # lowest page on top
        self._page_top = len(self._page_stack)

    # ------------------------------------------------------------ sizes

    @property
    def nbytes(self) -> int:
        return self.data.numel() * self.data.element_size()

    def __len__(self) -> int:
        return len(self._slot_of)

    def free_slot_count(self) -> int:
        return len(self._free_slots)

    def free_page_count(self) -> int:
        return self._page_top

    # ------------------------------------------------------------ device tables

    @property
    def tables(self) -> torch.Tensor:
        """The device block tables (slots, width) int32, brought up to date with every reservation made so far."""
        self.sync()
        return self._dev_tables

    def sync(self) -> None:
        """Copy the block-table rows changed since the last copy to the device (one copy of their row range). Runs on
        the current stream, ahead of any pass enqueued after it."""
        if self._stale_lo < self._stale_hi:
            lo, hi = self._stale_lo, self._stale_hi
            self._dev_tables[lo:hi].copy_(torch.from_numpy(self._host_tables[lo:hi]))
            self._stale_lo, self._stale_hi = self.slots, 0

    # ------------------------------------------------------------ lookups

    def _touch(self, slot: int) -> None:
        self._clock += 1
        self._stamp[slot] = self._clock

    def lookup(self, adapter_index: int, text: str) -> int | None:
        slot = self._slot_of.get((adapter_index, text))
        if slot is not None:
            self._touch(slot)
        return slot

    def _require(self, slot: int) -> None:
        if not (0 < slot < self.slots and self._held[slot]):
            raise ValueError(f"Prefix slot {slot} holds no prefix")

    def key(self, slot: int) -> tuple[int, str]:
        self._require(slot)
        key = self._key_of[slot]
        assert key is not None
        return key

    def length(self, slot: int) -> int:
        if slot == 0:
            return 0
        self._require(slot)
        return int(self._tokens[slot])

    def block_table(self, slot: int) -> list[int]:
        if slot == 0:
            return [ZERO_PAGE] * self.fixed_pages
        self._require(slot)
        return self._host_tables[slot, :self._npages[slot]].tolist()

    # ------------------------------------------------------------ reservations

    def _evictable(self) -> np.ndarray:
        """Held, unpinned slots, least recently used first."""
        cand = np.flatnonzero(self._held & (self._pins == 0))
        return cand[np.argsort(self._stamp[cand], kind="stable")]

    def reserve(self, adapter_index: int, text: str, tokens: int) -> int:
        """A slot and its pages for a new prefix of `tokens` tokens, evicting least recently used unpinned prefixes
        as needed. The pages' contents are whatever was there: the prefix pass writes them."""
        key = (adapter_index, text)
        if key in self._slot_of:
            raise ValueError(f"Prefix of adapter row {adapter_index} is already in the pool "
                             f"(slot {self._slot_of[key]})")
        if tokens > self.max_prefix_tokens:
            raise ValueError(f"A prefix of {tokens} tokens is longer than the longest prefix ({self.max_prefix_tokens})")
        wanted = self.shapes.pages_per_prefix(tokens)
        usable = self.pages - RESERVED_PAGES
        if wanted > usable:
            raise EngineError(f"A prefix of {tokens} tokens needs {wanted} pages; the prefix pool has {usable} in all "
                              "(raise --prefix-pool-mb)")
        if not self._free_slots or self._page_top < wanted:
            victims = self._evictable()
            slots_ok = bool(self._free_slots) or victims.size > 0
            pages_ok = self._page_top + int(self._npages[victims].sum()) >= wanted
            if not (slots_ok and pages_ok):
                pinned = int(np.count_nonzero(self._pins))
                raise EngineError(f"No room in the prefix pool for a prefix of {tokens} tokens ({wanted} pages): "
                                  f"{pinned} prefixes are pinned by the pass being formed, and the others free "
                                  f"too few pages. Lower --max-batch-rows or raise --prefix-pool-mb.")
            for victim in victims.tolist():
                if self._free_slots and self._page_top >= wanted:
                    break
                self._drop(victim)
        slot = self._free_slots.pop()
        top = self._page_top - wanted
        self._host_tables[slot, :wanted] = self._page_stack[top:self._page_top][::-1]
        self._page_top = top
        self._stale_lo, self._stale_hi = min(self._stale_lo, slot), max(self._stale_hi, slot + 1)
        self._held[slot] = True
        self._npages[slot] = wanted
        self._tokens[slot] = tokens
        self._key_of[slot] = key
        self._slot_of[key] = slot
        self._touch(slot)
        return slot

    def _drop(self, slot: int) -> None:
        n = int(self._npages[slot])
        self._page_stack[self._page_top:self._page_top + n] = self._host_tables[slot, :n][::-1]
        self._page_top += n
        key = self._key_of[slot]
        assert key is not None
        del self._slot_of[key]
        self._key_of[slot] = None
        self._held[slot] = False
        self._npages[slot] = 0
        self._tokens[slot] = 0
        self._free_slots.append(slot)

    def release(self, slot: int) -> None:
        """Free a prefix (for example a reservation whose prefix pass failed)."""
        if 0 < slot < self.slots and self._pins[slot]:
            raise ValueError(f"Prefix slot {slot} is pinned")
        self._require(slot)
        self._drop(slot)

    # ------------------------------------------------------------ pins

    def pin(self, slots: Iterable[int]) -> None:
        """Count one pin per listed slot (a slot listed twice is pinned twice); all or none."""
        arr = np.fromiter(slots, dtype=np.int64)
        for slot in arr.tolist():
            self._require(slot)
        np.add.at(self._pins, arr, 1)

    def unpin(self, slots: Iterable[int]) -> None:
        for slot in slots:
            if not (0 <= slot < self.slots) or self._pins[slot] == 0:
                raise ValueError(f"Prefix slot {slot} is not pinned")
            self._pins[slot] -= 1

    @property
    def _pinned(self) -> dict[int, int]:
        """Pinned slots and their pin counts."""
        where = np.flatnonzero(self._pins)
        return dict(zip(where.tolist(), self._pins[where].tolist(), strict=True))

    def forget_adapter(self, adapter_index: int) -> None:
        """Drop every prefix of an adapter row (its row in the adapter pools was filled or freed)."""
        mine = [slot for (index, _), slot in self._slot_of.items() if index == adapter_index]
        pinned = sorted(slot for slot in mine if self._pins[slot])
        if pinned:
            raise ValueError(f"Adapter row {adapter_index} has pinned prefix slots {pinned}: an adapter changes only "
                             "between passes")
        for slot in mine:
            self._drop(slot)

    # ------------------------------------------------------------ page contents (tests and tools)

    def _page_index(self, slot: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        table = torch.tensor(self.block_table(slot), dtype=torch.long, device=self.data.device)
        s, c = self.shapes.state_pages, self.shapes.conv_pages
        return table[:s], table[s:s + c], table[s + c:]

    def gather(self, slot: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """A prefix's state read out of its pages: conv (layers, 3, channels), state (layers, heads, key dim, value
        dim), kv (attention layers, 2, prefix length, heads, dim)."""
        sh = self.shapes
        st, cv, kvp = self._page_index(slot)
        state = self.state[st].reshape(sh.gdn_layers, *sh.state)
        conv = self.conv[cv].reshape(sh.gdn_layers, *sh.conv)
        tokens = self.length(slot)
        kv = self.kv[kvp].permute(1, 2, 0, 3, 4, 5).reshape(sh.attn_layers, 2, len(kvp) * self.page_tokens, *sh.kv)
        return conv, state, kv[:, :, :tokens]

    def write(self, slot: int, conv: torch.Tensor, state: torch.Tensor, kv: torch.Tensor) -> None:
        """Put one prefix's state into its slot's pages (the prefix pass writes from its kernels; this is for tests
        and tools): conv (layers, 3, channels), state (layers, heads, kd, vd), kv (attention layers, 2, tokens, heads,
        dim)."""
        sh = self.shapes
        st, cv, kvp = self._page_index(slot)
        self.state[st] = state.reshape(len(st), *self.state.shape[1:]).to(self.state)
        self.conv[cv] = conv.reshape(len(cv), *self.conv.shape[1:]).to(self.conv)
        tokens = kv.shape[2]
        n = _ceil_div(tokens, self.page_tokens)
        if n == 0:
            return
        block = torch.zeros(sh.attn_layers, 2, n * self.page_tokens, *sh.kv, dtype=self.kv.dtype,
                            device=self.kv.device)
        block[:, :, :tokens] = kv.to(self.kv)
        self.kv[kvp[:n]] = block.view(sh.attn_layers, 2, n, self.page_tokens, *sh.kv).permute(2, 0, 1, 3, 4, 5)
