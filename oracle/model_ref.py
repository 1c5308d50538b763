"""TEST INFRASTRUCTURE ONLY (the checker, never the product): torch restatement of the batched decision pass (CPU,
or a GPU through to_device when a test runs it there as the checker).

Each function restates one kernel of the reference's fast path with its bfloat16 rounding points, citing the
reference (paths relative to runtime/python/src/jeff_runtime/engine/; "T5" is transformers'
models/qwen3_5/modeling_qwen3_5.py, the standard path's model):

- add_rms                 fast_path.py:80-100 (residual add rounded to bf16, RMSNorm in float32 times 1 + w)
- product                 int4_kernels.py:1-30 and :105-129 (base product in float32 plus bf16(x A^T) Bt, rounded
                          once: the reference's cut-product rule), lora.py:212-220 for the exact form
- gdn_prep                batched_kernels.py:89-149 (conv over [3 cached; new], SiLU->bf16, L2 norm, g, beta),
                          T5:463-495
- gdn_scan                batched_kernels.py:200-237 (the gated delta rule token by token, float32 state),
                          T5:234-311 (the same rule in chunks)
- gated_norm              fast_path.py:103-120, T5:175-190
- attn_prep               batched_kernels.py:302-345 (q/k RMSNorm, partial RoPE at prefix length + t), T5:647-669
- attention               batched_kernels.py:370-436 (prefix fully, new keys causally, GQA 4:1, scale 1/16)
- gate_mul                fast_path.py:123-138, T5:690
- silu_mul                fast_path.py:141-156, T5:695-707
- readout                 batched_kernels.py:492-518, model.py:264-269 (bf16 logits, mask >= count to -1e9,
                          / temperature, softmax)
- decision_pass           batched_path.py:242-276 (the recorded pass), prefix_pass batched_path.py:291-349.

`exact=True` drops every intermediate rounding: the float32 arithmetic of the reference's standard path
(DecisionModel on CPU, model.py:210), which tests/golden pins against the transformers model itself."""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

EPS = 1e-6
HIDDEN, INTER = 1024, 3584
NK, DK, NV, DV = 16, 128, 16, 128
NQ, NKV, HD, ROT = 8, 2, 256, 64
QKV, ZD = 6144, 2048
ROPE_THETA = 1e7
BF = torch.bfloat16


def bf(x: torch.Tensor) -> torch.Tensor:
    return x.to(BF).float()


def _r(exact: bool):
    return (lambda x: x) if exact else bf


def add_rms(x: torch.Tensor, d: torch.Tensor | None, w: torch.Tensor, exact: bool = False
            ) -> tuple[torch.Tensor, torch.Tensor]:
    """(x + d, rms(x + d) * (1 + w)): x, d (T, 1024) float32 holding bf16 values; w the RMSNorm weight."""
    r = _r(exact)
    if d is not None:
        x = r(x + d)
    var = (x * x).mean(-1, keepdim=True)
    return x, r(x * torch.rsqrt(var + EPS) * (1.0 + w.float()))


def product(x: torch.Tensor, W: torch.Tensor, lora: list[tuple[torch.Tensor, torch.Tensor] | None],
            row_of_token: torch.Tensor, exact: bool = False, wide: bool = False) -> torch.Tensor:
    """x (T, k) @ W^T plus each token's LoRA update: lora[row] = (A (R, k), B (out, R)) or None; row_of_token (T,).
    wide: the sums in float64 before the same roundings (a second valid summation order, to measure how far two
    float32-accumulating implementations with identical rounding points drift apart)."""
    acc = torch.float64 if wide else torch.float32
    xa = x.to(acc)
    y = xa @ W.to(acc).T
    for row in torch.unique(row_of_token).tolist():
        pair = lora[row]
        if pair is None:
            continue
        a, b = pair
        sel = row_of_token == row
        mid = (xa[sel] @ a.to(acc).T).float()
        y[sel] = y[sel] + (mid if exact else bf(mid)).to(acc) @ b.to(acc).T
    y = y.float()
    return y if exact else bf(y)


def gdn_prep(pr: torch.Tensor, tail: torch.Tensor, conv_w: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor,
             exact: bool = False) -> tuple[torch.Tensor, ...]:
    """One row: pr (N, 8224) [qkv 6144 | z 2048 | b 16 | a 16], tail (3, 6144) the cached convolution inputs,
    conv_w (6144, 4) depthwise weights. Returns q, k, v (N, 16, 128), g (N, 16) float32, beta (N, 16)."""
    r = _r(exact)
    n = pr.shape[0]
    xs = torch.cat([tail.float(), pr[:, :QKV].float()], 0)          # (3 + N, 6144)
    w = conv_w.float()
    acc = sum(w[:, i] * xs[i:i + n] for i in range(4))
    c = r(acc * torch.sigmoid(acc)).view(n, 3 * NK, DK)
    qk = c[:, :2 * NK]
    y = r(qk * torch.rsqrt((qk * qk).sum(-1, keepdim=True) + 1e-6))
    bv = pr[:, QKV + ZD:QKV + ZD + NV].float()
    av = pr[:, QKV + ZD + NV:QKV + ZD + 2 * NV].float() + dt_bias.float()
    sp = torch.where(av > 20.0, av, torch.log1p(torch.exp(av)))
    g = -torch.exp(A_log.float()) * sp
    beta = r(torch.sigmoid(bv))
    return y[:, :NK], y[:, NK:], c[:, 2 * NK:], g, beta


def gdn_scan(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
             s0: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Rows batched: q, k, v (B, N, 16, 128), g, beta (B, N, 16), s0 (B, 16, 128, 128) float32. The gated delta
    rule token by token: S <- S e^g; v' = beta (v - S^T k); S <- S + k v'^T; o = S^T q / sqrt(128). Returns o
    (B, N, 16, 128) float32 and the final state."""
    s = s0.float().clone()
    out = torch.empty(v.shape, dtype=torch.float32, device=v.device)
    scale = DK ** -0.5
    for t in range(q.shape[1]):
        s = s * torch.exp(g[:, t])[..., None, None]
        kt, vt, qt = k[:, t].float(), v[:, t].float(), q[:, t].float() * scale
        vnew = beta[:, t].float()[..., None] * (vt - torch.einsum("bhkv,bhk->bhv", s, kt))
        s = s + kt[..., :, None] * vnew[..., None, :]
        out[:, t] = torch.einsum("bhkv,bhk->bhv", s, qt)
    return out, s


def gated_norm(o: torch.Tensor, z: torch.Tensor, w: torch.Tensor, exact: bool = False) -> torch.Tensor:
    """o (N, 16, 128), z (N, 2048), w (128,) bf16: bf16(w * bf16(rms(o))) * silu(z), per head."""
    r = _r(exact)
    y = r(o * torch.rsqrt((o * o).mean(-1, keepdim=True) + EPS))
    y = r(w.float() * y)
    zz = z.float().view(o.shape)
    return r(y * (zz * torch.sigmoid(zz))).reshape(o.shape[0], -1)


def inv_freq(device: torch.device | str = "cpu") -> torch.Tensor:
    return 1.0 / (ROPE_THETA ** (torch.arange(0, ROT, 2, dtype=torch.float32, device=device) / ROT))


def attn_prep(pr: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor, pos0: int, exact: bool = False
              ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """One row: pr (N, 5120) [q_proj: per head 256 query then 256 gate | k 512 | v 512]. Returns q (N, 8, 256),
    k, v (N, 2, 256) and the gate (N, 8, 256); the rotary position of token t is pos0 + t."""
    r = _r(exact)
    n = pr.shape[0]
    x = pr.float()
    qg = x[:, :NQ * 2 * HD].view(n, NQ, 2 * HD)
    queries, gate = qg[:, :, :HD], qg[:, :, HD:]
    keys = x[:, NQ * 2 * HD:NQ * 2 * HD + NKV * HD].view(n, NKV, HD)
    values = x[:, NQ * 2 * HD + NKV * HD:].view(n, NKV, HD)
    positions = (pos0 + torch.arange(n, device=pr.device)).float()
    f = positions[:, None, None] * torch.cat([inv_freq(pr.device), inv_freq(pr.device)])
    cos, sin = r(torch.cos(f)), r(torch.sin(f))

    def norm_rope(h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        y = r(h * torch.rsqrt((h * h).mean(-1, keepdim=True) + EPS) * (1.0 + w.float()))
        rot = torch.cat([-y[..., 32:64], y[..., :32]], -1)
        out = r(r(y[..., :64] * cos) + r(rot * sin))
        return torch.cat([out, y[..., 64:]], -1)

    return norm_rope(queries, q_w), norm_rope(keys, k_w), values, gate


def attention(q: torch.Tensor, kp: torch.Tensor, vp: torch.Tensor, kn: torch.Tensor, vn: torch.Tensor,
              round_weights: bool = False) -> torch.Tensor:
    """One row: q (N, 8, 256) over its prefix keys/values kp, vp (P, 2, 256) fully and its new kn, vn (N, 2, 256)
    causally; query head h reads key/value head h // 4; float32 softmax. round_weights: the unnormalised weights
    exp(s - max) are rounded to bf16 before the value product and the sum taken from the unrounded ones, as the
    reference's paged kernel does (batched_kernels.py:405-412). Returns (N, 8, 256) float32."""
    n, p = q.shape[0], kp.shape[0]
    keys = torch.cat([kp, kn]).float().repeat_interleave(NQ // NKV, 1)
    values = torch.cat([vp, vn]).float().repeat_interleave(NQ // NKV, 1)
    scores = torch.einsum("nhd,mhd->hnm", q.float(), keys) * HD ** -0.5
    m = torch.arange(p + n, device=q.device)
    allowed = (m[None, :] < p) | (m[None, :] - p <= torch.arange(n, device=q.device)[:, None])
    scores = scores.masked_fill(~allowed, float("-inf"))
    if not round_weights:
        return torch.einsum("hnm,mhd->nhd", scores.softmax(-1), values)
    e = torch.exp(scores - scores.amax(-1, keepdim=True))
    return torch.einsum("hnm,mhd->nhd", bf(e), values) / e.sum(-1).transpose(0, 1)[..., None]


def gate_mul(o: torch.Tensor, gate: torch.Tensor, exact: bool = False) -> torch.Tensor:
    r = _r(exact)
    return r(o * r(torch.sigmoid(gate.float()))).reshape(o.shape[0], -1)


def silu_mul(gu: torch.Tensor, exact: bool = False) -> torch.Tensor:
    r = _r(exact)
    g, u = gu[:, :INTER].float(), gu[:, INTER:].float()
    return r(r(g * torch.sigmoid(g)) * u)


def readout(h: torch.Tensor, W: torch.Tensor, count: int, temperature: float, exact: bool = False) -> torch.Tensor:
    """One row: h (1024,), W (255, 1024) -> probabilities (255,) float32, zero from `count` on."""
    logits = W.float() @ h.float()
    if not exact:
        logits = bf(logits)
    logits = logits.masked_fill(torch.arange(W.shape[0], device=logits.device) >= count, -1e9)
    return (logits / temperature).softmax(-1)


@dataclass
class PrefixState:
    """A prefix's cached state: per GDN layer the last three convolution inputs (3, 6144) and the recurrent state
    (16, 128, 128) float32; per attention layer its keys and values (P, 2, 256)."""
    length: int
    conv: list[torch.Tensor] = field(default_factory=list)
    state: list[torch.Tensor] = field(default_factory=list)
    keys: list[torch.Tensor] = field(default_factory=list)
    values: list[torch.Tensor] = field(default_factory=list)

    @staticmethod
    def empty(gdn_layers: int, attn_layers: int, device: torch.device | str = "cpu") -> "PrefixState":
        return PrefixState(0, [torch.zeros(3, QKV, device=device) for _ in range(gdn_layers)],
                           [torch.zeros(NV, DK, DV, device=device) for _ in range(gdn_layers)],
                           [torch.zeros(0, NKV, HD, device=device) for _ in range(attn_layers)],
                           [torch.zeros(0, NKV, HD, device=device) for _ in range(attn_layers)])


@dataclass
class RowIn:
    ids: list[int]
    lora: dict | None        # {(layer, group key): (A, B)} or None (the base)
    readout: torch.Tensor    # (255, 1024)
    temperature: float
    count: int
    prefix: PrefixState


@dataclass
class PassOut:
    probs: list[torch.Tensor]
    hidden: list[torch.Tensor]                       # each row's final normed hidden (1024,)
    layer_last: list[list[torch.Tensor]]             # per layer, each row's residual stream at its last token
    prefix_out: list[PrefixState] | None = None
    layer_all: list[torch.Tensor] | None = None      # per layer, all tokens' residual stream (when asked)


def run_pass(model, rows: list[RowIn], exact: bool = False, want_prefix: bool = False,
             keep_all: bool = False, wide: bool = False) -> PassOut:
    """The forward of every row's tokens from its cached prefix (batched_path.py:242-276): rows may have different
    lengths. With want_prefix, also each row's state after its tokens (the prefix pass, batched_path.py:291-349),
    starting from the row's given prefix state. wide: every product summed in float64 (see product)."""
    r = _r(exact)
    lengths = [len(row.ids) for row in rows]
    starts = [sum(lengths[:i]) for i in range(len(rows))]
    dev = model.embed.device
    row_of = torch.cat([torch.full((n,), i, dtype=torch.long, device=dev) for i, n in enumerate(lengths)])
    ids = torch.tensor([t for row in rows for t in row.ids], dtype=torch.long, device=dev)
    x = model.embed[ids].float()
    d: torch.Tensor | None = None
    gi = ai = 0
    layer_last: list[list[torch.Tensor]] = []
    layer_all: list[torch.Tensor] = []
    outs = [PrefixState(rows[i].prefix.length + lengths[i]) for i in range(len(rows))] if want_prefix else None

    def lora_of(layer: int, key: str) -> list:
        return [None if row.lora is None else row.lora.get((layer, key)) for row in rows]

    for li, layer in enumerate(model.layers):
        x, h = add_rms(x, d, layer.norm_in, exact)
        pr = product(h, layer.groups["proj"].W, lora_of(li, "proj"), row_of, exact, wide)
        ys = []
        if layer.kind == "linear_attention":
            by_len: dict[int, list[int]] = {}
            for i, n in enumerate(lengths):
                by_len.setdefault(n, []).append(i)
            y_rows: dict[int, torch.Tensor] = {}
            for n, members in by_len.items():
                prepped = [gdn_prep(pr[starts[i]:starts[i] + n], rows[i].prefix.conv[gi], layer.conv.float(),
                                    layer.A_log, layer.dt_bias, exact) for i in members]
                q, k, v, g, beta = (torch.stack(t) for t in zip(*prepped))
                s0 = torch.stack([rows[i].prefix.state[gi] for i in members])
                o, s_fin = gdn_scan(q, k, v, g, beta, s0)
                for j, i in enumerate(members):
                    z = pr[starts[i]:starts[i] + n, QKV:QKV + ZD]
                    y_rows[i] = gated_norm(r(o[j]), z, layer.gnorm, exact)
                    if outs is not None:
                        tail_src = torch.cat([rows[i].prefix.conv[gi].float(), pr[starts[i]:starts[i] + n, :QKV]], 0)
                        outs[i].conv.append(tail_src[-3:].clone())
                        outs[i].state.append(s_fin[j].clone())
            ys = [y_rows[i] for i in range(len(rows))]
            gi += 1
        else:
            for i, row in enumerate(rows):
                n = lengths[i]
                q, kn, vn, gate = attn_prep(pr[starts[i]:starts[i] + n], layer.q_norm, layer.k_norm,
                                            row.prefix.length, exact)
                kp, vp = row.prefix.keys[ai], row.prefix.values[ai]
                o = r(attention(q, kp, vp, kn, vn, round_weights=not exact))
                ys.append(gate_mul(o, gate, exact))
                if outs is not None:
                    outs[i].keys.append(torch.cat([kp.float(), kn]))
                    outs[i].values.append(torch.cat([vp.float(), vn.float()]))
            ai += 1
        y = torch.cat(ys, 0)
        d = product(y, layer.groups["out"].W, lora_of(li, "out"), row_of, exact, wide)
        x, h = add_rms(x, d, layer.norm_post, exact)
        gu = product(h, layer.groups["mlp_in"].W, lora_of(li, "mlp_in"), row_of, exact, wide)
        d = product(silu_mul(gu, exact), layer.groups["mlp_down"].W, lora_of(li, "mlp_down"), row_of, exact, wide)
        resid = x + d if exact else bf(x + d)
        layer_last.append([resid[starts[i] + lengths[i] - 1].clone() for i in range(len(rows))])
        if keep_all:
            layer_all.append(resid.clone())
    assert d is not None
    last = torch.tensor([starts[i] + lengths[i] - 1 for i in range(len(rows))], device=dev)
    xl = x[last] + d[last]
    if not exact:
        xl = bf(xl)
    _, hidden = add_rms(xl, None, model.final_norm, exact)
    probs = [readout(hidden[i], row.readout, row.count, row.temperature, exact) for i, row in enumerate(rows)]
    return PassOut(probs, list(hidden), layer_last, outs, layer_all if keep_all else None)


def decision(probs: torch.Tensor, count: int, threshold: float) -> tuple[int, float, bool]:
    """(chosen option, confidence, abstained): the max probability over the row's options (jeff decision.py:87-113,
    checked_probabilities :68-84 normalises by the sum first), abstaining below the threshold."""
    p = probs[:count].double()
    p = p / p.sum()
    best = int(torch.argmax(p))
    conf = float(p[best])
    return best, conf, conf < threshold


def to_device(obj, device: torch.device | str):
    """A copy of a weights object (dataclasses, dicts, lists and tuples of tensors: a model, an adapter, a prefix
    state) with every tensor moved to `device`, so the oracle can run as a checker on a GPU box; the arithmetic is
    the same float32 restatement wherever it runs."""
    import dataclasses

    if isinstance(obj, torch.Tensor):
        return obj.to(device)
    if dataclasses.is_dataclass(obj) and not isinstance(obj, type):
        return dataclasses.replace(obj, **{f.name: to_device(getattr(obj, f.name), device)
                                          for f in dataclasses.fields(obj) if f.init})
    if isinstance(obj, dict):
        return {k: to_device(v, device) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(to_device(v, device) for v in obj)
    return obj


def rel_error(a: torch.Tensor, b: torch.Tensor) -> float:
    """Norm-wise relative error ||a - b|| / ||b||."""
    return float((a.double() - b.double()).norm() / max(b.double().norm(), 1e-30))
