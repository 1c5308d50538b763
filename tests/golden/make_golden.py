"""Generate the golden vectors under tests/golden/ by running the REFERENCE's own code (firelex/jeff and the
transformers Qwen3.5 model its standard path runs). Needs a checkout of the reference, named by $JEFF_REFERENCE,
and is run by hand on a machine that has one; the fixtures it writes are committed, and nothing at test time reads
the reference.

    JEFF_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Writes:
- int4_golden.npz: the reference's pack_int4, pack_kernel (words, scales), dequantize and round_to_nearest on seeded
  integers and weights (engine/int4.py:183-262, engine/quantize.py:259-267), including its known-answer word
  0xFED98710 and the 64-column padding;
- pool_layout.json: the reference PrefixShapes numbers (engine/prefix_pool.py:55-98) for the fast-path layout;
- gdn_scan_golden.npz: transformers torch_chunk_gated_delta_rule (the standard path's Gated DeltaNet scan) from an
  initial state, with its final state;
- model_golden.npz: a 4-layer model at the real layer dimensions (3 Gated DeltaNet + 1 attention layer, vocabulary
  4,096), synthetic int4-g64 weights (jeff_b200.synthetic, quantised by the reference's round_to_nearest and
  dequantised by its dequantize), two rank-16 adapters applied through the reference's LoraLinear, the whole prompt
  (prefix + new tokens) run through transformers' Qwen3_5Model and DecisionModel.forward's readout, mask and
  temperature softmax: each row's probabilities and per-layer last-token hidden states."""

from __future__ import annotations

import json
import os
import sys
import zlib
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
if "JEFF_REFERENCE" not in os.environ:
    sys.exit("make_golden.py: set JEFF_REFERENCE to a checkout of the reference")
REF = Path(os.environ["JEFF_REFERENCE"])
sys.path[:0] = [str(ROOT), str(REF / "runtime/python/src"), str(REF / "packages/python/src")]

from jeff_runtime.engine import int4 as ref_int4  # noqa: E402
from jeff_runtime.engine import prefix_pool as ref_pool  # noqa: E402
from jeff_runtime.engine.lora import LoraLinear  # noqa: E402
from jeff_runtime.engine.model import DecisionModel, PreparedBatch  # noqa: E402
from jeff_runtime.engine.quantize import round_to_nearest  # noqa: E402

from jeff_b200 import synthetic  # noqa: E402

MODEL_LAYERS = 4
MODEL_VOCAB = 4096
MODEL_SEED = 11


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def int4_golden() -> None:
    g = torch.Generator().manual_seed(0)
    q = torch.randint(-8, 8, (128, 256), generator=g, dtype=torch.int8)
    q[0, :8] = torch.tensor([-8, -7, -1, 0, 1, 5, 6, 7])
    scales = (torch.rand(128, 4, generator=g) + 0.01).to(torch.bfloat16)
    packed = ref_int4.pack_kernel(q, scales)
    q70 = torch.randint(-8, 8, (70, 128), generator=g, dtype=torch.int8)
    s70 = (torch.rand(70, 2, generator=g) + 0.01).to(torch.bfloat16)
    p70 = ref_int4.pack_kernel(q70, s70)
    w = torch.randn(64, 256, generator=g) * 0.02
    rq, rs = round_to_nearest(w)
    q7 = torch.full((1, 64), 7, dtype=torch.int8)
    s7 = torch.tensor([[1.0078125]], dtype=torch.bfloat16)
    np.savez_compressed(
        HERE / "int4_golden.npz",
        q=q.numpy(), scales=bits(scales), words=packed.words.numpy(), kscales=bits(packed.scales),
        folder=ref_int4.pack_int4(q).numpy(), deq=bits(ref_int4.dequantize(q, scales)),
        q70=q70.numpy(), s70=bits(s70), words70=p70.words.numpy(), kscales70=bits(p70.scales),
        w_rtn=w.numpy(), q_rtn=rq.numpy(), s_rtn=bits(rs),
        deq7=bits(ref_int4.dequantize(q7, s7)))


def pool_golden() -> None:
    s = ref_pool.FAST_PATH_SHAPES
    out = {"page_bytes": s.page_bytes, "state_pages": s.state_pages, "heads_per_page": s.heads_per_page,
           "conv_pages": s.conv_pages, "layers_per_conv_page": s.layers_per_conv_page, "fixed_pages": s.fixed_pages,
           "pages_per_prefix": {str(t): s.pages_per_prefix(t) for t in (0, 1, 31, 32, 33, 512, 1000, 2000, 8192)},
           "pool_pages_8192": ref_pool.pool_pages(8192), "prefixes_held_8192_1000": ref_pool.prefixes_held(8192, 1000),
           "prefix_pool_mb_for": {str(r): ref_pool.prefix_pool_mb_for(r) for r in (1, 8, 64)}}
    (HERE / "pool_layout.json").write_text(json.dumps(out, indent=1) + "\n")


def gdn_golden() -> None:
    from transformers.models.qwen3_5.modeling_qwen3_5 import torch_chunk_gated_delta_rule

    g = torch.Generator().manual_seed(3)
    b, t, h, d = 1, 80, 2, 128

    def unit() -> torch.Tensor:
        x = torch.randn(b, t, h, d, generator=g)
        return (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16)

    q, k = unit(), unit()
    v = torch.randn(b, t, h, d, generator=g).to(torch.bfloat16)
    gg = torch.nn.functional.logsigmoid(torch.randn(b, t, h, generator=g) * 0.5 + 2.0)
    beta = torch.sigmoid(torch.randn(b, t, h, generator=g)).to(torch.bfloat16)
    h0 = torch.randn(b, h, d, d, generator=g) * 0.1
    o, s = torch_chunk_gated_delta_rule(q.float(), k.float(), v.float(), gg, beta.float(), chunk_size=64,
                                        initial_state=h0, output_final_state=True, use_qk_l2norm_in_kernel=False)
    np.savez_compressed(HERE / "gdn_scan_golden.npz", q=bits(q), k=bits(k), v=bits(v), g=gg.numpy(),
                        beta=bits(beta), h0=h0.numpy(), o=o.float().numpy(), s=s.float().numpy())


def model_golden() -> None:
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5Config
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5Model

    spec = synthetic.ModelSpec(layers=MODEL_LAYERS, vocab=MODEL_VOCAB, fmt="g64", seed=MODEL_SEED, norm_noise=0.1)
    model = synthetic.make_model(spec)
    adapters = [synthetic.make_adapter(model, i, seed=MODEL_SEED + i) for i in (1, 2)]
    heads = [synthetic.base_head(model)] + [(a.readout, a.temperature) for a in adapters]
    text = {"hidden_size": 1024, "intermediate_size": 3584, "num_hidden_layers": MODEL_LAYERS,
            "layer_types": model.kinds, "full_attention_interval": 4, "num_attention_heads": 8,
            "num_key_value_heads": 2, "head_dim": 256, "linear_key_head_dim": 128, "linear_value_head_dim": 128,
            "linear_num_key_heads": 16, "linear_num_value_heads": 16, "linear_conv_kernel_dim": 4,
            "vocab_size": MODEL_VOCAB, "attn_output_gate": True, "rms_norm_eps": 1e-6,
            "rope_parameters": {"mrope_interleaved": True, "mrope_section": [11, 11, 10],
                                "partial_rotary_factor": 0.25, "rope_theta": 10000000, "rope_type": "default"}}
    vision = {"depth": 1, "hidden_size": 32, "intermediate_size": 64, "num_heads": 2, "out_hidden_size": 1024,
              "num_position_embeddings": 16, "deepstack_visual_indexes": []}
    torch.manual_seed(0)
    backbone = Qwen3_5Model(Qwen3_5Config(text_config=text, vision_config=vision)).float().eval()
    state = {}
    lm = "language_model."
    state[lm + "embed_tokens.weight"] = model.embed.float()
    state[lm + "norm.weight"] = model.final_norm.float()
    checks = {}
    for i, layer in enumerate(model.layers):
        p = f"{lm}layers.{i}."
        state[p + "input_layernorm.weight"] = layer.norm_in
        state[p + "post_attention_layernorm.weight"] = layer.norm_post
        for grp in layer.groups.values():
            # the reference's own quantiser and dequantiser must give the same bf16 weights the synthetic ones hold
            o0 = 0
            for name, size in zip(grp.names, grp.sizes, strict=True):
                w = grp.W[o0:o0 + size].float()
                state[lm + name + ".weight"] = w
                o0 += size
            checks[grp.names[0]] = int(zlib.crc32(grp.W.contiguous().view(torch.int16).numpy().tobytes()))
        if layer.kind == "linear_attention":
            la = p + "linear_attn."
            state[la + "conv1d.weight"] = layer.conv.float()[:, None, :]
            state[la + "A_log"] = layer.A_log
            state[la + "dt_bias"] = layer.dt_bias
            state[la + "norm.weight"] = layer.gnorm.float()
        else:
            sa = p + "self_attn."
            state[sa + "q_norm.weight"] = layer.q_norm
            state[sa + "k_norm.weight"] = layer.k_norm
    missing, unexpected = backbone.load_state_dict(state, strict=False)
    assert not unexpected, unexpected
    assert all(not m.startswith(lm) for m in missing), [m for m in missing if m.startswith(lm)]
    # the reference round_to_nearest + dequantize reproduce the synthetic g64 weights bit for bit
    w0 = synthetic.normal(MODEL_SEED, "layers.0.mlp.down_proj", (1024, 3584), 0.02)
    rq, rs = round_to_nearest(w0)
    down = model.layers[0].groups["mlp_down"].W
    assert torch.equal(ref_int4.dequantize(rq, rs), down), "synthetic g64 weights differ from the reference's RTN"

    # LoRA through the reference's LoraLinear (model precision, float32 on CPU), one adapter active at a time
    wrappers = {}
    for i, layer in enumerate(model.layers):
        for grp in layer.groups.values():
            for name in grp.names:
                if name.rsplit(".", 1)[-1] not in ("in_proj_qkv", "in_proj_z", "out_proj", "q_proj", "k_proj",
                                                   "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"):
                    continue
                full = lm + name
                parent, _, child = full.rpartition(".")
                base = backbone.get_submodule(full)
                wrapper = LoraLinear(base, "model")
                for ad in adapters:
                    a, b = ad.matrices[name]
                    wrapper.add(ad.name, a.float(), b.float(), 1.0)
                setattr(backbone.get_submodule(parent), child, wrapper)
                wrappers[full] = wrapper

    dm = object.__new__(DecisionModel)
    torch.nn.Module.__init__(dm)
    dm.backbone = backbone
    g = torch.Generator().manual_seed(MODEL_SEED)
    rows = [(0, 40, 24, 5), (1, 40, 24, 17), (2, 33, 31, 2), (1, 0, 32, 9)]   # adapter, prefix, new tokens, count
    probs, hidden_last, ids_all = [], [], []
    for adapter, plen, nlen, count in rows:
        ids = torch.randint(0, MODEL_VOCAB, (plen + nlen,), generator=g)
        ids_all.append(ids.numpy())
        for w in wrappers.values():
            w.active = None if adapter == 0 else adapters[adapter - 1].name
        readout, temperature = heads[adapter]
        dm.readout = torch.nn.Linear(1024, 255, bias=False)
        dm.readout.weight.data = readout.float()
        dm.temperature = temperature
        with torch.no_grad():
            batch = PreparedBatch({"input_ids": ids[None], "attention_mask": torch.ones(1, len(ids), dtype=torch.long)},
                                  (count,), len(ids))
            logits = dm.forward(batch)
            p = (logits / temperature).softmax(-1)
            out = backbone(input_ids=ids[None], attention_mask=torch.ones(1, len(ids), dtype=torch.long),
                           use_cache=False, output_hidden_states=True)
        probs.append(p[0].numpy())
        hidden_last.append(np.stack([h[0, -1].numpy() for h in out.hidden_states[1:]]))
    np.savez_compressed(HERE / "model_golden.npz", rows=np.array(rows), probs=np.stack(probs),
                        hidden_last=np.stack(hidden_last), ids=np.concatenate(ids_all),
                        crc_names=np.array(list(checks)), crc_values=np.array(list(checks.values()), dtype=np.int64))
    (HERE / "model_golden.json").write_text(json.dumps({"layers": MODEL_LAYERS, "vocab": MODEL_VOCAB,
                                                        "seed": MODEL_SEED, "fmt": "g64", "norm_noise": 0.1,
                                                        "adapters": [1, 2]}, indent=1) + "\n")


if __name__ == "__main__":
    int4_golden()
    pool_golden()
    gdn_golden()
    model_golden()
    print("golden vectors written to", HERE)
