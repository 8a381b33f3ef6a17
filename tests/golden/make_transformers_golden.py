"""Model-level fixture for the oracle from an independent implementation:
Transformers' Ministral3ForCausalLM (the architecture of the reference's
checkpoint, Ministral-3-3B-Instruct-2512) in CPU FP32 with eager attention,
holding the seed-0 synthetic checkpoint's weights dequantized the way the
reference reads them (E4M3 code value x the tensor's BF16 weight_scale_inv,
BF16 tensors widened exactly), run on a seeded prompt.

The configuration restates the reference's fixed model facts
(src/model_facts.h: 3072 hidden, 26 layers, 32/8 heads of 128, 9216 inner,
131072 vocabulary, RMS eps 1e-5, RoPE theta 1e6, YaRN factor 16 over an original
context of 16384 with beta_fast 32 and mscale 1, query scale 0.1, tied
embeddings). The reference itself pins its RoPE against Transformers
(tests/rope_golden.h, "Transformers v5.0.0 CPU FP32"); this fixture extends
that pin from the RoPE table to the whole decoder graph: norms, GQA attention
with RoPE and the query scale, SwiGLU, residuals, final norm and tied head.

Writes tests/golden/transformers_model.json: the prompt ids; per layer and
token the L2 norm of the hidden state after the layer and its projections on
eight seeded unit directions; the full last-token hidden state after layer
25 and after the final norm; per position the 16 largest logits (ids and
values) and 256 logits at seeded vocabulary indices; a fingerprint of
the checkpoint (SHA-256 of its header and of the first 64 KB of layer 0's q
codes) so the test knows it reads the same weights.

Usage (any machine with the image's Python; about 15 GB of host memory):
    python tests/golden/make_transformers_golden.py [--checkpoint PATH]
"""
import argparse
import hashlib
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

PROMPT_SEED, PROMPT_LEN = 2718, 8
DIRECTION_SEED, DIRECTIONS = 99, 8
SAMPLE_SEED, SAMPLES = 31, 256
FULL_LAYERS = (25,)
PREFIX = "language_model.model."
LINEARS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
           "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def r9(values):
    """FP32 values as the shortest decimals that round-trip them (9 digits)."""
    return [float("%.9g" % v) for v in np.asarray(values, np.float64).ravel()]


def prompt_ids():
    return np.random.default_rng(PROMPT_SEED).integers(1000, 131072, PROMPT_LEN).astype(np.int64)


def directions():
    d = np.random.default_rng(DIRECTION_SEED).standard_normal((DIRECTIONS, 3072))
    return (d / np.linalg.norm(d, axis=1, keepdims=True)).astype(np.float64)


def sample_indices():
    return np.sort(np.random.default_rng(SAMPLE_SEED).choice(131072, SAMPLES, replace=False))


def fingerprint(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = f.read(n)
        meta = json.loads(header)
        start = meta[PREFIX + "layers.0.self_attn.q_proj.weight"]["data_offsets"][0]
        f.seek(8 + n + start)
        codes = f.read(65536)
    return {"header_sha256": hashlib.sha256(header).hexdigest(),
            "layer0_q_first64k_sha256": hashlib.sha256(codes).hexdigest()}


def model_config():
    """Ministral3Config with the reference's model facts (eager attention)."""
    from transformers import Ministral3Config
    config = Ministral3Config(
        vocab_size=131072, hidden_size=3072, intermediate_size=9216, num_hidden_layers=26,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, max_position_embeddings=262144,
        rms_norm_eps=1e-5, tie_word_embeddings=True, sliding_window=None, hidden_act="silu",
        rope_parameters={"rope_type": "yarn", "rope_theta": 1e6, "factor": 16.0,
                         "original_max_position_embeddings": 16384, "beta_fast": 32.0, "beta_slow": 1.0,
                         "mscale": 1.0, "mscale_all_dim": 1.0, "llama_4_scaling_beta": 0.1})
    config._attn_implementation = "eager"
    return config


def build_model(path):
    import torch
    from safetensors import safe_open
    from transformers import Ministral3ForCausalLM
    from transformers.models.ministral3.modeling_ministral3 import Ministral3RotaryEmbedding

    config = model_config()
    with torch.device("meta"):
        model = Ministral3ForCausalLM(config)
    state = {}
    with safe_open(path, framework="pt") as f:
        state["model.embed_tokens.weight"] = f.get_tensor(PREFIX + "embed_tokens.weight").float()
        state["model.norm.weight"] = f.get_tensor(PREFIX + "norm.weight").float()
        for layer in range(26):
            p = "layers.%d." % layer
            for norm in ("input_layernorm", "post_attention_layernorm"):
                state["model." + p + norm + ".weight"] = f.get_tensor(PREFIX + p + norm + ".weight").float()
            for lin in LINEARS:
                codes = f.get_tensor(PREFIX + p + lin + ".weight")
                if codes.dtype != torch.float8_e4m3fn:
                    codes = codes.view(torch.float8_e4m3fn)
                scale = f.get_tensor(PREFIX + p + lin + ".weight_scale_inv").float()
                state["model." + p + lin + ".weight"] = codes.float() * scale
    state["lm_head.weight"] = state["model.embed_tokens.weight"]
    model.load_state_dict(state, strict=True, assign=True)
    model.tie_weights()
    model.model.rotary_emb = Ministral3RotaryEmbedding(config)  # its buffers were built on meta
    return model.eval()


def run(path):
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    model = build_model(path)
    ids = prompt_ids()
    layers_out = []
    hooks = [layer.register_forward_hook(lambda _m, _i, out: layers_out.append(
        (out[0] if isinstance(out, tuple) else out).detach().clone())) for layer in model.model.layers]
    normed = []
    hooks.append(model.model.norm.register_forward_hook(lambda _m, _i, out: normed.append(out.detach().clone())))
    with torch.no_grad():
        logits = model(torch.from_numpy(ids)[None, :], use_cache=False).logits[0].float().numpy()
    for h in hooks:
        h.remove()
    hidden = np.stack([t[0].float().numpy() for t in layers_out])  # [26][tokens][3072]
    final = normed[0][0].float().numpy()
    dirs = directions()
    samples = sample_indices()
    top = []
    for pos in range(ids.size):
        order = np.argsort(-logits[pos], kind="stable")[:16]
        top.append({"ids": order.tolist(), "values": r9(logits[pos][order])})
    return {
        "source": "transformers %s Ministral3ForCausalLM, CPU FP32, eager attention, torch %s" % (
            __import__("transformers").__version__, torch.__version__),
        "weights": "seed-0 synthetic checkpoint: E4M3 code value x BF16 weight_scale_inv, BF16 widened",
        "checkpoint": fingerprint(path),
        "ids": ids.tolist(),
        "direction_seed": DIRECTION_SEED,
        "sample_seed": SAMPLE_SEED,
        "hidden_norms": [r9(row) for row in np.linalg.norm(hidden.astype(np.float64), axis=2)],
        "hidden_projections": [[r9(t) for t in layer]
                               for layer in np.einsum("ltc,dc->ltd", hidden.astype(np.float64), dirs)],
        "last_hidden": {str(layer): r9(hidden[layer, -1]) for layer in FULL_LAYERS},
        "last_final_norm": r9(final[-1]),
        "top_logits": top,
        "sampled_logits": [r9(logits[pos][samples]) for pos in range(ids.size)],
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--checkpoint", default=None,
                    help="seed-0 synthetic checkpoint (written with oracle/libsynth.so when absent)")
    ap.add_argument("--out", default=os.path.join(HERE, "transformers_model.json"))
    args = ap.parse_args()
    path = args.checkpoint
    if not path:
        import tempfile
        path = os.path.join(tempfile.gettempdir(), "lunelette_synth_seed0.safetensors")
    if not os.path.exists(path):
        from tests.oracle_lib import synth_checkpoint
        synth_checkpoint(path, 0)
    out = run(path)
    with open(args.out, "w") as f:
        json.dump(out, f, separators=(",", ":"))
        f.write("\n")
    print("wrote %s (%d bytes)" % (args.out, os.path.getsize(args.out)))


if __name__ == "__main__":
    main()
