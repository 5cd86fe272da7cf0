"""The Qwen2-architecture decoder end to end against a whole-sequence numpy forward.

A small random-init model (2 layers, GQA, q/k/v biases, jittered norm weights) runs a
ragged prefill of three prompts over shuffled cache pages, then greedy decode steps
through the paged cache; at every step the logits of each sequence's last token are
compared with oracle/decoder_np.forward over the sequence so far (no cache: every
position recomputed, with the tokens the GPU chose). Greedy tokens must be the
argmax of the GPU's own logits (the argmax epilogue sees the same rounded logits),
and a CUDA-graph replay of the decode step must reproduce the eager steps bit for bit.

Tolerance: max|d| <= 2e-2 * max|ref| on the logits (bf16 activations; the oracle
computes norms, angles and softmax in float64)."""
import numpy as np
import pytest
import torch

from mlx_server_runtime_b200 import qwen2
from mlx_server_runtime_b200.attention import PagedKVCache
from oracle import decoder_np as D, oracle_np as O

from gpu_util import close, to_np

pytestmark = pytest.mark.gpu

DT = "bfloat16"


def _q(m):
    return tuple(to_np(t) for t in (m.weight, m.scales, m.biases))


def _f(t):
    return O.to_f32(to_np(t), DT)


def host_params(model):
    P = {"embed": _q(model.embed_tokens), "norm": _f(model.norm), "head": _q(model.lm_head),
         "layers": []}
    for layer in model.layers:
        at, mlp = layer.self_attn, layer.mlp
        P["layers"].append({
            "in_norm": _f(layer.input_layernorm), "post_norm": _f(layer.post_attention_layernorm),
            "qkv": _q(at.qkv_proj), "qkv_bias": to_np(at.qkv_proj.bias), "o": _q(at.o_proj),
            "gate_up": _q(mlp.gate_up_proj), "down": _q(mlp.down_proj)})
    return P


CONFIGS = {
    # head_dim 64, 4 query heads per kv head, K/group a multiple of 8 (TMA decode kernel)
    "hd64": qwen2.Qwen2Config(hidden_size=512, intermediate_size=1024, num_attention_heads=8,
                              num_key_value_heads=2, num_hidden_layers=2, vocab_size=512,
                              rope_theta=1e4),
    # head_dim 128, 7 query heads per kv head as in Qwen2.5-7B
    "hd128": qwen2.Qwen2Config(hidden_size=896, intermediate_size=1536, num_attention_heads=7,
                               num_key_value_heads=1, num_hidden_layers=2, vocab_size=640,
                               rope_theta=1e6),
}


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_prefill_and_decode_match_whole_sequence_forward(name):
    cfg = CONFIGS[name]
    model = qwen2.Qwen2ForCausalLM(cfg, seed=3, norm_jitter=0.1, bias_std=0.5)
    cache = PagedKVCache(cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim,
                         num_pages=64)
    lengths = [5, 37, 130]
    dec = qwen2.GreedyDecoder(model, cache, len(lengths), max_len=160,
                              page_generator=torch.Generator().manual_seed(4))
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, cfg.vocab_size, n).astype(np.int32) for n in lengths]
    first = dec.prefill(torch.from_numpy(np.concatenate(prompts)), lengths)
    P = host_params(model)
    ocfg = {"group_size": cfg.group_size, "bits": cfg.bits, "heads": cfg.num_attention_heads,
            "kv_heads": cfg.num_key_value_heads, "head_dim": cfg.head_dim,
            "eps": cfg.rms_norm_eps, "rope_theta": cfg.rope_theta}
    seqs = [list(p) for p in prompts]
    toks = first.cpu().numpy()
    for b in range(len(lengths)):
        _, lg = D.forward(P, ocfg, seqs[b])
        ref = lg[-1]
        assert toks[b] == int(np.argmax(ref)) or \
            np.sort(ref)[-1] - ref[toks[b]] <= 2e-2 * np.abs(ref).max()
    logits = torch.empty(len(lengths), cfg.vocab_size, dtype=torch.bfloat16, device="cuda")
    for step in range(4):
        for b in range(len(lengths)):
            seqs[b].append(int(toks[b]))
        dec.step(logits_out=logits)
        got = _f(logits)
        new = dec.ids.cpu().numpy()
        for b in range(len(lengths)):
            _, lg = D.forward(P, ocfg, seqs[b])
            close(O.from_f32(got[b], DT), O.from_f32(lg[-1], DT), DT)
            # the greedy epilogue picks the first maximum of the logits the step wrote
            assert new[b] == int(np.argmax(got[b]))
        toks = new
    dec.close()


def test_graph_replay_equals_eager_steps():
    cfg = CONFIGS["hd64"]
    model = qwen2.Qwen2ForCausalLM(cfg, seed=7, norm_jitter=0.1, bias_std=0.5)
    lengths = [9, 20, 140, 3]
    rng = np.random.default_rng(8)
    flat = torch.from_numpy(rng.integers(0, cfg.vocab_size, sum(lengths)).astype(np.int32))
    runs = []
    for use_graph in (False, True):
        cache = PagedKVCache(cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim,
                             num_pages=64)
        dec = qwen2.GreedyDecoder(model, cache, len(lengths), max_len=160)
        out = [dec.prefill(flat, lengths).cpu()]
        if use_graph:
            dec.capture()          # its warm-up step generates the second token
            out.append(dec.ids.cpu())
            for _ in range(5):
                dec.replay()
                out.append(dec.ids.cpu())
        else:
            for _ in range(6):
                dec.step()
                out.append(dec.ids.cpu())
        runs.append(torch.stack(out))
        dec.close()
    assert torch.equal(runs[0], runs[1])
