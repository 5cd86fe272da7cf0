"""Qwen2-architecture decoder on the B200 operators, with greedy decoding.

Mirrors the reference's native Qwen2 graph (python/mlx_worker/native_mlx/models/
qwen2.py of the reference): Qwen2Attention (q/k/v with bias, RoPE, paged attention,
o without bias, qwen2.py:46-118), Qwen2Mlp (SwiGLU, qwen2.py:121-134),
Qwen2TransformerBlock (pre-norm residual block, qwen2.py:137-165), the backbone
(embedding, layers, final norm, qwen2.py:168-201) and Qwen2ForCausalLM with an
untied or tied head (qwen2.py:204-227), quantized by nn.quantize as
build_qwen2_model does (qwen2.py:305-324). Greedy decoding takes the argmax of
the last logits per sequence (executor.py:406-414).

Every projection is a quantized_matmul (q/k/v stacked into one launch with their
biases, gate/up stacked with the SwiGLU in the epilogue at decode); the residual
adds ride in the RMSNorm launches; the decode step is replayable as one CUDA graph
(decode_advance moves positions, cache lengths and slots on the device).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import core, nn
from .attention import (PagedBatch, PagedKVCache, decode_advance, paged_attention_decode,
                        paged_attention_prefill, quantized_embedding, rms_norm, rope_kv_append)

__all__ = ["Qwen2Config", "Qwen2Attention", "Qwen2Mlp", "Qwen2TransformerBlock",
           "Qwen2ForCausalLM", "GreedyDecoder"]


@dataclass(frozen=True)
class Qwen2Config:
    """Fields of the reference's Qwen2ModelConfig (qwen2.py:21-38) the graph uses;
    defaults are Qwen2.5-7B's."""
    hidden_size: int = 3584
    intermediate_size: int = 18944
    num_attention_heads: int = 28
    num_key_value_heads: int = 4
    num_hidden_layers: int = 28
    vocab_size: int = 152064
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    tie_word_embeddings: bool = False
    group_size: int = 64
    bits: int = 4

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


def _norm_weight(dim, device, dtype, generator, jitter):
    w = torch.ones(dim, device=device, dtype=torch.float32)
    if jitter:
        w += jitter * torch.randn(dim, device=device, generator=generator)
    return w.to(dtype)


class Qwen2Attention(nn.Module):
    """q/k/v projections (with bias) stacked into one quantized launch, RoPE and the
    paged KV append in one kernel, paged attention, then o_proj (qwen2.py:46-118)."""

    def __init__(self, cfg: Qwen2Config, *, device, dtype, generator, bias_std=0.0):
        D, hd = cfg.hidden_size, cfg.head_dim
        self.n_heads, self.n_kv_heads, self.head_dim = (cfg.num_attention_heads,
                                                        cfg.num_key_value_heads, hd)
        self.scale = hd ** -0.5
        self.rope_base = cfg.rope_theta
        kw = dict(group_size=cfg.group_size, bits=cfg.bits, device=device, dtype=dtype,
                  generator=generator)
        q = nn.QuantizedLinear(D, self.n_heads * hd, bias=True, **kw)
        k = nn.QuantizedLinear(D, self.n_kv_heads * hd, bias=True, **kw)
        v = nn.QuantizedLinear(D, self.n_kv_heads * hd, bias=True, **kw)
        if bias_std:
            for m in (q, k, v):
                m.bias = (bias_std * torch.randn(m.bias.shape, device=device,
                                                 generator=generator)).to(dtype)
        self.qkv_proj = nn.FusedQuantizedLinear([q, k, v])
        self.o_proj = nn.QuantizedLinear(self.n_heads * hd, D, bias=False, **kw)

    def __call__(self, x, batch: PagedBatch, k_cache, v_cache):
        f = self.qkv_proj
        qkv = core.quantized_matmul(x, f.weight, f.scales, f.biases, True, f.group_size, f.bits,
                                    f.mode, bias=f.bias)
        q = rope_kv_append(qkv, batch.positions, batch.slots, k_cache, v_cache, self.n_heads,
                           self.n_kv_heads, self.head_dim, self.rope_base)
        if batch.cu_q is None:
            a = paged_attention_decode(q, k_cache, v_cache, batch.block_table, batch.kv_lens,
                                       batch.max_kv_len, self.scale)
        else:
            a = paged_attention_prefill(q, batch.cu_q, batch.max_q_len, k_cache, v_cache,
                                        batch.block_table, batch.kv_lens, self.scale)
        return self.o_proj(a.reshape(a.shape[0], -1))


class Qwen2Mlp(nn.Module):
    """down(silu(gate(x)) * up(x)) (qwen2.py:121-134); gate and up interleaved into
    one launch whose epilogue applies the SwiGLU at decode."""

    def __init__(self, cfg: Qwen2Config, *, device, dtype, generator):
        kw = dict(group_size=cfg.group_size, bits=cfg.bits, device=device, dtype=dtype,
                  generator=generator)
        gate = nn.QuantizedLinear(cfg.hidden_size, cfg.intermediate_size, bias=False, **kw)
        up = nn.QuantizedLinear(cfg.hidden_size, cfg.intermediate_size, bias=False, **kw)
        self.gate_up_proj = nn.FusedGateUp(gate, up)
        self.down_proj = nn.QuantizedLinear(cfg.intermediate_size, cfg.hidden_size, bias=False,
                                            **kw)

    def __call__(self, x):
        return self.down_proj(self.gate_up_proj(x))


class Qwen2TransformerBlock(nn.Module):
    """Pre-norm block (qwen2.py:137-165): h += attn(norm(h)); h += mlp(norm(h)).
    The residual adds run inside the norms: a block takes the stream h and the
    previous block's pending MLP output, and returns both for the next."""

    def __init__(self, cfg: Qwen2Config, *, device, dtype, generator, norm_jitter=0.0,
                 bias_std=0.0):
        self.self_attn = Qwen2Attention(cfg, device=device, dtype=dtype, generator=generator,
                                        bias_std=bias_std)
        self.mlp = Qwen2Mlp(cfg, device=device, dtype=dtype, generator=generator)
        self.input_layernorm = _norm_weight(cfg.hidden_size, device, dtype, generator,
                                            norm_jitter)
        self.post_attention_layernorm = _norm_weight(cfg.hidden_size, device, dtype, generator,
                                                     norm_jitter)
        self.eps = cfg.rms_norm_eps

    def __call__(self, h, pending, batch, k_cache, v_cache):
        if pending is None:
            x = rms_norm(h, self.input_layernorm, self.eps)
        else:
            x, h = rms_norm(h, self.input_layernorm, self.eps, residual=pending,
                            residual_out=True)
        a = self.self_attn(x, batch, k_cache, v_cache)
        x, h = rms_norm(h, self.post_attention_layernorm, self.eps, residual=a,
                        residual_out=True)
        return h, self.mlp(x)


class Qwen2ForCausalLM(nn.Module):
    """Random-init Qwen2 decoder with every linear layer and the embedding quantized
    (group_size, bits of the config), as an MLX 4-bit checkpoint is laid out."""

    def __init__(self, cfg: Qwen2Config, *, device="cuda", dtype=torch.bfloat16, seed=0,
                 norm_jitter=0.0, bias_std=0.0):
        self.config = cfg
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        emb = nn.Embedding(cfg.vocab_size, cfg.hidden_size, device=device, dtype=dtype,
                           generator=g)
        self.embed_tokens = emb.to_quantized(cfg.group_size, cfg.bits)
        del emb
        self.layers = [Qwen2TransformerBlock(cfg, device=device, dtype=dtype, generator=g,
                                             norm_jitter=norm_jitter, bias_std=bias_std)
                       for _ in range(cfg.num_hidden_layers)]
        self.norm = _norm_weight(cfg.hidden_size, device, dtype, g, norm_jitter)
        if not cfg.tie_word_embeddings:
            self.lm_head = nn.QuantizedLinear(cfg.hidden_size, cfg.vocab_size, bias=False,
                                              group_size=cfg.group_size, bits=cfg.bits,
                                              device=device, dtype=dtype, generator=g)
        self.dtype = dtype

    def embed(self, ids):
        e = self.embed_tokens
        return quantized_embedding(ids, e.weight, e.scales, e.biases, e.group_size, e.bits)

    def hidden(self, ids, batch: PagedBatch, cache: PagedKVCache, last_rows=None):
        """Final-normed hidden states of the step's tokens ids [T] (or of rows
        `last_rows` of them only)."""
        h = self.embed(ids)
        pending = None
        for i, layer in enumerate(self.layers):
            h, pending = layer(h, pending, batch, cache.keys[i], cache.values[i])
        if last_rows is not None:
            h, pending = h[last_rows], pending[last_rows]
        return rms_norm(h, self.norm, self.config.rms_norm_eps, residual=pending)

    def head(self):
        if self.config.tie_word_embeddings:
            e = self.embed_tokens
            return e.weight, e.scales, e.biases, e.group_size, e.bits
        m = self.lm_head
        return m.weight, m.scales, m.biases, m.group_size, m.bits

    def logits(self, x):
        w, s, b, gs, bits = self.head()
        return core.quantized_matmul(x, w, s, b, True, gs, bits)

    def greedy(self, x, out=None):
        w, s, b, gs, bits = self.head()
        return core.quantized_matmul_argmax(x, w, s, b, gs, bits, out=out)


class GreedyDecoder:
    """Batched greedy generation: one prefill of every prompt (flat batch, paged
    attention over each sequence's pages), then decode steps of one token per
    sequence, each step replayable as a CUDA graph with all state on the device."""

    def __init__(self, model: Qwen2ForCausalLM, cache: PagedKVCache, batch_size: int,
                 max_len: int, page_generator=None):
        cfg = model.config
        self.model, self.cache = model, cache
        self.B, self.max_len = batch_size, max_len
        dev = cache.keys[0].device
        self.block_table = cache.allocate([max_len] * batch_size, generator=page_generator)
        self.page = cache.page_size
        self.ids = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.kv_lens = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.slots = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.graph = None
        self.head_dim = cfg.head_dim

    def prefill(self, prompts: torch.Tensor, lengths) -> torch.Tensor:
        """prompts: flat int32 token ids of every sequence, lengths[b] tokens each;
        returns (and holds for the next step) the first greedy token per sequence."""
        dev = self.ids.device
        lengths = [int(n) for n in lengths]
        if max(lengths) >= self.max_len:
            raise ValueError("prompt longer than the sequence capacity")
        cu = [0]
        for n in lengths:
            cu.append(cu[-1] + n)
        batch = PagedBatch(
            block_table=self.block_table,
            kv_lens=torch.tensor(lengths, dtype=torch.int32, device=dev),
            positions=torch.cat([torch.arange(n, dtype=torch.int32) for n in lengths]).to(dev),
            slots=self.cache.slots(self.block_table, [range(n) for n in lengths]),
            max_kv_len=max(lengths),
            cu_q=torch.tensor(cu, dtype=torch.int32, device=dev), max_q_len=max(lengths))
        last = torch.tensor(cu[1:], dtype=torch.long, device=dev) - 1
        x = self.model.hidden(prompts.to(dev, torch.int32), batch, self.cache, last_rows=last)
        self.model.greedy(x, out=self.ids)
        # state of the first decode step: the new token at position n, n + 1 keys
        self.positions.copy_(torch.tensor(lengths, dtype=torch.int32))
        self.kv_lens.copy_(self.positions + 1)
        self.slots.copy_(self.cache.slots(self.block_table, [[n] for n in lengths]))
        return self.ids.clone()

    def step(self, logits_out: torch.Tensor | None = None) -> None:
        """One decode step on the device: embeds self.ids, runs the layers over the
        cache, writes the next greedy tokens into self.ids and advances the state.
        With logits_out [B, vocab], the step's logits are written there too."""
        batch = PagedBatch(block_table=self.block_table, kv_lens=self.kv_lens,
                           positions=self.positions, slots=self.slots, max_kv_len=self.max_len)
        x = self.model.hidden(self.ids, batch, self.cache)
        if logits_out is not None:
            logits_out.copy_(self.model.logits(x))
        self.model.greedy(x, out=self.ids)
        decode_advance(self.positions, self.kv_lens, self.slots, self.block_table, self.page)

    def capture(self, stream: torch.cuda.Stream | None = None) -> None:
        """Records step() as a CUDA graph (after one warm-up step on the capture stream
        has set up its workspaces). Run it after prefill: the warm-up step generates."""
        dev = self.ids.device
        stream = stream or torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            self.step()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            self.step()
        self.graph = g

    def replay(self) -> None:
        self.graph.replay()

    def close(self) -> None:
        self.graph = None
        self.cache.release(self.block_table, [self.max_len] * self.B)
