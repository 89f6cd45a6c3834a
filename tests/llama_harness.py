"""Test harness: a Llama-shaped decoder around a pluggable attention layer.

TEST INFRASTRUCTURE.  It restates the reference model of the end-to-end case
(snapmind/models/llama.py:15-80 with RMSNorm snapmind/layers/normalization/rms_norm.py:11-21,
RoPE snapmind/layers/positional/rope.py:11-61, the gated FFN
snapmind/layers/gated_feed_forward.py:9-20 and SiLU
snapmind/layers/activation/silu.py) so that the attention plugin under test
runs inside the same model the golden vectors were generated with:

* parameters are created in the reference's order and with its names
  (``embed``, ``layers.i.self_attn.{q,k,v,out}_proj``, ``layers.i.input_layernorm``,
  ``layers.i.post_attention_layernorm``, ``layers.i.mlp.{gate,up,down}_proj``,
  ``norm``, ``lm_head``), so :func:`init_weights` reproduces the weights of
  the reference model drawn with the same recipe;
* ``generate`` drives prefill and greedy decode steps the way
  snapmind/engine/generate.py:108-133 does (prefill without position ids,
  then one token per step at position ``step``).

``DenseDictGQA`` is the reference attention math (snapmind/layers/attention/gqa.py:48-85:
dict growth by ``cat``, ``repeat_interleave``, matmul, softmax, matmul) in
torch, used to pin this harness on the CPU; the GPU tests plug in the
package's ``gqa_paged`` layer instead.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class LlamaShape:
    vocab_size: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    n_layers: int
    d_ff: int
    max_seq_len: int
    norm_eps: float = 1e-5
    rope_theta: float = 10000.0


TINYLLAMA = LlamaShape(vocab_size=32000, d_model=2048, n_heads=32, n_kv_heads=4, n_layers=22, d_ff=5632,
                       max_seq_len=2048)
SMALL = LlamaShape(vocab_size=512, d_model=256, n_heads=8, n_kv_heads=2, n_layers=2, d_ff=688, max_seq_len=128)


class Rope(nn.Module):
    """Rotate-half RoPE with cos/sin tables over ``max_seq_len`` positions."""

    def __init__(self, dim: int, max_seq_len: int, theta: float):
        super().__init__()
        inv = 1.0 / (theta ** (torch.arange(0, dim, 2).float() / dim))
        ang = torch.outer(torch.arange(max_seq_len), inv)
        self.register_buffer("cos_cached", torch.cat([ang.cos(), ang.cos()], dim=-1))
        self.register_buffer("sin_cached", torch.cat([ang.sin(), ang.sin()], dim=-1))

    @staticmethod
    def _rotate_half(x):
        h = x.shape[-1] // 2
        return torch.cat((-x[..., h:], x[..., :h]), dim=-1)

    def apply_to_qk(self, q, k, position_ids=None):
        if position_ids is None:
            n = q.shape[-2]
            cos = self.cos_cached[:n][None, None].to(q.dtype)
            sin = self.sin_cached[:n][None, None].to(q.dtype)
        else:
            cos = self.cos_cached[position_ids].unsqueeze(1).to(q.dtype)
            sin = self.sin_cached[position_ids].unsqueeze(1).to(q.dtype)
        return q * cos + self._rotate_half(q) * sin, k * cos + self._rotate_half(k) * sin


class RMSNorm(nn.Module):
    def __init__(self, n: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(n))

    def forward(self, x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight


class GatedFFN(nn.Module):
    def __init__(self, d_model: int, d_ff: int):
        super().__init__()
        self.gate_proj = nn.Linear(d_model, d_ff, bias=False)
        self.up_proj = nn.Linear(d_model, d_ff, bias=False)
        self.down_proj = nn.Linear(d_ff, d_model, bias=False)

    def forward(self, x):
        g = self.gate_proj(x)
        return self.down_proj(g * torch.sigmoid(g) * self.up_proj(x))


class DenseDictGQA(nn.Module):
    """The reference GQA layer's math on a plain dict cache (CPU pin only)."""

    def __init__(self, d_model, n_heads, n_kv_heads=None, dropout=0.0, bias=False, pe=None, head_dim=None):
        super().__init__()
        self.n_heads, self.n_kv_heads = n_heads, n_kv_heads or n_heads
        self.head_dim = head_dim or d_model // n_heads
        self.pe = pe
        self.q_proj = nn.Linear(d_model, n_heads * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(d_model, self.n_kv_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(d_model, self.n_kv_heads * self.head_dim, bias=bias)
        self.out_proj = nn.Linear(n_heads * self.head_dim, d_model, bias=bias)

    def forward(self, x, kv_cache=None, position_ids=None, mask=None):
        b, t, _ = x.shape
        q = self.q_proj(x).view(b, t, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(b, t, self.n_kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(b, t, self.n_kv_heads, self.head_dim).transpose(1, 2)
        if self.pe is not None:
            q, k = self.pe.apply_to_qk(q, k, position_ids)
        if kv_cache is not None:
            if kv_cache["k"] is not None:
                k = torch.cat([kv_cache["k"], k], dim=-2)
                v = torch.cat([kv_cache["v"], v], dim=-2)
            kv_cache["k"], kv_cache["v"] = k, v
        rep = self.n_heads // self.n_kv_heads
        k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
        s = torch.matmul(q, k.transpose(-2, -1)) * self.head_dim ** -0.5
        if mask is not None:
            s = s + mask.to(s.dtype)
        o = torch.matmul(F.softmax(s, dim=-1), v)
        return self.out_proj(o.transpose(1, 2).reshape(b, t, -1)), None


class Block(nn.Module):
    def __init__(self, shape: LlamaShape, pe: Rope, attn_cls):
        super().__init__()
        self.self_attn = attn_cls(d_model=shape.d_model, n_heads=shape.n_heads, n_kv_heads=shape.n_kv_heads,
                                  dropout=0.0, bias=False, pe=pe)
        self.input_layernorm = RMSNorm(shape.d_model, shape.norm_eps)
        self.post_attention_layernorm = RMSNorm(shape.d_model, shape.norm_eps)
        self.mlp = GatedFFN(shape.d_model, shape.d_ff)

    def forward(self, x, kv_cache=None, position_ids=None):
        prefill = kv_cache is None or kv_cache.get("k") is None
        mask = None
        if prefill:
            n = x.shape[1]
            mask = torch.triu(torch.full((n, n), float("-inf")), diagonal=1).to(x.device)
        a, _ = self.self_attn(self.input_layernorm(x), kv_cache=kv_cache, mask=mask, position_ids=position_ids)
        x = x + a
        return x + self.mlp(self.post_attention_layernorm(x))


class LlamaHarness(nn.Module):
    def __init__(self, shape: LlamaShape, attn_cls=DenseDictGQA):
        super().__init__()
        self.shape = shape
        self.embed = nn.Embedding(shape.vocab_size, shape.d_model)
        self.pe = Rope(shape.d_model // shape.n_heads, shape.max_seq_len, shape.rope_theta)
        self.layers = nn.ModuleList([Block(shape, self.pe, attn_cls) for _ in range(shape.n_layers)])
        self.norm = RMSNorm(shape.d_model, shape.norm_eps)
        self.lm_head = nn.Linear(shape.d_model, shape.vocab_size, bias=False)

    def forward(self, tokens, kv_cache=None, position_ids=None):
        x = self.embed(tokens)
        for i, layer in enumerate(self.layers):
            x = layer(x, kv_cache=None if kv_cache is None else kv_cache[i], position_ids=position_ids)
        return self.lm_head(self.norm(x))


def init_weights(model: nn.Module, seed: int) -> None:
    """N(0, 0.02) for every parameter of 2 or more dims, in ``named_parameters``
    order from one CPU generator; 1-dim parameters (norm weights) = 1."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for _, p in model.named_parameters():
            if p.dim() >= 2:
                p.copy_(torch.empty(p.shape).normal_(0.0, 0.02, generator=g))
            else:
                p.fill_(1.0)


def prompt_ids(vocab: int, n: int, seed: int) -> torch.Tensor:
    return torch.randint(0, vocab, (n,), generator=torch.Generator().manual_seed(seed))


@torch.no_grad()
def generate(model: nn.Module, prompt: torch.Tensor, n_tokens: int, kv_cache) -> tuple[list[int], list]:
    """Greedy generation of ``n_tokens`` ids: prefill, then ``n_tokens - 1``
    decode steps.  Returns the ids and each step's top-2 (values, ids) logits."""
    model.eval()
    dev = next(model.parameters()).device
    logits = model(prompt[None].to(dev), kv_cache=kv_cache)[0, -1]
    ids, tops = [], []
    step = prompt.numel()
    for i in range(n_tokens):
        top = torch.topk(logits.float(), 2)
        tops.append((top.values.cpu().tolist(), top.indices.cpu().tolist()))
        ids.append(int(logits.argmax(dim=-1)))
        if i == n_tokens - 1:
            break
        tok = torch.tensor([[ids[-1]]], dtype=torch.long, device=dev)
        logits = model(tok, kv_cache=kv_cache, position_ids=torch.tensor([step], device=dev))[0, -1]
        step += 1
    return ids, tops


def param_checksums(model: nn.Module) -> list[tuple[str, list[int], int]]:
    """(name, shape, int64 sum of the fp32 bit patterns) per parameter: exact and
    independent of summation order, so it is equal on any machine."""
    return [(n, list(p.shape), int(p.detach().float().contiguous().view(torch.int32).sum(dtype=torch.int64)))
            for n, p in model.named_parameters()]
