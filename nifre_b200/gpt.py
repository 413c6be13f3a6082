"""GPT-2 style causal LM whose forward runs a whole continuous-batching step.

Parameters, module names and construction order follow the reference's
``src/inference/models/gpt.py:13-141`` and ``models/layers.py:7-47``: with the
same seed, ``GptModel(cfg)`` draws exactly the reference's initial weights and
loads its checkpoints' ``state_dict`` unchanged.

The forward is different.  The reference runs a left-padded ``(B, T)`` batch
per call and loops over rows for positions (``gpt.py:108-126``) and attention.
Here one step is a flat list of ``T`` tokens from any mix of prefill chunks
and decodes (``forward_step``): embeddings, one fused QKV GEMM per layer whose
K/V column slices go straight into the paged pools (``nf_kv_append``), one
``nf_paged_attention`` launch for all rows, and logits only for the rows that
are sampled.  Dense matmuls are cuBLAS through torch; layer norm and GELU are
torch ops with the reference's formulas (biased variance, eps 1e-5; tanh
GELU).  ``forward`` keeps the reference's call signature for callers that
still pass padded batches.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import Attention

GPT_CONFIG_124M = {
    "vocab_size": 50257,
    "context_length": 256,
    "emb_dim": 768,
    "num_heads": 12,
    "num_layers": 12,
    "drop_rate": 0.1,
    "qkv_bias": False,
}

_LN_EPS = 1e-5


class GELU(nn.Module):
    """tanh approximation (layers.py:7-15)."""

    def forward(self, x):
        return F.gelu(x, approximate="tanh")


class LayerNorm(nn.Module):
    """Parameters ``scale``/``shift`` as in layers.py:18-31; biased variance, eps 1e-5."""

    def __init__(self, emb_dim):
        super().__init__()
        self.eps = _LN_EPS
        self.scale = nn.Parameter(torch.ones(emb_dim))
        self.shift = nn.Parameter(torch.zeros(emb_dim))

    def forward(self, x):
        return F.layer_norm(x, (x.shape[-1],), self.scale, self.shift, self.eps)


class FeedForward(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        e = cfg["emb_dim"]
        self.layers = nn.Sequential(nn.Linear(e, 4 * e), GELU(), nn.Linear(4 * e, e))

    def forward(self, x):
        return self.layers(x)


class GptAttention(nn.Module):
    def __init__(self, d_in, d_out, num_heads, dropout=0.0, qkv_bias=False):
        super().__init__()
        self.d_out = d_out
        self.num_heads = num_heads
        self.head_dim = d_out // num_heads
        self.W_query = nn.Linear(d_in, d_out, bias=qkv_bias)
        self.W_key = nn.Linear(d_in, d_out, bias=qkv_bias)
        self.W_value = nn.Linear(d_in, d_out, bias=qkv_bias)
        self.out_proj = nn.Linear(d_out, d_out)
        self.attn = Attention(num_heads, self.head_dim, dropout=dropout)
        self._fused = None  # (versions, weight, bias) of the concatenated projection

    def qkv_params(self):
        """One (3*d_out, d_in) weight (and bias) for the fused projection, rebuilt when a parameter changes."""
        lins = (self.W_query, self.W_key, self.W_value)
        key = tuple((l.weight.data_ptr(), l.weight._version) for l in lins)
        if self._fused is None or self._fused[0] != key:
            w = torch.cat([l.weight.detach() for l in lins], 0)
            b = torch.cat([l.bias.detach() for l in lins], 0) if lins[0].bias is not None else None
            self._fused = (key, w, b)
        return self._fused[1], self._fused[2]

    def forward(self, x, kv_cache=None, layer_id=None, input_lens=None, cache_batch_indices=None):
        q, k, v = self.W_query(x), self.W_key(x), self.W_value(x)
        ctx = self.attn(q, k, v, kv_cache=kv_cache, layer_id=layer_id, input_lens=input_lens,
                        cache_batch_indices=cache_batch_indices)
        return self.out_proj(ctx)


class TransformerBlock(nn.Module):
    # bf16/fp16 models project and append in one tensor-core kernel on the flat step path
    fused_projection = True

    def __init__(self, cfg):
        super().__init__()
        self.att = GptAttention(cfg["emb_dim"], cfg["emb_dim"], cfg["num_heads"], dropout=cfg["drop_rate"],
                                qkv_bias=cfg["qkv_bias"])
        self.ff = FeedForward(cfg)
        self.norm1 = LayerNorm(cfg["emb_dim"])
        self.norm2 = LayerNorm(cfg["emb_dim"])
        self.drop_shortcut = nn.Dropout(cfg["drop_rate"])

    def forward(self, x, kv_cache=None, layer_id=None, input_lens=None, cache_batch_indices=None):
        x = x + self.drop_shortcut(self.att(self.norm1(x), kv_cache=kv_cache, layer_id=layer_id,
                                            input_lens=input_lens, cache_batch_indices=cache_batch_indices))
        return x + self.drop_shortcut(self.ff(self.norm2(x)))

    def step(self, x, cache, plan, layer_id):
        """One layer over a flat step of rows (T, E), inference only (no dropout); see GptModel.forward_step."""
        E = x.shape[1]
        w, b = self.att.qkv_params()
        xn = self.norm1(x)
        if self.fused_projection and cache.projection_fusable(xn, plan, E) and w.dtype == cache.dtype:
            # 16-bit model: one tcgen05 kernel projects and scatters K/V into the pools (nf_qkv_append)
            q = torch.empty(x.shape[0], E, device=x.device, dtype=x.dtype)
            cache.project_append_step(layer_id, xn, w, b, plan, q)
        else:
            qkv = F.linear(xn, w, b)
            cache.append_step(layer_id, qkv[:, E:2 * E], qkv[:, 2 * E:], plan)
            q = qkv[:, :E]
        ctx = torch.empty(x.shape[0], E, device=x.device, dtype=x.dtype)
        cache.attention_step(layer_id, q, plan, ctx)
        x = x + self.att.out_proj(ctx)
        return x + self.ff(self.norm2(x))


class GptModel(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        self.token_embedding = nn.Embedding(cfg["vocab_size"], cfg["emb_dim"])
        self.position_embedding = nn.Embedding(cfg["context_length"], cfg["emb_dim"])
        self.drop_embedding = nn.Dropout(cfg["drop_rate"])
        self.trf_blocks = nn.ModuleList([TransformerBlock(cfg) for _ in range(cfg["num_layers"])])
        self.final_norm = LayerNorm(cfg["emb_dim"])
        self.out_head = nn.Linear(cfg["emb_dim"], cfg["vocab_size"], bias=False)

    @torch.no_grad()
    def forward_step(self, token_ids: torch.Tensor, positions: torch.Tensor, cache, plan,
                     sample_rows: torch.Tensor) -> torch.Tensor:
        """Logits (len(sample_rows), vocab) of one continuous-batching step.

        ``token_ids``/``positions``: (T,) int64 on the device, row r being token
        r of the step in the order of ``plan`` (built by ``cache.plan`` over the
        same rows); ``sample_rows``: rows whose next-token logits are needed.
        """
        x = self.token_embedding(token_ids) + self.position_embedding(positions)
        for layer_id, block in enumerate(self.trf_blocks):
            x = block.step(x, cache, plan, layer_id)
        return self.out_head(self.final_norm(x.index_select(0, sample_rows)))

    def forward(self, in_idx, kv_cache=None, input_lens=None, cache_batch_indices=None):
        """The reference's call (gpt.py:103-141): left-padded (B, T) ids -> (B, T, vocab) logits.

        With a cache, real tokens run as one flat step; pad positions get zero
        logits (the reference leaves them unused).
        """
        B, T = in_idx.shape
        if kv_cache is None:
            x = self.token_embedding(in_idx) + self.position_embedding(torch.arange(T, device=in_idx.device))
            x = self.drop_embedding(x)
            for block in self.trf_blocks:
                x = block(x)
            return self.out_head(self.final_norm(x))
        slots = list(range(B)) if cache_batch_indices is None else [int(s) for s in cache_batch_indices]
        if T == 1:
            lens = [1] * B
        elif input_lens is None:
            raise ValueError("input_lens is required for batched prefill with kv_cache")
        else:
            lens = [int(n) for n in input_lens.tolist()]
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]]).tolist()
        ids = torch.cat([in_idx[i, T - n:] for i, n in enumerate(lens)])
        pos0 = kv_cache.pos_host[slots]
        positions = torch.from_numpy(np.concatenate([np.arange(p, p + n) for p, n in zip(pos0, lens)]))
        rows = torch.arange(sum(lens), device=in_idx.device)
        plan = kv_cache.plan(slots, lens, starts, q_heads=self.cfg["num_heads"])
        logits = self.forward_step(ids, positions.to(in_idx.device), kv_cache, plan, rows)
        out = torch.zeros(B, T, logits.shape[-1], device=logits.device, dtype=logits.dtype)
        for i, (s, n) in enumerate(zip(starts, lens)):
            out[i, T - n:] = logits[s:s + n]
        return out


def gpt_model_config(cfg: dict, pad_token_id: int = 50256):
    """ModelConfig of a GPT config dict (backends/gpt.py:30-44)."""
    from .data_model import ModelConfig
    return ModelConfig(num_layers=cfg["num_layers"], max_seq_len=cfg["context_length"], n_heads=cfg["num_heads"],
                       head_dim=cfg["emb_dim"] // cfg["num_heads"], vocab_size=cfg["vocab_size"],
                       pad_token_id=pad_token_id, block_size=cfg.get("block_size", 16))


class GptInferenceModel:
    """The engine's model protocol around GptModel (backends/gpt.py:27-62), plus ``forward_step``."""

    def __init__(self, model: GptModel, pad_token_id: int = 50256):
        self._model = model
        self.config = gpt_model_config(model.cfg, pad_token_id)

    @property
    def module(self) -> GptModel:
        return self._model

    @property
    def dtype(self):
        return next(self._model.parameters()).dtype

    def eval(self) -> None:
        self._model.eval()

    def forward_step(self, token_ids, positions, cache, plan, sample_rows):
        return self._model.forward_step(token_ids, positions, cache, plan, sample_rows)

    def __call__(self, token_ids, kv_cache=None, input_lens=None, cache_batch_indices=None):
        with torch.no_grad():
            return self._model(token_ids, kv_cache=kv_cache, input_lens=input_lens,
                               cache_batch_indices=cache_batch_indices)


def param_count(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


def flops_per_token(cfg: dict, ctx: int) -> float:
    """Dense forward FLOPs of one token with `ctx` keys (projections, MLP, head, attention)."""
    e, L, v = cfg["emb_dim"], cfg["num_layers"], cfg["vocab_size"]
    return 2.0 * L * (4 * e * e + 8 * e * e) + 2.0 * e * v + 4.0 * L * e * ctx
