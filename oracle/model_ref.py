"""Model-level oracle (CPU, fp32 math).  Test infrastructure only.

A restatement of the reference Llama graph (src/llama_pure_compute/model.py:28-477)
evaluated in fp32 from a state dict with the reference's parameter names:
embed -> per layer [RMSNorm (rmsnorm.py:88-96) -> q/k/v -> RoPE (ops.py:27-42,
tables model.py:28-64 gathered at model.py:388-393) -> causal attention with
queries at the end of the keys (tests/test_attention_correctness.py:39-64) ->
o_proj + residual (model.py:305) -> RMSNorm+SwiGLU (ops.py:45-59) -> down +
residual (model.py:323)] -> final norm -> lm_head.  Greedy = argmax
(generate.py:71-76).  The KV cache here is plain per-layer tensors; its slot
semantics are those of kv_cache.cu:25-42 (pinned separately).
"""
from __future__ import annotations

from typing import Dict, List, Tuple

import torch
import torch.nn.functional as F

from .ops_ref import attention_ref


def make_state_dict(cfg: Dict, seed: int, std: float = 0.02) -> Dict[str, torch.Tensor]:
    """Deterministic fp32 weights: N(0, std) for every matrix, drawn from a CPU
    generator in the fixed key order below; RMSNorm weights 1.0."""
    g = torch.Generator().manual_seed(seed)
    D, I, V = cfg["dim"], cfg["inter_dim"], cfg["vocab_size"]
    H, Hkv = cfg["num_heads"], cfg["num_kv_heads"]
    hd = D // H
    sd: Dict[str, torch.Tensor] = {}

    def rn(*shape):
        return torch.randn(*shape, generator=g) * std

    sd["model.embed_tokens.weight"] = rn(V, D)
    for i in range(cfg["num_layers"]):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = torch.ones(D)
        sd[p + "self_attn.q_proj.weight"] = rn(H * hd, D)
        sd[p + "self_attn.k_proj.weight"] = rn(Hkv * hd, D)
        sd[p + "self_attn.v_proj.weight"] = rn(Hkv * hd, D)
        sd[p + "self_attn.o_proj.weight"] = rn(D, H * hd)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(D)
        sd[p + "gate_proj.weight"] = rn(I, D)
        sd[p + "up_proj.weight"] = rn(I, D)
        sd[p + "down_proj.weight"] = rn(D, I)
    sd["model.norm.weight"] = torch.ones(D)
    sd["lm_head.weight"] = rn(V, D)
    return sd


def rope_tables(head_dim: int, end: int, theta: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """precompute_freqs_cis (model.py:28-64)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    f = torch.outer(torch.arange(end, dtype=torch.float32), inv)
    f = torch.cat([f, f], -1)
    return torch.cos(f), torch.sin(f)


class OracleLlama:
    """fp32 evaluation of the reference graph with an explicit KV cache.

    ``table_dtype`` rounds the RoPE tables the way a model cast to that dtype
    holds them (model.py:363-373 buffers follow model.to(dtype))."""

    def __init__(self, cfg: Dict, sd: Dict[str, torch.Tensor], max_seq_len: int,
                 table_dtype: torch.dtype = torch.float32, dtype: torch.dtype = torch.float32,
                 device: str = "cpu"):
        """dtype/device: the arithmetic type and device of the evaluation
        (fp32 on the CPU for the oracle proper; bf16 on a GPU gives a plain
        per-op-rounded torch evaluation of the same graph, used only to size
        the bf16 noise of a model in tests)."""
        self.cfg = cfg
        self.dtype = dtype
        self.w = {k: v.to(device=device, dtype=dtype) for k, v in sd.items()}
        self.H, self.Hkv = cfg["num_heads"], cfg["num_kv_heads"]
        self.D = cfg["dim"] // self.H
        self.eps = cfg.get("rms_norm_eps", 1e-5)
        c, s = rope_tables(self.D, max_seq_len, cfg.get("rope_theta", 10000.0))
        self.cos = c.to(table_dtype).to(device=device, dtype=dtype)
        self.sin = s.to(table_dtype).to(device=device, dtype=dtype)
        self.L = cfg["num_layers"]

    def _norm(self, x, w):
        xf = x.float()  # statistics in fp32 (rmsnorm.py:88-96), result in the working dtype
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * w.float()).to(self.dtype)

    def _rope(self, x, pos):
        h = self.D // 2
        c = self.cos[pos].unsqueeze(2)
        s = self.sin[pos].unsqueeze(2)
        x0, x1 = x[..., :h], x[..., h:]
        return torch.cat([x0 * c[..., :h] - x1 * s[..., :h], x1 * c[..., h:] + x0 * s[..., h:]], -1)

    def forward(self, ids: torch.Tensor, pos: torch.Tensor, cache: List) -> torch.Tensor:
        """ids/pos [B, S]; cache: list of per-layer [k, v] tensors [B, Hkv, T, D]
        (appended in place, T grows).  Returns logits [B, S, V] (fp32)."""
        W = self.w
        B, S = ids.shape
        x = W["model.embed_tokens.weight"][ids]
        for i in range(self.L):
            p = f"model.layers.{i}."
            hn = self._norm(x, W[p + "input_layernorm.weight"])
            q = F.linear(hn, W[p + "self_attn.q_proj.weight"]).view(B, S, self.H, self.D)
            k = F.linear(hn, W[p + "self_attn.k_proj.weight"]).view(B, S, self.Hkv, self.D)
            v = F.linear(hn, W[p + "self_attn.v_proj.weight"]).view(B, S, self.Hkv, self.D)
            q, k = self._rope(q, pos), self._rope(k, pos)
            q, k, v = (t.transpose(1, 2) for t in (q, k, v))
            if cache[i] is None:
                cache[i] = [k, v]
            else:
                cache[i] = [torch.cat([cache[i][0], k], 2), torch.cat([cache[i][1], v], 2)]
            o = attention_ref(q, cache[i][0], cache[i][1], causal=True, sm_scale=self.D ** -0.5)
            x = x + F.linear(o.transpose(1, 2).reshape(B, S, -1), W[p + "self_attn.o_proj.weight"])
            hn = self._norm(x, W[p + "post_attention_layernorm.weight"])
            g = F.linear(hn, W[p + "gate_proj.weight"])
            u = F.linear(hn, W[p + "up_proj.weight"])
            x = x + F.linear(F.silu(g) * u, W[p + "down_proj.weight"])
        x = self._norm(x, W["model.norm.weight"])
        return F.linear(x, W["lm_head.weight"])

    @torch.no_grad()
    def greedy(self, prompt: torch.Tensor, steps: int, forced: torch.Tensor | None = None):
        """Greedy decode of one batch of equal-length prompts [B, P].

        With ``forced`` [B, steps] the oracle is teacher-forced on those tokens
        (to replay another implementation's choices) and reports, per step, its
        own argmax and the logit gap between its top choice and the forced one.
        Returns (tokens [B, steps], gap [B, steps], top2 margin [B, steps])."""
        B, P = prompt.shape
        cache = [None] * self.L
        logits = self.forward(prompt, torch.arange(P).unsqueeze(0).expand(B, -1), cache)[:, -1]
        toks, gaps, margins = [], [], []
        for t in range(steps):
            top2 = torch.topk(logits, 2, dim=-1)
            mine = top2.indices[:, 0]
            margins.append(top2.values[:, 0] - top2.values[:, 1])
            nxt = forced[:, t] if forced is not None else mine
            gaps.append(top2.values[:, 0] - logits.gather(1, nxt[:, None])[:, 0])
            toks.append(mine)
            if t + 1 < steps:
                pos = torch.full((B, 1), P + t, dtype=torch.long)
                logits = self.forward(nxt[:, None], pos, cache)[:, -1]
        return torch.stack(toks, 1), torch.stack(gaps, 1), torch.stack(margins, 1)
