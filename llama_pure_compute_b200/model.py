"""Llama model graph on the sm_100a hot-path kernels.

Class names, constructor arguments, parameter names (state-dict keys) and
forward signatures follow src/llama_pure_compute/model.py:28-580, so
checkpoints and call sites carry over.  What runs underneath:

  input_layernorm   -> lpc_rmsnorm_forward (model.py:305 via rmsnorm.py)
  q/k/v projections -> one GEMM on the concatenated [(H+2Hkv)*D, dim] weight
                       (cuBLAS through torch; the q/k/v parameters are views of it)
  RoPE + KV append  -> lpc_rope_kv_append (model.py:146-168 fused into one kernel;
                       per-row positions, so batches may be ragged)
                       decode steps of <= FUSED_QKV_MAX_TOKENS tokens (head_dim
                       128): projection, RoPE and KV append in one kernel,
                       lpc_qkv_rope_append, on a packed copy of the q/k/v
                       weight; with ``norm_in_gemm`` (default) the input norm
                       too, its weight folded into the copy
  attention         -> decode: lpc_decode_attention over device seq_lens
                       (no per-layer .item() sync, model.py:159-161);
                       prefill / no cache: lpc_flash_attention (tcgen05)
  o_proj + residual -> one addmm (residual added in the GEMM epilogue); decode
                       steps of <= PACKED_RESIDUAL_MAX_TOKENS tokens: lpc_wsgemm
                       (residual epilogue) on a packed copy of o_proj
  post norm + SwiGLU-> lpc_rmsswiglu_forward (model.py:315-321; row norm, then
                       the tcgen05 GEMM with the SiLU*up epilogue launched
                       under it, no torch.cat of weights), or with
                       ``fuse_mlp_norm`` lpc_rmsswiglu_folded_forward (the norm
                       inside the CTA-pair GEMM on gate/up with the norm weight
                       folded in); decode steps of <= 128 tokens: row norm +
                       lpc_wsgemm on a packed copy of gate/up; up to
                       NORM_IN_GEMM_MAX_TOKENS tokens with ``norm_in_gemm``
                       (default) one lpc_wsgemm, norm weight folded
  down + residual   -> one addmm; decode steps of <= PACKED_RESIDUAL_MAX_TOKENS
                       tokens: lpc_wsgemm (residual epilogue), packed down_proj
  lm_head           -> all positions by default (model.py:475), or only the
                       last one with ``last_token_only=True``

There is no PyTorch attention fallback: a custom additive ``mask`` raises.
"""
from __future__ import annotations

import math
import os
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import LlamaModelConfig
from .flash_attention import flash_attention_v2
from .kv_manager import KVCacheManager
from .ops import rmsswiglu_forward, rope_forward
from .rmsnorm import RMSNorm

# Decode steps with at most this many tokens run the SwiGLU GEMM on packed
# weights (lpc_wsgemm); the packed copy of gate/up is built on first use.
PACKED_SWIGLU_MAX_TOKENS = 128
# Decode steps with at most this many tokens run the input norm, the q/k/v
# projection, RoPE and the KV append in one kernel (lpc_qkv_rope_append) on a
# packed copy of the q/k/v weight, built on first use.
FUSED_QKV_MAX_TOKENS = 32
# Decode steps with at most this many tokens (and LlamaModel.norm_in_gemm)
# normalise inside those packed GEMMs: the epilogue warps sum each token row's
# squares from global memory while the weights stream, and the norm weight is
# folded into the packed copy.  32-token SwiGLU 30.0 us against 35.3 for the
# norm kernel + GEMM, q/k/v 23.0 against 22.5 + the norm; at 128 tokens the
# rows' re-reads cost more than the norm kernel (49.8 against 43.5 us).
NORM_IN_GEMM_MAX_TOKENS = 64
# Decode steps with at most this many tokens run o_proj and down_proj with the
# residual add on packed copies of their weights (lpc_wsgemm): 13.3 against
# 15.6 us (cuBLAS) for o_proj and 22.0 against 25.0 for down_proj at 32
# tokens.  With the norms inside the packed GEMMs every kernel of the layer
# after attention is a programmatic launch under the one before it: decode
# step 4.35 against 4.46 ms at 32 sequences, 3.52 against 3.74 at 16; at 64
# sequences it loses (6.07 against 5.90 ms).
PACKED_RESIDUAL_MAX_TOKENS = 32

__all__ = ["precompute_freqs_cis", "LlamaAttention", "LlamaDecodeLayer", "LlamaModel",
           "LlamaForCausalLM"]


def precompute_freqs_cis(dim: int, end: int, theta: float = 10000.0,
                         device: Optional[torch.device] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables [end, dim], halves duplicated (model.py:28-64)."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    t = torch.arange(end, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    f = torch.cat([f, f], dim=-1)
    return torch.cos(f), torch.sin(f)


def _weight_key(w: torch.Tensor):
    """Identity of a weight's current contents for derived copies (stacked or
    packed weights): storage, version counter, dtype, device.  Inference
    tensors (a model built under torch.inference_mode) have no version
    counter; they are keyed on their storage alone."""
    try:
        ver = w._version
    except RuntimeError:
        ver = None
    return (w.data_ptr(), ver, w.dtype, w.device)


class _StepContext:
    """Per-forward data shared by all layers (computed once, not per layer)."""

    __slots__ = ("positions", "seq_lens", "start_pos", "cos_table", "sin_table", "decode",
                 "workspace", "packed_max", "fused_qkv_max", "resid_max", "fuse_norm",
                 "norm_in_gemm")

    def __init__(self):
        self.positions = None
        self.seq_lens = None
        self.start_pos = None
        self.cos_table = None
        self.sin_table = None
        self.decode = False
        self.packed_max = 0
        self.fused_qkv_max = 0
        self.resid_max = 0
        self.fuse_norm = False
        self.norm_in_gemm = False
        self.workspace = None


def _packable(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype
            and x.shape[-1] % 64 == 0 and w.is_cuda)


class LlamaAttention(nn.Module):
    def __init__(self, config: LlamaModelConfig) -> None:
        super().__init__()
        self.config = config
        self.dim = config.dim
        self.num_heads = config.num_heads
        self.num_kv_heads = config.num_kv_heads
        self.head_dim = config.head_dim
        self.num_kv_groups = config.gqa_group_size
        self.scale = self.head_dim ** -0.5
        self.q_proj = nn.Linear(self.dim, self.num_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(self.dim, self.num_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(self.dim, self.num_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, self.dim, bias=False)
        self._qkv_key = None
        self._qkv = None
        self._packed_qkv = None
        self._packed_qkv_key = None
        self._packed_o = None
        self._packed_o_key = None

    def qkv_weight(self) -> torch.Tensor:
        """[(H+2Hkv)*D, dim] weight; q/k/v parameters are re-pointed into it once."""
        ws = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        key = tuple(_weight_key(w) for w in ws)
        if self._qkv is None or key != self._qkv_key:
            fused = torch.cat([w.detach() for w in ws], dim=0).contiguous()
            n_q = self.num_heads * self.head_dim
            n_kv = self.num_kv_heads * self.head_dim
            with torch.no_grad():
                self.q_proj.weight.data = fused[:n_q]
                self.k_proj.weight.data = fused[n_q:n_q + n_kv]
                self.v_proj.weight.data = fused[n_q + n_kv:]
            self._qkv = fused
            ws = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
            self._qkv_key = tuple(_weight_key(w) for w in ws)
        return self._qkv

    def packed_qkv(self, norm_weight: Optional[torch.Tensor] = None):
        """The q/k/v weight in the packed "heads" layout (lpc_pack_weights),
        with ``norm_weight`` (the input RMSNorm's) folded in when given; built
        on first use and rebuilt when a weight changes."""
        from .packed_linear import PackedWeight
        w = self.qkv_weight()
        # the stacked weight may be an inference tensor (no version counter):
        # key on the q/k/v parameters it was built from
        key = (w.data_ptr(), self._qkv_key, None if norm_weight is None else _weight_key(norm_weight))
        if self._packed_qkv is None or key != self._packed_qkv_key:
            self._packed_qkv = PackedWeight(w, layout="heads", norm_weight=norm_weight)
            self._packed_qkv_key = key
        return self._packed_qkv

    def packed_o(self):
        """o_proj in the packed linear layout, built on first use."""
        from .packed_linear import PackedWeight
        key = _weight_key(self.o_proj.weight)
        if self._packed_o is None or key != self._packed_o_key:
            self._packed_o = PackedWeight(self.o_proj.weight)
            self._packed_o_key = key
        return self._packed_o

    def _fused_qkv(self, x: torch.Tensor, ctx: Optional[_StepContext]) -> bool:
        return (ctx is not None and ctx.decode and 0 < x.numel() // x.shape[-1] <= ctx.fused_qkv_max
                and self.head_dim == 128 and x.dtype in (torch.bfloat16, torch.float16)
                and ctx.cos_table is not None and ctx.cos_table.dtype == x.dtype
                and self.q_proj.weight.dtype == x.dtype and x.shape[-1] % 64 == 0)

    def forward(
        self,
        x: torch.Tensor,
        *,
        positions: torch.Tensor,
        cos: torch.Tensor,
        sin: torch.Tensor,
        kv_cache: Optional[KVCacheManager],
        layer_idx: int,
        mask: Optional[torch.Tensor] = None,
        use_triton_flash: bool = True,
        ctx: Optional[_StepContext] = None,
        input_norm: Optional[RMSNorm] = None,
    ) -> torch.Tensor:
        """Attention block output before the residual add (model.py:110-249).

        ``input_norm``: ``x`` is the raw residual stream and this RMSNorm is
        applied inside the fused decode kernel (only on the path where
        ``fuses_input_norm`` holds)."""
        if mask is not None:
            raise NotImplementedError(
                "custom attention masks are not supported by the B200 kernels; causal attention "
                "is applied by passing mask=None")
        B, S, _ = x.shape
        H, Hkv, D = self.num_heads, self.num_kv_heads, self.head_dim
        if kv_cache is not None and self._fused_qkv(x, ctx):
            # decode-sized: (input norm +) projection + RoPE + KV append in one kernel
            if input_norm is not None:
                return kv_cache.attend(layer_idx=layer_idx, x=x,
                                       packed_qkv=self.packed_qkv(input_norm.weight),
                                       norm_eps=input_norm.eps, positions=positions, ctx=ctx,
                                       num_heads=H, scale=self.scale)
            return kv_cache.attend(layer_idx=layer_idx, x=x, packed_qkv=self.packed_qkv(),
                                   positions=positions, ctx=ctx, num_heads=H, scale=self.scale)
        if input_norm is not None:
            raise ValueError("input_norm is only applied inside the fused decode kernel")
        qkv = F.linear(x, self.qkv_weight())
        if kv_cache is not None:
            if ctx is None or ctx.cos_table is None:
                raise ValueError("cached attention needs the model's RoPE tables (call via LlamaModel)")
            # RoPE + append + attention over the cache (dense or ragged layout)
            out = kv_cache.attend(layer_idx=layer_idx, qkv=qkv, positions=positions, ctx=ctx,
                                  num_heads=H, scale=self.scale)
        else:
            q = qkv[..., : H * D].reshape(B, S, H, D)
            k = qkv[..., H * D:(H + Hkv) * D].reshape(B, S, Hkv, D)
            v = qkv[..., (H + Hkv) * D:].reshape(B, S, Hkv, D)
            q, k = rope_forward(q, k, cos, sin, positions)
            out = flash_attention_v2(q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous(),
                                     v.transpose(1, 2).contiguous(), causal=True,
                                     sm_scale=self.scale)
            out = out.transpose(1, 2).reshape(B, S, H * D)
        return out

    def fuses_input_norm(self, x: torch.Tensor, ctx: Optional[_StepContext]) -> bool:
        """Whether this step's input norm runs inside the q/k/v kernel."""
        return (ctx is not None and ctx.norm_in_gemm and self._fused_qkv(x, ctx)
                and x.numel() // x.shape[-1] <= NORM_IN_GEMM_MAX_TOKENS)

    def project_out(self, attn: torch.Tensor, residual: torch.Tensor,
                    ctx: Optional[_StepContext] = None) -> torch.Tensor:
        """residual + attn @ o_proj^T in one GEMM (the residual added in the
        epilogue): the packed weight-streaming kernel for decode steps of at
        most ``ctx.resid_max`` tokens, else cuBLAS (beta=1 epilogue)."""
        shp = residual.shape
        r2 = residual.reshape(-1, shp[-1])
        a2 = attn.reshape(-1, attn.shape[-1])
        if (ctx is not None and ctx.decode and a2.shape[0] <= ctx.resid_max
                and _packable(a2, self.o_proj.weight) and r2.is_contiguous()):
            from .packed_linear import packed_linear
            return packed_linear(a2, self.packed_o(), "residual", resid=r2).view(shp)
        return torch.addmm(r2, a2, self.o_proj.weight.t()).view(shp)


class LlamaDecodeLayer(nn.Module):
    def __init__(self, config: LlamaModelConfig, layer_idx: int) -> None:
        super().__init__()
        self.layer_idx = layer_idx
        self.input_layernorm = RMSNorm(config.dim, eps=config.rms_norm_eps)
        self.self_attn = LlamaAttention(config)
        self.post_attention_layernorm = RMSNorm(config.dim, eps=config.rms_norm_eps)
        self.gate_proj = nn.Linear(config.dim, config.inter_dim, bias=False)
        self.up_proj = nn.Linear(config.dim, config.inter_dim, bias=False)
        self.down_proj = nn.Linear(config.inter_dim, config.dim, bias=False)
        self._packed_gate_up = None
        self._packed_key = None
        self._packed_down = None
        self._packed_down_key = None
        self._folded = None
        self._folded_key = None

    def packed_gate_up(self, fold_norm: bool = False):
        """gate/up weights in the packed SwiGLU tile layout (lpc_pack_weights),
        with the post-attention norm weight folded in when ``fold_norm``; built
        on first use and rebuilt when a weight changes."""
        from .packed_linear import PackedWeight
        nw = self.post_attention_layernorm.weight
        ws = (self.gate_proj.weight, self.up_proj.weight, nw)
        key = tuple(_weight_key(w) for w in ws) + (fold_norm,)
        if self._packed_gate_up is None or key != self._packed_key:
            self._packed_gate_up = PackedWeight(ws[0], ws[1], layout="swiglu",
                                                norm_weight=nw if fold_norm else None)
            self._packed_key = key
        return self._packed_gate_up

    def packed_down(self):
        """down_proj in the packed linear layout, built on first use."""
        from .packed_linear import PackedWeight
        key = _weight_key(self.down_proj.weight)
        if self._packed_down is None or key != self._packed_down_key:
            self._packed_down = PackedWeight(self.down_proj.weight)
            self._packed_down_key = key
        return self._packed_down

    def folded_gate_up(self):
        """(gate, up) weights with the post-attention norm weight folded in
        (W[n, k] * w[k]) for the one-kernel norm + SwiGLU; the parameters
        themselves when w is all ones.  Built outside stream capture (it reads
        w on the host once per weight version); None while capturing."""
        nw = self.post_attention_layernorm.weight
        ws = (self.gate_proj.weight, self.up_proj.weight, nw)
        key = tuple(_weight_key(w) for w in ws)
        if self._folded is None or key != self._folded_key:
            if torch.cuda.is_current_stream_capturing():
                return None
            with torch.no_grad():
                if bool((nw == 1).all()):
                    self._folded = (ws[0], ws[1])
                else:
                    scale = nw.float().unsqueeze(0)
                    self._folded = tuple((w.float() * scale).to(w.dtype) for w in ws[:2])
                    # the GEMM streams weights before it waits on earlier kernels
                    torch.cuda.current_stream(nw.device).synchronize()
            self._folded_key = key
        return self._folded

    def _mlp_inter(self, h: torch.Tensor, packed_max: int, fuse_norm: bool = False,
                   norm_in_gemm: bool = False) -> torch.Tensor:
        norm = self.post_attention_layernorm
        tokens = h.numel() // h.shape[-1]
        if tokens <= packed_max and _packable(h, self.gate_proj.weight):
            # decode-sized: the weight-streaming GEMM on the packed gate/up with
            # the SiLU*up epilogue; the norm either in its own kernel (faster on
            # B200, see norm_in_gemm) or inside the GEMM on the folded weight
            from .packed_linear import packed_linear
            if norm_in_gemm and tokens <= NORM_IN_GEMM_MAX_TOKENS:
                return packed_linear(h, self.packed_gate_up(True), "swiglu", norm_eps=norm.eps)
            from .ops import rmsnorm_forward
            return packed_linear(rmsnorm_forward(h, norm.weight, norm.eps), self.packed_gate_up(),
                                 "swiglu")
        if (fuse_norm and _packable(h, self.gate_proj.weight)
                and self.gate_proj.weight.shape[0] % 16 == 0):
            folded = self.folded_gate_up()
            if folded is not None:
                # the norm inside the CTA-pair SwiGLU GEMM (statistics from its
                # activation tiles, the row scale in the epilogue)
                from .ops import rmsswiglu_folded_forward
                return rmsswiglu_folded_forward(h, folded[0], folded[1], norm.eps)
        return rmsswiglu_forward(h, rms_weight=norm.weight, gate_w=self.gate_proj.weight,
                                 up_w=self.up_proj.weight, eps=norm.eps)

    def _down(self, inter: torch.Tensor, h: torch.Tensor, ctx: Optional[_StepContext]) -> torch.Tensor:
        """h + inter @ down_proj^T (residual in the GEMM epilogue)."""
        shp = h.shape
        h2 = h.reshape(-1, shp[-1])
        i2 = inter.reshape(-1, inter.shape[-1])
        if (ctx is not None and ctx.decode and i2.shape[0] <= ctx.resid_max
                and _packable(i2, self.down_proj.weight) and h2.is_contiguous()):
            from .packed_linear import packed_linear
            return packed_linear(i2, self.packed_down(), "residual", resid=h2).view(shp)
        return torch.addmm(h2, i2, self.down_proj.weight.t()).view(shp)

    def forward(
        self,
        x: torch.Tensor,
        *,
        positions: torch.Tensor,
        cos: torch.Tensor,
        sin: torch.Tensor,
        kv_cache: Optional[KVCacheManager],
        mask: Optional[torch.Tensor],
        ctx: Optional[_StepContext] = None,
    ) -> torch.Tensor:
        if kv_cache is not None and self.self_attn.fuses_input_norm(x, ctx):
            # the input norm runs inside the fused q/k/v kernel
            attn = self.self_attn(x, positions=positions, cos=cos, sin=sin, kv_cache=kv_cache,
                                  layer_idx=self.layer_idx, mask=mask, ctx=ctx,
                                  input_norm=self.input_layernorm)
        else:
            attn = self.self_attn(self.input_layernorm(x), positions=positions, cos=cos, sin=sin,
                                  kv_cache=kv_cache, layer_idx=self.layer_idx, mask=mask, ctx=ctx)
        h = self.self_attn.project_out(attn, x, ctx)
        mlp_inter = self._mlp_inter(h, ctx.packed_max if ctx is not None and ctx.decode else 0,
                                    ctx.fuse_norm if ctx is not None else False,
                                    ctx.norm_in_gemm if ctx is not None else False)
        return self._down(mlp_inter, h, ctx)


class LlamaModel(nn.Module):
    def __init__(self, config: LlamaModelConfig) -> None:
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.dim)
        self.layers = nn.ModuleList([LlamaDecodeLayer(config, i) for i in range(config.num_layers)])
        self.norm = RMSNorm(config.dim, eps=config.rms_norm_eps)
        cos, sin = precompute_freqs_cis(config.head_dim, config.max_seq_len, theta=config.rope_theta)
        self.register_buffer("cos_cached", cos, persistent=False)
        self.register_buffer("sin_cached", sin, persistent=False)
        # decode steps with at most this many tokens use the packed SwiGLU
        # weights (0 disables the packed copy, e.g. when HBM is tight)
        self.packed_swiglu_max_tokens = PACKED_SWIGLU_MAX_TOKENS
        # decode steps with at most this many tokens use the fused input norm +
        # q/k/v projection + RoPE + KV append on a packed q/k/v copy (0 disables it)
        self.fused_qkv_max_tokens = FUSED_QKV_MAX_TOKENS
        # decode steps with at most this many tokens run o_proj / down_proj
        # with the residual on packed copies (0 disables them)
        self.packed_residual_max_tokens = PACKED_RESIDUAL_MAX_TOKENS
        # True: steps above packed_swiglu_max_tokens run the post-attention
        # norm inside the CTA-pair SwiGLU GEMM (lpc_rmsswiglu_folded_forward,
        # on gate/up with the norm weight folded in; a folded copy is made only
        # when that weight is not all ones).  False (default): the row-norm
        # kernel, then the GEMM, launched under it -- measured 1% faster per
        # decode step at 256 sequences, where the separate norm's early launch
        # trigger lets the GEMM's weight stream start under it.
        self.fuse_mlp_norm = False
        # True (default): decode steps of at most NORM_IN_GEMM_MAX_TOKENS
        # tokens normalise inside the weight-streaming GEMMs (q/k/v + RoPE +
        # append, SwiGLU), norm weights folded into the packed copies: 4.47
        # against 4.52 ms per decode step at 32 sequences.  False: a row-norm
        # kernel before each GEMM.
        self.norm_in_gemm = True

    def reset_rope_tables(self) -> None:
        """Recompute cos/sin (e.g. after materialising a meta-device model)."""
        dev = self.embed_tokens.weight.device
        cos, sin = precompute_freqs_cis(self.config.head_dim, self.config.max_seq_len,
                                        theta=self.config.rope_theta, device=dev)
        dt = self.embed_tokens.weight.dtype
        self.cos_cached = cos.to(dt)
        self.sin_cached = sin.to(dt)

    def forward(
        self,
        input_ids: torch.Tensor,
        *,
        positions: torch.Tensor,
        kv_cache: Optional[KVCacheManager],
        mask: Optional[torch.Tensor],
    ) -> torch.Tensor:
        h = self.embed_tokens(input_ids)
        B, S = input_ids.shape
        ctx = _StepContext()
        ctx.positions = positions
        ctx.packed_max = self.packed_swiglu_max_tokens
        ctx.fused_qkv_max = self.fused_qkv_max_tokens
        ctx.resid_max = self.packed_residual_max_tokens
        ctx.fuse_norm = self.fuse_mlp_norm
        ctx.norm_in_gemm = self.norm_in_gemm
        cos = sin = None
        if kv_cache is not None:
            ctx.cos_table, ctx.sin_table = self.cos_cached, self.sin_cached
            kv_cache.prepare_forward(positions, ctx, self.config.num_heads)
        else:
            cos = self.cos_cached[positions]
            sin = self.sin_cached[positions]
            if cos.ndim == 3:
                cos = cos.unsqueeze(2)
                sin = sin.unsqueeze(2)
        for layer in self.layers:
            h = layer(h, positions=positions, cos=cos, sin=sin, kv_cache=kv_cache, mask=mask,
                      ctx=ctx)
        return self.norm(h)


class LlamaForCausalLM(nn.Module):
    def __init__(self, config: LlamaModelConfig) -> None:
        super().__init__()
        self.config = config
        self.model = LlamaModel(config)
        self.lm_head = nn.Linear(config.dim, config.vocab_size, bias=False)

    def forward(
        self,
        input_ids: torch.Tensor,
        *,
        positions: Optional[torch.Tensor] = None,
        kv_cache: Optional[KVCacheManager] = None,
        mask: Optional[torch.Tensor] = None,
        last_token_only: bool = False,
    ) -> torch.Tensor:
        """Logits [B, S, vocab] (model.py:427-477); [B, 1, vocab] with
        ``last_token_only``.  Without a cache the causal mask is applied by the
        attention kernel itself (the reference builds a -inf triu mask, model.py:451-466)."""
        B, S = input_ids.shape
        if positions is None:
            positions = torch.arange(S, device=input_ids.device).unsqueeze(0).expand(B, -1)
        hidden = self.model(input_ids, positions=positions, kv_cache=kv_cache, mask=mask)
        if last_token_only:
            hidden = hidden[:, -1:, :]
        return self.lm_head(hidden)

    # -- construction helpers ----------------------------------------------
    @classmethod
    def random_init(cls, config: LlamaModelConfig, *, device="cuda", dtype=torch.bfloat16,
                    seed: int = 0, std: float = 0.02) -> "LlamaForCausalLM":
        """Random-init model built directly in device memory: every matrix
        ~N(0, std) drawn from a generator seeded with ``seed`` on ``device``,
        RMSNorm weights 1.0."""
        with torch.device("meta"):
            model = cls(config)
        model = model.to_empty(device=device).to(dtype)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        with torch.no_grad():
            for name, p in model.named_parameters():
                if name.endswith("layernorm.weight") or name == "model.norm.weight":
                    p.fill_(1.0)
                else:
                    p.normal_(0.0, std, generator=gen)
        model.model.reset_rope_tables()
        model.eval()
        return model

    @classmethod
    def from_state_dict(cls, config: LlamaModelConfig, state_dict: Dict[str, torch.Tensor], *,
                        device="cuda", dtype=torch.bfloat16) -> "LlamaForCausalLM":
        with torch.device("meta"):
            model = cls(config)
        model = model.to_empty(device=device).to(dtype)
        missing, unexpected = model.load_state_dict(state_dict, strict=False)
        if missing:
            raise RuntimeError("Missing checkpoint weights:\n" + "\n".join(missing))
        if unexpected:
            raise RuntimeError("Unexpected checkpoint weights:\n" + "\n".join(unexpected))
        model.model.reset_rope_tables()
        model.eval()
        return model

    @classmethod
    def from_pretrained(cls, model_dir: str, *, device: str = "cuda",
                        dtype: torch.dtype = torch.float16) -> "LlamaForCausalLM":
        """Loads config.json + .safetensors/.bin with strict key checks (model.py:479-580)."""
        cfg_file = os.path.join(model_dir, "config.json")
        if not os.path.isfile(cfg_file):
            raise FileNotFoundError(f"Missing config: {cfg_file}")
        config = LlamaModelConfig.from_json(cfg_file)
        files = [os.path.join(model_dir, f) for f in os.listdir(model_dir)
                 if f.endswith((".safetensors", ".bin"))]
        if not files:
            raise FileNotFoundError(f"No checkpoint weights found in {model_dir}")
        sd: Dict[str, torch.Tensor] = {}
        for f in files:
            if f.endswith(".safetensors"):
                from safetensors.torch import load_file
                sd.update(load_file(f, device="cpu"))
            else:
                sd.update(torch.load(f, map_location="cpu", weights_only=True))
        return cls.from_state_dict(config, sd, device=device, dtype=dtype)
