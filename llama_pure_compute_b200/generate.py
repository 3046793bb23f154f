"""Generation drivers: the reference's batch-1 generator and a batched greedy
decoder with on-device argmax and CUDA-graph capture of the decode step.

``GenerationConfig``, ``apply_repetition_penalty``, ``sample_next_token`` and
``LlamaGenerator.generate`` keep the behaviour of
src/llama_pure_compute/generate.py:13-333 (greedy = argmax at temperature 0).

``BatchedGreedyDecoder`` is the batched serving loop of the 7B decode
workload: ragged prompts are prefilled into their own cache rows, then every
decode step is one graph replay (embedding -> 32 layers -> norm -> lm_head of
the last position -> argmax) with no host synchronisation inside the step.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Generator, List, Optional, Sequence, Union

import torch
import torch.nn.functional as F

from .config import LlamaModelConfig
from .kv_manager import KVCacheManager
from .ragged_cache import RaggedKVCache

__all__ = ["GenerationConfig", "apply_repetition_penalty", "sample_next_token", "LlamaGenerator",
           "BatchedGreedyDecoder"]


@dataclass(frozen=True)
class GenerationConfig:
    max_new_tokens: int = 128
    temperature: float = 0.0
    top_k: int = 50
    top_p: float = 0.9
    repetition_penalty: float = 1.0
    eos_token_ids: tuple = ()


def apply_repetition_penalty(logits: torch.Tensor, history: torch.Tensor, penalty: float) -> torch.Tensor:
    """generate.py:23-55."""
    if penalty <= 0:
        raise ValueError("repetition_penalty must be > 0")
    if penalty == 1.0 or history.numel() == 0:
        return logits
    scores = torch.gather(logits, -1, history)
    scores = torch.where(scores < 0, scores * penalty, scores / penalty)
    logits.scatter_(-1, history, scores)
    return logits


def sample_next_token(logits: torch.Tensor, *, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    """generate.py:58-153: argmax at temperature 0, else top-k / top-p sampling."""
    if temperature < 0:
        raise ValueError("temperature must be >= 0")
    if temperature == 0:
        return torch.argmax(logits, dim=-1, keepdim=True)
    logits = logits / temperature
    if top_k > 0:
        k = min(top_k, logits.shape[-1])
        thr = torch.topk(logits, k, dim=-1).values[..., -1, None]
        logits = logits.masked_fill(logits < thr, float("-inf"))
    if not 0 < top_p <= 1:
        raise ValueError("top_p must be in (0, 1]")
    if top_p < 1.0:
        sl, si = torch.sort(logits, descending=True, dim=-1)
        cum = torch.cumsum(F.softmax(sl, dim=-1), dim=-1)
        remove = cum > top_p
        remove[..., 1:] = remove[..., :-1].clone()
        remove[..., 0] = False
        orig = torch.zeros_like(remove)
        orig.scatter_(-1, si, remove)
        logits = logits.masked_fill(orig, float("-inf"))
    return torch.multinomial(F.softmax(logits, dim=-1), num_samples=1)


class _RowView:
    """Cache rows [start, start+count) of a KVCacheManager, same interface."""

    def __init__(self, base: KVCacheManager, start: int, count: int):
        self.base = base
        self.k_cache = [t[start:start + count] for t in base.k_cache]
        self.v_cache = [t[start:start + count] for t in base.v_cache]
        self.seq_lens = base.seq_lens[start:start + count]
        self.max_seq_len = base.max_seq_len
        self.max_batch_size = count
        self.n_kv_heads = base.n_kv_heads
        self.head_dim = base.head_dim
        self.num_layers = base.num_layers

    def append_qkv(self, **kw):
        return KVCacheManager.append_qkv(self, **kw)  # type: ignore[arg-type]

    def set_seq_lens(self, positions):
        return KVCacheManager.set_seq_lens(self, positions)  # type: ignore[arg-type]

    def decode_workspace(self, batch, num_heads):
        return KVCacheManager.decode_workspace(self, batch, num_heads)  # type: ignore[arg-type]

    def prepare_forward(self, positions, ctx, num_heads):
        return KVCacheManager.prepare_forward(self, positions, ctx, num_heads)  # type: ignore[arg-type]

    def attend(self, **kw):
        return KVCacheManager.attend(self, **kw)  # type: ignore[arg-type]

    def _check_layer(self, layer_idx: int) -> None:
        if not 0 <= layer_idx < self.num_layers:
            raise IndexError(f"layer_idx={layer_idx} outside [0, {self.num_layers})")


class LlamaGenerator:
    """Batch-1 streaming generator (generate.py:156-333)."""

    def __init__(self, model: torch.nn.Module, config: LlamaModelConfig) -> None:
        self.model = model
        self.config = config
        p = next(model.parameters())
        self.device = p.device
        self.kv_cache = KVCacheManager(num_layers=config.num_layers, max_batch_size=1,
                                       max_seq_len=config.max_seq_len, n_kv_heads=config.num_kv_heads,
                                       head_dim=config.head_dim, dtype=p.dtype, device=self.device)

    def reset(self) -> None:
        self.kv_cache.reset()

    @torch.inference_mode()
    def generate(self, prompt_tokens: Sequence[int], *, generation: GenerationConfig) -> Generator[int, None, None]:
        if not prompt_tokens:
            raise ValueError("prompt_tokens must not be empty")
        P = len(prompt_tokens)
        if P + generation.max_new_tokens > self.config.max_seq_len:
            raise ValueError("Requested generation exceeds configured max_seq_len.")
        self.model.eval()
        self.reset()
        self.kv_cache.begin_request(batch_size=1)
        prompt = torch.tensor([list(prompt_tokens)], dtype=torch.long, device=self.device)
        cap = P + generation.max_new_tokens
        history = torch.empty((1, cap), dtype=torch.long, device=self.device)
        history[:, :P] = prompt
        positions = torch.arange(P, device=self.device, dtype=torch.long).unsqueeze(0)
        logits = self.model(prompt, positions=positions, kv_cache=self.kv_cache, last_token_only=True)
        nl = apply_repetition_penalty(logits[:, -1, :], history[:, :P], generation.repetition_penalty)
        tok = sample_next_token(nl, temperature=generation.temperature, top_k=generation.top_k,
                                top_p=generation.top_p)
        history[:, P] = tok
        hl = P + 1
        tid = int(tok.item())
        yield tid
        if tid in generation.eos_token_ids:
            return
        for pos in range(P, cap - 1):
            pid = torch.tensor([[pos]], dtype=torch.long, device=self.device)
            logits = self.model(tok, positions=pid, kv_cache=self.kv_cache, last_token_only=True)
            nl = apply_repetition_penalty(logits[:, -1, :], history[:, :hl], generation.repetition_penalty)
            tok = sample_next_token(nl, temperature=generation.temperature, top_k=generation.top_k,
                                    top_p=generation.top_p)
            history[:, hl] = tok
            hl += 1
            tid = int(tok.item())
            yield tid
            if tid in generation.eos_token_ids:
                return


class BatchedGreedyDecoder:
    """Greedy decoding of a (possibly ragged) batch, one graph replay per step.

    Sequence i lives in cache row i.  ``prefill`` writes every prompt (equal
    lengths in one forward, ragged ones group by group) and returns the first
    generated tokens; ``step`` advances every sequence by one token.
    """

    def __init__(self, model: torch.nn.Module, kv_cache: Union[KVCacheManager, RaggedKVCache],
                 batch_size: int, use_cuda_graph: bool = True, prefill_chunk: int = 16) -> None:
        self.ragged = isinstance(kv_cache, RaggedKVCache)
        cap = kv_cache.num_sequences if self.ragged else kv_cache.max_batch_size
        if batch_size > cap:
            raise ValueError("batch_size exceeds the cache's capacity")
        self.model = model
        self.kv = kv_cache
        self.B = batch_size
        self.device = kv_cache.device
        self.use_graph = use_cuda_graph
        self.prefill_chunk = prefill_chunk
        self.tokens = torch.zeros(batch_size, 1, dtype=torch.long, device=self.device)
        self.positions = torch.zeros(batch_size, 1, dtype=torch.long, device=self.device)
        self.next_tokens = torch.zeros(batch_size, dtype=torch.long, device=self.device)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    # -- prefill -------------------------------------------------------------
    @torch.inference_mode()
    def prefill(self, prompts: Union[torch.Tensor, List[List[int]]]) -> torch.Tensor:
        """Returns the first generated token of each sequence (device, [B])."""
        if not self.ragged:
            self.kv.begin_request(self.B)
        if isinstance(prompts, torch.Tensor):
            rows = [prompts[i] for i in range(prompts.shape[0])]
        else:
            rows = [torch.tensor(p, dtype=torch.long) for p in prompts]
        if len(rows) != self.B:
            raise ValueError("one prompt per sequence is required")
        lens = [int(r.numel()) for r in rows]
        caps = self.kv.capacities[:self.B] if self.ragged else [self.kv.max_seq_len] * self.B
        if any(n >= c for n, c in zip(lens, caps)):
            raise ValueError("prompt does not fit the cache")
        first = torch.empty(self.B, dtype=torch.long, device=self.device)
        i = 0
        while i < self.B:  # group consecutive equal-length prompts
            j = i
            while j < self.B and j - i < self.prefill_chunk and lens[j] == lens[i]:
                j += 1
            ids = torch.stack([r.to(self.device) for r in rows[i:j]])
            P = lens[i]
            pos = torch.arange(P, device=self.device, dtype=torch.long).unsqueeze(0).expand(j - i, -1)
            if self.ragged:
                self.kv.select(range(i, j))
                view = self.kv
            else:
                view = _RowView(self.kv, i, j - i)
            logits = self.model(ids, positions=pos, kv_cache=view, last_token_only=True)
            first[i:j] = torch.argmax(logits[:, -1, :], dim=-1)
            i = j
        if self.ragged:
            self.kv.select(range(self.B))  # decode steps run on every sequence
        self.positions[:, 0] = torch.tensor(lens, dtype=torch.long, device=self.device)
        self.tokens[:, 0] = first
        return first

    # -- decode --------------------------------------------------------------
    def _step_body(self) -> None:
        logits = self.model(self.tokens, positions=self.positions, kv_cache=self.kv,
                            last_token_only=True)
        nxt = torch.argmax(logits[:, -1, :], dim=-1)
        self.next_tokens.copy_(nxt)
        self.tokens[:, 0].copy_(nxt)
        self.positions.add_(1)

    @torch.inference_mode()
    def capture(self) -> None:
        """Warm up once (sets kernel attributes, builds fused weights) and
        capture the decode step in a CUDA graph.  The warm-up step's effect
        on the state is undone (tokens/positions restored)."""
        tok0 = self.tokens.clone()
        pos0 = self.positions.clone()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self._step_body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.tokens.copy_(tok0)
        self.positions.copy_(pos0)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._step_body()
        self.graph = g
        self.tokens.copy_(tok0)
        self.positions.copy_(pos0)
        torch.cuda.synchronize(self.device)

    @torch.inference_mode()
    def step(self) -> torch.Tensor:
        """Advance every sequence by one greedy token; returns the tokens (device)."""
        if self.use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            self._step_body()
        return self.next_tokens

    @torch.inference_mode()
    def generate(self, prompts, max_new_tokens: int) -> torch.Tensor:
        """Prefill + greedy decode; returns [B, max_new_tokens] generated ids (device)."""
        out = torch.empty(self.B, max_new_tokens, dtype=torch.long, device=self.device)
        out[:, 0] = self.prefill(prompts)
        if max_new_tokens > 1 and self.use_graph and self.graph is None:
            self.capture()
        for t in range(1, max_new_tokens):
            out[:, t] = self.step()
        return out

    def release(self) -> None:
        self.graph = None
