"""Greedy-token parity on the path the 7B decode benchmark times.

Workload: the Llama-2-7B shape (32 layers, 4096, 32x128 heads, FFN 11008,
vocab 32000), random-init bf16 weights ~N(0, 0.02) drawn on the GPU with seed
3, RMSNorm weights 1.0; 256 prompts of 512 tokens drawn uniformly over the
vocabulary from a CPU generator seeded with 3 -- the one-GPU share of the
decode benchmark.  At 256 sequences per step the decode step runs the CTA-pair
SwiGLU kernel (more than 128 tokens), the stacked q/k/v GEMM followed by the
fused RoPE + KV append kernel, and split-KV decode attention; the prefill runs
16 prompts (8192 tokens) per forward through the tcgen05 prefill attention.

32 greedy steps are generated on the GPU (prefill + CUDA-graph decode), then
replayed eagerly on the same batch to read the logits of eight of the 256
sequences (the eager step must pick the graph's tokens).  The eight sequences
are evaluated teacher-forced on the GPU's tokens by

  * the fp32 oracle (on the GPU in fp32, TF32 off, from the same bf16
    weights), the ground truth, and
  * a plain bf16 evaluation of the same graph (torch ops, one rounding per
    op, cuBLAS GEMMs): what any bf16 implementation of the reference's model
    deviates from the fp32 truth by.

Reported: identical steps against the oracle, and the oracle's gap and top-2
margin at every flip, for both bf16 evaluations.  Asserted: the GPU's logits
are no further from the fp32 oracle than the plain bf16 evaluation's (mean
and max |logit - oracle| within BF16_SLACK of it), and the GPU flips no more
steps than the plain bf16 evaluation does (plus FLIP_SLACK).
"""
import pytest
import torch

from llama_pure_compute_b200 import _lib
from llama_pure_compute_b200.config import PRESETS, LlamaModelConfig
from llama_pure_compute_b200.generate import BatchedGreedyDecoder, _RowView
from llama_pure_compute_b200.kv_manager import KVCacheManager
from llama_pure_compute_b200.model import LlamaForCausalLM
from oracle.model_ref import OracleLlama

pytestmark = pytest.mark.gpu
DEV = "cuda"
BATCH, PROMPT, STEPS = 256, 512, 32
CHECKED = [0, 36, 73, 109, 146, 182, 219, 255]
BF16_SLACK = 1.1
FLIP_SLACK = 4


def _teacher_forced_logits(orc, prompt, forced):
    """[B, steps, V] logits of `orc` for prompt [B, P] then the forced tokens."""
    B, P = prompt.shape
    cache = [None] * orc.L
    out = [orc.forward(prompt, torch.arange(P, device=prompt.device)[None].expand(B, -1),
                       cache)[:, -1].float()]
    for t in range(forced.shape[1] - 1):
        pos = torch.full((B, 1), P + t, device=prompt.device, dtype=torch.long)
        out.append(orc.forward(forced[:, t:t + 1], pos, cache)[:, -1].float())
    return torch.stack(out, 1)


def _flips(logits, oracle, toks, names):
    mine = oracle.argmax(-1)
    top2 = torch.topk(oracle, 2, dim=-1).values
    gap = top2[..., 0] - oracle.gather(-1, toks[..., None])[..., 0]
    margin = top2[..., 0] - top2[..., 1]
    agree = mine == toks
    return agree, [(names[b], t, round(float(gap[b, t]), 4), round(float(margin[b, t]), 4))
                   for b, t in (~agree).nonzero().tolist()]


@torch.no_grad()
def test_decode_config_greedy_tokens_match_oracle():
    base = PRESETS["llama-2-7b"]
    max_seq = PROMPT + STEPS
    cfg = LlamaModelConfig(vocab_size=base.vocab_size, dim=base.dim, inter_dim=base.inter_dim,
                           num_layers=base.num_layers, num_heads=base.num_heads,
                           num_kv_heads=base.num_kv_heads, max_seq_len=max_seq,
                           rms_norm_eps=1e-5, rope_theta=10000.0)
    model = LlamaForCausalLM.random_init(cfg, device=DEV, dtype=torch.bfloat16, seed=3)
    prompts = torch.randint(0, 32000, (BATCH, PROMPT), generator=torch.Generator().manual_seed(3))
    kv = KVCacheManager(num_layers=cfg.num_layers, max_batch_size=BATCH, max_seq_len=max_seq,
                        n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, dtype=torch.bfloat16,
                        device=DEV)
    dec = BatchedGreedyDecoder(model, kv, BATCH, use_cuda_graph=True)
    toks = dec.generate(prompts.to(DEV), STEPS)
    dec.release()
    # the same steps eagerly, teacher-forced on the graph's tokens, keeping the
    # logits of the checked sequences
    sel = torch.tensor(CHECKED, device=DEV)
    kv.begin_request(BATCH)
    P = PROMPT
    first = []
    for i in range(0, BATCH, 16):  # the decoder's prefill groups: 16 prompts per forward
        pos = torch.arange(P, device=DEV)[None].expand(16, -1)
        first.append(model(prompts[i:i + 16].to(DEV), positions=pos, kv_cache=_RowView(kv, i, 16),
                           last_token_only=True)[:, -1])
    lg = torch.cat(first)
    assert torch.equal(lg.argmax(-1), toks[:, 0])
    gl = [lg[sel].float()]
    for t in range(STEPS - 1):
        lg = model(toks[:, t:t + 1], positions=torch.full((BATCH, 1), P + t, device=DEV),
                   kv_cache=kv, last_token_only=True)[:, -1]
        assert torch.equal(lg.argmax(-1), toks[:, t + 1]), t
        gl.append(lg[sel].float())
    gpu_logits = torch.stack(gl, 1)
    assert _lib.device_status() == 0
    sd = {k: v.detach().float() for k, v in model.state_dict().items()}
    del model, kv, dec
    torch.cuda.empty_cache()

    cfgd = dict(vocab_size=32000, dim=4096, inter_dim=11008, num_layers=32, num_heads=32,
                num_kv_heads=32, rms_norm_eps=1e-5, rope_theta=10000.0, max_seq_len=max_seq)
    forced = toks[sel]
    ps = prompts[sel.cpu()].to(DEV)
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        orc = OracleLlama(cfgd, sd, max_seq, table_dtype=torch.bfloat16, device=DEV)
        oracle = _teacher_forced_logits(orc, ps, forced)
        del orc
        torch.cuda.empty_cache()
        t16 = OracleLlama(cfgd, sd, max_seq, table_dtype=torch.bfloat16, dtype=torch.bfloat16,
                          device=DEV)
        del sd
        plain = _teacher_forced_logits(t16, ps, forced)
        del t16
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    torch.cuda.empty_cache()
    ours_agree, ours_flips = _flips(gpu_logits, oracle, forced, CHECKED)
    plain_agree, plain_flips = _flips(plain, oracle, plain.argmax(-1), CHECKED)
    dev_ours = (gpu_logits - oracle).abs()
    dev_plain = (plain - oracle).abs()
    print(f"\ndecode-config greedy parity (8 sequences x {STEPS} steps against the fp32 oracle):\n"
          f"  this build: {int(ours_agree.sum())}/{ours_agree.numel()} steps identical; "
          f"|logit - oracle| mean {dev_ours.mean().item():.4f} max {dev_ours.max().item():.4f}; "
          f"flips (sequence, step, oracle gap, oracle top-2 margin): {ours_flips}\n"
          f"  plain bf16 evaluation: {int(plain_agree.sum())}/{plain_agree.numel()} identical; "
          f"|logit - oracle| mean {dev_plain.mean().item():.4f} max {dev_plain.max().item():.4f}; "
          f"flips: {plain_flips}")
    assert dev_ours.mean().item() <= BF16_SLACK * dev_plain.mean().item()
    assert dev_ours.max().item() <= BF16_SLACK * dev_plain.max().item()
    assert len(ours_flips) <= len(plain_flips) + FLIP_SLACK
