"""Model-level parity: greedy tokens of the bf16 GPU model against the fp32
CPU oracle evaluated from the same (bf16-rounded) weights, teacher-forced on
the GPU's tokens.  A step passes when the GPU token is the oracle's argmax, or
when the oracle's own logit gap between its argmax and the GPU token is below
TIE_TOL (a near-tie that bf16 activations may legitimately flip)."""
import pytest
import torch

from llama_pure_compute_b200 import _lib
from llama_pure_compute_b200.config import LlamaModelConfig
from llama_pure_compute_b200.generate import (BatchedGreedyDecoder, GenerationConfig,
                                              LlamaGenerator)
from llama_pure_compute_b200.kv_manager import KVCacheManager
from llama_pure_compute_b200.model import LlamaForCausalLM
from oracle.model_ref import OracleLlama, make_state_dict

pytestmark = pytest.mark.gpu
DEV = "cuda"
TIE_TOL = 5e-2


@pytest.fixture(autouse=True)
def _clean_status():
    yield
    assert _lib.device_status() == 0


def build(cfgd, seed, dtype=torch.bfloat16):
    cfg = LlamaModelConfig(**cfgd)
    sd = make_state_dict(cfgd, seed)
    model = LlamaForCausalLM.from_state_dict(cfg, sd, device=DEV, dtype=dtype)
    sd_rounded = {k: v.to(dtype).float() for k, v in sd.items()}
    return cfg, model, sd_rounded


def check_against_oracle(cfgd, sd_rounded, prompt, gpu_tokens):
    orc = OracleLlama(cfgd, sd_rounded, cfgd["max_seq_len"], table_dtype=torch.bfloat16)
    mine, gap, margin = orc.greedy(prompt.cpu(), gpu_tokens.shape[1], forced=gpu_tokens.cpu())
    agree = mine == gpu_tokens.cpu()
    assert bool((agree | (gap <= TIE_TOL)).all()), (mine, gpu_tokens, gap)
    return agree.float().mean().item()


@pytest.mark.parametrize("name", ["mha", "gqa"])
def test_greedy_tokens_match_oracle(golden, name):
    g = golden("model")[name]
    cfgd = g["cfg"]
    cfg, model, sdr = build(cfgd, g["seed"])
    B, P = g["prompt"].shape
    steps = g["tokens"].shape[1]
    kv = KVCacheManager(num_layers=cfg.num_layers, max_batch_size=B, max_seq_len=cfg.max_seq_len,
                        n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, dtype=torch.bfloat16,
                        device=DEV)
    dec = BatchedGreedyDecoder(model, kv, B, use_cuda_graph=True)
    toks = dec.generate(g["prompt"].to(DEV), steps)
    check_against_oracle(cfgd, sdr, g["prompt"], toks)
    dec.release()


def test_graph_equals_eager_and_generator(golden):
    g = golden("model")["mha"]
    cfgd = g["cfg"]
    cfg, model, _ = build(cfgd, g["seed"])
    outs = []
    for graph in (True, False):
        kv = KVCacheManager(num_layers=cfg.num_layers, max_batch_size=2, max_seq_len=cfg.max_seq_len,
                            n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                            dtype=torch.bfloat16, device=DEV)
        dec = BatchedGreedyDecoder(model, kv, 2, use_cuda_graph=graph)
        outs.append(dec.generate(g["prompt"].to(DEV), 12).cpu())
        dec.release()
    assert torch.equal(outs[0], outs[1])
    gen = LlamaGenerator(model, cfg)
    one = list(gen.generate(g["prompt"][0].tolist(), generation=GenerationConfig(max_new_tokens=12)))
    assert one == outs[0][0].tolist()


def test_ragged_prompts_match_single_sequence_runs():
    cfgd = dict(vocab_size=320, dim=256, inter_dim=512, num_layers=2, num_heads=2, num_kv_heads=2,
                max_seq_len=96, rms_norm_eps=1e-5, rope_theta=10000.0)
    cfg, model, sdr = build(cfgd, 77)
    gen = torch.Generator().manual_seed(3)
    lens = [5, 17, 17, 40]
    prompts = [torch.randint(0, 320, (n,), generator=gen).tolist() for n in lens]
    kv = KVCacheManager(num_layers=2, max_batch_size=4, max_seq_len=96, n_kv_heads=2, head_dim=128,
                        dtype=torch.bfloat16, device=DEV)
    dec = BatchedGreedyDecoder(model, kv, 4, use_cuda_graph=True)
    toks = dec.generate(prompts, 16).cpu()
    dec.release()
    for i, p in enumerate(prompts):
        kv1 = KVCacheManager(num_layers=2, max_batch_size=1, max_seq_len=96, n_kv_heads=2,
                             head_dim=128, dtype=torch.bfloat16, device=DEV)
        d1 = BatchedGreedyDecoder(model, kv1, 1, use_cuda_graph=False)
        t1 = d1.generate([p], 16).cpu()
        assert torch.equal(t1[0], toks[i]), i
        check_against_oracle(cfgd, sdr, torch.tensor([p]), t1)


def test_full_forward_matches_cached_decode():
    cfgd = dict(vocab_size=256, dim=256, inter_dim=512, num_layers=2, num_heads=2, num_kv_heads=1,
                max_seq_len=64, rms_norm_eps=1e-5, rope_theta=10000.0)
    cfg, model, _ = build(cfgd, 5)
    ids = torch.randint(0, 256, (2, 20), generator=torch.Generator().manual_seed(1)).to(DEV)
    full = model(ids)  # no cache: tcgen05 causal flash attention over the whole prompt
    kv = KVCacheManager(num_layers=2, max_batch_size=2, max_seq_len=64, n_kv_heads=1, head_dim=128,
                        dtype=torch.bfloat16, device=DEV)
    kv.begin_request(2)
    pos = torch.arange(19, device=DEV).unsqueeze(0).expand(2, -1)
    model(ids[:, :19], positions=pos, kv_cache=kv, last_token_only=True)
    last = model(ids[:, 19:], positions=torch.full((2, 1), 19, device=DEV), kv_cache=kv)
    assert (last[:, 0].float() - full[:, -1].float()).abs().max().item() < 0.05
    assert kv.current_seq_len(0) == 20


def test_kv_manager_reference_update_api():
    kv = KVCacheManager(num_layers=2, max_batch_size=4, max_seq_len=32, n_kv_heads=2, head_dim=64,
                        dtype=torch.float16, device=DEV)
    k = torch.randn(3, 2, 16, 64, device=DEV, dtype=torch.float16)
    v = torch.randn_like(k)
    ko, vo = kv.update(layer_idx=1, key_states=k, value_states=v, start_pos=0)
    assert ko.shape == (3, 2, 16, 64) and torch.equal(ko, k) and torch.equal(vo, v)
    k1 = torch.randn(3, 2, 1, 64, device=DEV, dtype=torch.float16)
    ko, _ = kv.update(layer_idx=1, key_states=k1, value_states=k1, start_pos=16)
    assert ko.shape[-2] == 17 and torch.equal(kv.k_cache[1][:3, :, 16:17], k1)
    assert kv.current_seq_len(2) == 17
    with pytest.raises(ValueError, match="overflow"):
        kv.update(layer_idx=0, key_states=k, value_states=v, start_pos=20)
    with pytest.raises(IndexError):
        kv.update(layer_idx=2, key_states=k, value_states=v, start_pos=0)
