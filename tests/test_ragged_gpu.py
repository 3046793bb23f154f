"""Ragged KV layout (caches [Hkv, total_rows, D], sequence b at rows
seq_base[b] ..): kernels against the dense layout and the oracle, bounds
flags, and the model on a RaggedKVCache against dense single-sequence runs.

Bars: cache writes bit-exact; attention bit-identical to the dense kernel on
the same data (only the addressing differs) and within 2e-2 max-abs of the
fp32 oracle; greedy tokens identical to single-sequence dense-cache runs."""
import pytest
import torch

from llama_pure_compute_b200 import _lib, ops
from llama_pure_compute_b200.config import LlamaModelConfig
from llama_pure_compute_b200.generate import BatchedGreedyDecoder
from llama_pure_compute_b200.kv_manager import KVCacheManager
from llama_pure_compute_b200.model import LlamaForCausalLM, precompute_freqs_cis
from llama_pure_compute_b200.ragged_cache import RaggedKVCache
from oracle.model_ref import make_state_dict
from oracle.ops_ref import decode_attention_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _clean_status():
    yield
    assert _lib.device_status() == 0, "a kernel flagged a device-side error"


def ragged_index(caps):
    base, acc = [], 0
    for c in caps:
        base.append(acc)
        acc += c
    return (torch.tensor(base, dtype=torch.int64, device=DEV),
            torch.tensor(caps, dtype=torch.int32, device=DEV), acc, base)


def dense_to_ragged(dense, caps, base, total):
    """[B, Hkv, Smax, D] -> [Hkv, total, D] with sequence b's first caps[b] rows."""
    B, Hkv, Smax, D = dense.shape
    out = torch.zeros(Hkv, total, D, dtype=dense.dtype, device=dense.device)
    for b in range(B):
        out[:, base[b]:base[b] + caps[b]] = dense[b, :, :caps[b]]
    return out


@pytest.mark.parametrize("H,Hkv", [(8, 8), (8, 2)])
def test_rope_kv_append_ragged_bit_exact_vs_dense(H, Hkv):
    g = torch.Generator(device=DEV).manual_seed(H + Hkv)
    D, B, S = 128, 4, 3
    caps = [40, 7, 100, 33]
    Smax = max(caps)
    seq_base, seq_cap, total, base = ragged_index(caps)
    qkv = torch.randn(B, S, (H + 2 * Hkv) * D, device=DEV, generator=g).to(torch.bfloat16)
    pos = torch.tensor([[0, 1, 2], [4, 5, 6], [97, 98, 99], [10, 11, 12]], device=DEV)
    cos, sin = precompute_freqs_cis(D, 256, device=DEV)
    cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
    kd = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    vd = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    kr = dense_to_ragged(kd, caps, base, total)
    vr = dense_to_ragged(vd, caps, base, total)
    q_dense = ops.rope_kv_append(qkv, pos, cos, sin, kd, vd, H, Hkv)
    q_rag = ops.rope_kv_append_ragged(qkv, pos, cos, sin, kr, vr, seq_base, seq_cap, H, Hkv)
    assert torch.equal(q_dense, q_rag)
    assert torch.equal(dense_to_ragged(kd, caps, base, total), kr)
    assert torch.equal(dense_to_ragged(vd, caps, base, total), vr)


@pytest.mark.parametrize("G", [1, 4])
def test_decode_attention_ragged_matches_dense_and_oracle(G):
    g = torch.Generator(device=DEV).manual_seed(G)
    D, Hkv = 128, 4
    H = Hkv * G
    caps = [300, 1, 1030, 64, 513]
    lens = [257, 1, 1030, 0, 500]
    B, Smax = len(caps), max(caps)
    seq_base, seq_cap, total, base = ragged_index(caps)
    kd = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    vd = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    kr = dense_to_ragged(kd, caps, base, total)
    vr = dense_to_ragged(vd, caps, base, total)
    q = torch.randn(B, H, D, device=DEV, generator=g).to(torch.bfloat16)
    L = torch.tensor(lens, dtype=torch.int32, device=DEV)
    o_dense = ops.decode_attention(q, kd, vd, L)
    o_rag = ops.decode_attention_ragged(q, kr, vr, L, seq_base, seq_cap, Smax)
    assert torch.equal(o_dense, o_rag)
    ref = decode_attention_ref(q.float().cpu(), kd.float().cpu(), vd.float().cpu(), L.cpu())
    assert (o_rag.float().cpu() - ref).abs().max().item() < 2e-2


def test_decode_attention_ragged_one_split_matches_dense():
    """64 sequences x 32 KV heads: both layouts take one 1024-key split per
    sequence and KV head and launch no combine kernel; outputs bit-identical,
    an empty context gives zeros."""
    g = torch.Generator(device=DEV).manual_seed(11)
    D, Hkv, B = 128, 32, 64
    caps = [1000 - 7 * (b % 9) for b in range(B)]
    lens = [c - (b % 5) * 100 for b, c in enumerate(caps)]
    lens[3] = 0
    Smax = max(caps)
    seq_base, seq_cap, total, base = ragged_index(caps)
    assert _lib.decode_kernels(B, Hkv, Smax) == 1 and _lib.decode_kernels(B, Hkv, Smax, total) == 1
    kd = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    vd = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    kr = dense_to_ragged(kd, caps, base, total)
    vr = dense_to_ragged(vd, caps, base, total)
    q = torch.randn(B, Hkv, D, device=DEV, generator=g).to(torch.bfloat16)
    L = torch.tensor(lens, dtype=torch.int32, device=DEV)
    o_dense = ops.decode_attention(q, kd, vd, L)
    o_rag = ops.decode_attention_ragged(q, kr, vr, L, seq_base, seq_cap, Smax)
    assert torch.equal(o_dense, o_rag)
    assert o_rag[3].abs().sum().item() == 0
    sel = [0, 3, 17, 63]
    ref = decode_attention_ref(q[sel].float().cpu(), kd[sel].float().cpu(), vd[sel].float().cpu(),
                               L[sel].cpu())
    assert (o_rag[sel].float().cpu() - ref).abs().max().item() < 2e-2


def test_ragged_out_of_range_rows_are_flagged_not_read():
    D, Hkv, H = 128, 2, 2
    caps = [64, 64]
    seq_base, seq_cap, total, _ = ragged_index(caps)
    kr = torch.randn(Hkv, total, D, device=DEV).to(torch.bfloat16)
    vr = torch.randn(Hkv, total, D, device=DEV).to(torch.bfloat16)
    q = torch.randn(2, H, D, device=DEV).to(torch.bfloat16)
    bad_base = torch.tensor([0, total - 10], dtype=torch.int64, device=DEV)  # 2nd runs past the end
    L = torch.tensor([64, 64], dtype=torch.int32, device=DEV)
    out = ops.decode_attention_ragged(q, kr, vr, L, bad_base, seq_cap, 64)
    assert _lib.device_status() != 0
    assert torch.all(out[1] == 0)
    # a length past the capacity is clamped to it and flagged
    L2 = torch.tensor([80, 10], dtype=torch.int32, device=DEV)
    out2 = ops.decode_attention_ragged(q, kr, vr, L2, seq_base, seq_cap, 64)
    assert _lib.device_status() != 0
    ref = ops.decode_attention_ragged(q, kr, vr, torch.tensor([64, 10], dtype=torch.int32,
                                                              device=DEV), seq_base, seq_cap, 64)
    assert torch.equal(out2, ref)


def _model(seed=21):
    cfgd = dict(vocab_size=320, dim=256, inter_dim=512, num_layers=2, num_heads=2, num_kv_heads=1,
                max_seq_len=160, rms_norm_eps=1e-5, rope_theta=10000.0)
    cfg = LlamaModelConfig(**cfgd)
    model = LlamaForCausalLM.from_state_dict(cfg, make_state_dict(cfgd, seed), device=DEV,
                                             dtype=torch.bfloat16)
    return cfg, model


@pytest.mark.parametrize("graph", [True, False])
def test_model_on_ragged_cache_matches_dense_single_runs(graph):
    cfg, model = _model()
    gen = torch.Generator().manual_seed(9)
    lens = [7, 64, 33, 120, 33]
    new = 12
    prompts = [torch.randint(0, 320, (n,), generator=gen).tolist() for n in lens]
    cache = RaggedKVCache(num_layers=cfg.num_layers, capacities=[n + new for n in lens],
                          n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                          dtype=torch.bfloat16, device=DEV)
    assert cache.total_rows == sum(lens) + new * len(lens)
    dec = BatchedGreedyDecoder(model, cache, len(lens), use_cuda_graph=graph)
    toks = dec.generate(prompts, new).cpu()
    dec.release()
    for i, p in enumerate(prompts):
        kv1 = KVCacheManager(num_layers=cfg.num_layers, max_batch_size=1, max_seq_len=160,
                             n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                             dtype=torch.bfloat16, device=DEV)
        d1 = BatchedGreedyDecoder(model, kv1, 1, use_cuda_graph=False)
        t1 = d1.generate([p], new).cpu()
        assert torch.equal(t1[0], toks[i]), i


def test_ragged_cache_capacity_checks():
    cfg, model = _model()
    cache = RaggedKVCache(num_layers=cfg.num_layers, capacities=[10, 20],
                          n_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, device=DEV)
    dec = BatchedGreedyDecoder(model, cache, 2, use_cuda_graph=False)
    with pytest.raises(ValueError):
        dec.prefill([[1] * 10, [2] * 5])  # the first prompt fills its whole capacity
    with pytest.raises(ValueError):
        cache.select([0, 2])
    with pytest.raises(ValueError):
        RaggedKVCache(num_layers=1, capacities=[4, 0], n_kv_heads=1, head_dim=128, device=DEV)
