"""Host-side logic that needs no GPU: the model configuration the reference's
users load (config.py:27-179 of the reference), the bench's reference arm and
its JSON contract, and laws of the oracle that the parity tests lean on."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from llama_pure_compute_b200.config import PRESETS, LlamaModelConfig, Precision
from oracle.model_ref import rope_tables
from oracle.ops_ref import attention_ref, decode_attention_ref, kv_append_ref, rmsnorm_ref, rope_ref

REPO = Path(__file__).resolve().parents[1]


# ---------------------------------------------------------------------------
# configuration
# ---------------------------------------------------------------------------
def test_presets_have_the_reference_shapes():
    c = PRESETS["llama-2-7b"]
    assert (c.dim, c.inter_dim, c.num_layers, c.num_heads, c.num_kv_heads, c.head_dim) == \
        (4096, 11008, 32, 32, 32, 128)
    g = PRESETS["llama-3-8b"]
    assert (g.num_kv_heads, g.gqa_group_size, g.rope_theta, g.vocab_size) == (8, 4, 500000.0, 128256)
    big = PRESETS["llama-2-70b"]
    assert (big.dim, big.head_dim, big.gqa_group_size, big.num_layers) == (8192, 128, 8, 80)
    # 7B: 6.74e9 parameters with untied embeddings
    assert abs(c.num_parameters() - 6.738e9) / 6.738e9 < 1e-3


def test_config_checks_and_derived_sizes():
    with pytest.raises(ValueError, match="divisible by num_heads"):
        LlamaModelConfig(dim=100, num_heads=3)
    with pytest.raises(ValueError, match="multiple of num_kv_heads"):
        LlamaModelConfig(num_heads=32, num_kv_heads=5)
    with pytest.raises(ValueError, match="strictly positive"):
        LlamaModelConfig(max_seq_len=0)
    c = LlamaModelConfig(num_kv_heads=8, max_seq_len=1024, max_batch_size=2,
                         precision=Precision.BF16)
    assert c.kv_cache_elements_per_token == 2 * 8 * 128
    assert c.estimate_kv_cache_memory_bytes() == 32 * 2 * 1024 * 2 * 8 * 128 * 2
    assert LlamaModelConfig().num_kv_heads == 32  # defaults to num_heads


def test_from_json_maps_hugging_face_keys(tmp_path):
    hf = {"hidden_size": 2048, "intermediate_size": 5632, "num_hidden_layers": 22,
          "num_attention_heads": 32, "num_key_value_heads": 4, "vocab_size": 32000,
          "rms_norm_eps": 1e-6, "rope_theta": 10000.0, "precision": "BF16",
          "architectures": ["LlamaForCausalLM"]}
    path = tmp_path / "config.json"
    path.write_text(json.dumps(hf))
    c = LlamaModelConfig.from_json(path)
    assert (c.dim, c.inter_dim, c.num_layers, c.num_heads, c.num_kv_heads) == (2048, 5632, 22, 32, 4)
    assert c.head_dim == 64 and c.precision is Precision.BF16 and c.rms_norm_eps == 1e-6
    with pytest.raises(FileNotFoundError):
        LlamaModelConfig.from_json(tmp_path / "missing.json")


# ---------------------------------------------------------------------------
# the bench's reference arm: JSON contract on a bounded CPU sample
# ---------------------------------------------------------------------------
def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--layers", "2", "--cpu-seconds", "2"],
                         cwd=REPO, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["unit"] == "tok/s" and d["steps"] == 1 and d["warmup"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == pytest.approx(d["value"], rel=1e-3)
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]


# ---------------------------------------------------------------------------
# oracle laws used by the parity tests
# ---------------------------------------------------------------------------
def test_rope_tables_rotate_by_position_and_preserve_norm():
    cos, sin = rope_tables(128, 64, 10000.0)
    assert torch.allclose(cos[0], torch.ones(128)) and torch.allclose(sin[0], torch.zeros(128))
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 5, 2, 128, generator=g, dtype=torch.float64).float()
    pos = torch.tensor([[0, 1, 7, 33, 63]])
    hc, hs = cos[:, :64].contiguous(), sin[:, :64].contiguous()  # [max_pos, D/2] rows by position
    qo, _ = rope_ref(q, q[..., :1, :].clone(), hc, hs, pos)
    # a rotation: every (d, d + 64) pair keeps its length
    a = q[..., :64] ** 2 + q[..., 64:] ** 2
    b = qo[..., :64] ** 2 + qo[..., 64:] ** 2
    assert torch.allclose(a, b, rtol=1e-5, atol=1e-5)
    assert torch.equal(qo[:, 0], q[:, 0])  # position 0 is the identity


def test_rmsnorm_oracle_is_scale_invariant():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(4, 256, generator=g)
    w = 1 + 0.1 * torch.randn(256, generator=g)
    y = rmsnorm_ref(x, w, 1e-12)
    assert torch.allclose(rmsnorm_ref(8 * x, w, 1e-12), y, rtol=1e-5, atol=1e-6)
    assert torch.allclose((y / w).pow(2).mean(-1), torch.ones(4), rtol=1e-4)


def test_decode_oracle_equals_last_row_of_causal_attention():
    g = torch.Generator().manual_seed(2)
    B, H, Hkv, L, D = 2, 4, 2, 37, 64
    q = torch.randn(B, H, L, D, generator=g)
    k = torch.randn(B, Hkv, L, D, generator=g)
    v = torch.randn(B, Hkv, L, D, generator=g)
    full = attention_ref(q, k, v, causal=True, sm_scale=D ** -0.5)
    lens = torch.full((B,), L, dtype=torch.int32)
    dec = decode_attention_ref(q[:, :, -1], k, v, lens, D ** -0.5)
    assert torch.allclose(dec, full[:, :, -1], rtol=1e-4, atol=1e-5)


def test_kv_append_oracle_skips_negative_slots_and_is_idempotent():
    import numpy as np
    rng = np.random.default_rng(3)
    T, H, D, Bmax, S = 6, 2, 8, 2, 5
    k = rng.integers(-100, 100, (T, H, D), dtype=np.int16)
    v = rng.integers(-100, 100, (T, H, D), dtype=np.int16)
    slots = np.array([0, -1, 6, 9, -3, 4], dtype=np.int64)
    kc = np.zeros((Bmax, H, S, D), np.int16)
    vc = np.zeros_like(kc)
    kv_append_ref(k, v, kc, vc, slots)
    once = (kc.copy(), vc.copy())
    kv_append_ref(k, v, kc, vc, slots)
    assert np.array_equal(kc, once[0]) and np.array_equal(vc, once[1])
    written = sum(1 for s in slots if s >= 0)
    assert int((np.abs(kc).sum(axis=-1) > 0).sum()) <= written * H
    b, p = divmod(9, S)
    assert np.array_equal(kc[b, :, p], k[3])

