"""Pins the CPU oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import torch

from oracle.model_ref import OracleLlama, make_state_dict
from oracle.ops_ref import (attention_ref, kv_append_ref, rmsnorm_ref, rmsswiglu_ref, rope_ref,
                            rope_kv_append_ref)


def test_rope_fp32_bit_exact(golden):
    g = golden("rope")["model_f32"]
    qo, ko = rope_ref(g["q"], g["k"], g["cos"], g["sin"], g["pos"])
    assert torch.equal(qo, g["q_out"]) and torch.equal(ko, g["k_out"])


def test_rope_half_precision_single_rounding(golden):
    # reference fallback rounds after each op in bf16/fp16; the oracle (like
    # the reference CUDA kernel, rope.cu:39-45) rounds once: <= 1 ulp apart.
    for name, tol in (("model_bf16", 1.5e-2), ("model_f16", 1e-3)):
        g = golden("rope")[name]
        qo, ko = rope_ref(g["q"], g["k"], g["cos"], g["sin"], g["pos"])
        torch.testing.assert_close(qo.float(), g["q_out"].float(), rtol=tol, atol=tol)
        torch.testing.assert_close(ko.float(), g["k_out"].float(), rtol=tol, atol=tol)


def test_rope_half_table_convention(golden):
    g = golden("rope")["half_f32"]
    qo, ko = rope_ref(g["q"], g["k"], g["cos"], g["sin"], g["pos"])
    torch.testing.assert_close(qo, g["q_out"], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(ko, g["k_out"], rtol=1e-6, atol=1e-6)


def test_rmsnorm(golden):
    for name, tol in (("f32", 1e-6), ("bf16", 1e-2)):
        g = golden("rmsnorm")[name]
        y = rmsnorm_ref(g["x"], g["w"], g["eps"])
        torch.testing.assert_close(y.float(), g["y"].float(), rtol=tol, atol=tol)


def test_rmsswiglu(golden):
    g = golden("rmsswiglu")["f32"]
    y = rmsswiglu_ref(g["x"], g["w"], g["gate"], g["up"], g["eps"])
    torch.testing.assert_close(y, g["y"], rtol=1e-5, atol=1e-6)
    fused = torch.cat([g["gate"], g["up"]], 0)
    y2 = rmsswiglu_ref(g["x"], g["w"], fused, None, g["eps"])
    torch.testing.assert_close(y2, g["y"], rtol=1e-5, atol=1e-6)
    gb = golden("rmsswiglu")["bf16"]
    yb = rmsswiglu_ref(gb["x"], gb["w"], gb["gate"], gb["up"], gb["eps"])
    assert torch.equal(yb, gb["y"])


def test_kv_append_bit_exact(golden):
    g = golden("kv_cache")
    kc = torch.zeros_like(g["k_cache"])
    vc = torch.zeros_like(g["v_cache"])
    kv_append_ref(g["k_src"].view(torch.int16).numpy(), g["v_src"].view(torch.int16).numpy(),
                  kc.view(torch.int16).numpy(), vc.view(torch.int16).numpy(), g["slots"].numpy())
    assert torch.equal(kc.view(torch.int16), g["k_cache"].view(torch.int16))
    assert torch.equal(vc.view(torch.int16), g["v_cache"].view(torch.int16))
    # the slot semantics the reference test spells out (tests/test_kv_cache.py:85-118)
    S = g["max_seq"]
    for t, s in enumerate(g["slots"].tolist()):
        if s >= 0:
            assert torch.equal(g["k_cache"][s // S, :, s % S], g["k_src"][t])


def test_attention(golden):
    for name, g in golden("attention").items():
        o = attention_ref(g["q"], g["k"], g["v"], causal=g["causal"], sm_scale=128 ** -0.5)
        torch.testing.assert_close(o, g["out"], rtol=1e-5, atol=1e-5, msg=name)


def test_rope_kv_append_matches_composition():
    g = torch.Generator().manual_seed(3)
    B, S, H, Hkv, D, Smax = 2, 3, 2, 1, 128, 16
    qkv = torch.randn(B, S, (H + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    pos = torch.tensor([[4, 5, 6], [0, 1, 2]])
    from oracle.model_ref import rope_tables
    c, s = rope_tables(D, 32, 10000.0)
    c, s = c.to(torch.bfloat16), s.to(torch.bfloat16)
    kc = torch.zeros(B, Hkv, Smax, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = rope_kv_append_ref(qkv, pos, c, s, kc, vc, H, Hkv)
    qr, kr = rope_ref(qkv[..., :H * D].reshape(B, S, H, D), qkv[..., H * D:(H + Hkv) * D].reshape(B, S, Hkv, D),
                      c[pos].unsqueeze(2), s[pos].unsqueeze(2))
    assert torch.equal(q, qr.permute(0, 2, 1, 3))
    assert torch.equal(kc[1, 0, 0], kr[1, 0, 0])
    assert torch.equal(vc[0, 0, 6], qkv[0, 2, (H + Hkv) * D:])


def test_model_oracle_matches_reference_greedy(golden):
    for name, g in golden("model").items():
        cfg = g["cfg"]
        sd = make_state_dict(cfg, g["seed"])
        assert abs(float(sum(v.double().sum() for v in sd.values())) - g["weight_checksum"]) < 1e-6
        orc = OracleLlama(cfg, sd, max_seq_len=cfg["max_seq_len"])
        toks, gaps, margins = orc.greedy(g["prompt"], g["tokens"].shape[1])
        assert torch.equal(toks, g["tokens"]), name
        # cached decode logits == reference full-recompute logits at the last step
        cache = [None] * cfg["num_layers"]
        full = torch.cat([g["prompt"], g["tokens"][:, :-1]], 1)
        P = full.shape[1]
        lg = orc.forward(full, torch.arange(P).unsqueeze(0).expand(2, -1), cache)[:, -1]
        torch.testing.assert_close(lg, g["last_logits"], rtol=1e-4, atol=1e-4)
