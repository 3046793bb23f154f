"""Attention at head_dim 64 and 32 (the reference accepts 32, 64 and 128,
triton_kernels/flash_attention.py:1091-1098).

Mirrors the reference's own attention tests (tests/test_attention_correctness.py:
prefill grid :115-185 with head_dim 64, unaligned prefill :188-230, decode
:233-300) with their tolerances (rtol = atol = 1e-2 for fp16, 2e-2 for bf16),
against the fp32 oracle (evaluated on the GPU for the larger shapes), and adds
head_dim 32: prefill through the head_dim-64 tcgen05 kernel on zero-padded
q/k/v, decode natively (one dim per lane).
"""
import pytest
import torch

from llama_pure_compute_b200 import _lib, ops
from llama_pure_compute_b200.flash_attention import flash_attention_v2
from oracle.ops_ref import attention_ref, decode_attention_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _clean_status():
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    assert _lib.device_status() == 0


def close(actual, expected, dtype, what):
    tol = 1e-2 if dtype == torch.float16 else 2e-2
    torch.testing.assert_close(actual.float(), expected.float(), rtol=tol, atol=tol, msg=what)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("head_dim", [32, 64])
@pytest.mark.parametrize("S", [128, 512, 2048])
@pytest.mark.parametrize("B,H", [(1, 8), (4, 16)])
def test_prefill_head_dims(B, H, S, head_dim, causal, dtype):
    g = torch.Generator(device=DEV).manual_seed(42 + S + head_dim)
    q = torch.randn(B, H, S, head_dim, device=DEV, generator=g, dtype=dtype)
    k = torch.randn(B, H, S, head_dim, device=DEV, generator=g, dtype=dtype)
    v = torch.randn(B, H, S, head_dim, device=DEV, generator=g, dtype=dtype)
    scale = head_dim ** -0.5
    out = flash_attention_v2(q, k, v, causal=causal, sm_scale=scale)
    assert out.shape == q.shape
    close(out, attention_ref(q, k, v, causal=causal, sm_scale=scale), dtype,
          f"prefill B={B} H={H} S={S} D={head_dim} causal={causal} {dtype}")


@pytest.mark.parametrize("S", [127, 357, 513, 1025])
def test_unaligned_prefill_head_dim_64(S):
    g = torch.Generator(device=DEV).manual_seed(1337 + S)
    q = torch.randn(2, 4, S, 64, device=DEV, generator=g, dtype=torch.float16)
    k = torch.randn(2, 4, S, 64, device=DEV, generator=g, dtype=torch.float16)
    v = torch.randn(2, 4, S, 64, device=DEV, generator=g, dtype=torch.float16)
    close(flash_attention_v2(q, k, v, causal=False), attention_ref(q, k, v, causal=False),
          torch.float16, f"unaligned prefill S={S}")


def test_prefill_head_dim_64_gqa_and_q_shorter_than_kv():
    g = torch.Generator(device=DEV).manual_seed(7)
    q = torch.randn(2, 8, 300, 64, device=DEV, generator=g, dtype=torch.bfloat16)
    k = torch.randn(2, 2, 700, 64, device=DEV, generator=g, dtype=torch.bfloat16)
    v = torch.randn(2, 2, 700, 64, device=DEV, generator=g, dtype=torch.bfloat16)
    close(flash_attention_v2(q, k, v, causal=True), attention_ref(q, k, v, causal=True),
          torch.bfloat16, "GQA, q_len < kv_len, D=64")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [32, 64])
@pytest.mark.parametrize("kv_len", [128, 512, 2048])
@pytest.mark.parametrize("B,H", [(1, 8), (4, 16)])
def test_decode_head_dims(B, H, kv_len, head_dim, dtype):
    g = torch.Generator(device=DEV).manual_seed(1234 + kv_len)
    q = torch.randn(B, H, 1, head_dim, device=DEV, generator=g, dtype=dtype)
    k = torch.randn(B, H, kv_len, head_dim, device=DEV, generator=g, dtype=dtype)
    v = torch.randn(B, H, kv_len, head_dim, device=DEV, generator=g, dtype=dtype)
    scale = head_dim ** -0.5
    out = flash_attention_v2(q, k, v, causal=True, sm_scale=scale)
    close(out, attention_ref(q, k, v, causal=True, sm_scale=scale), dtype,
          f"decode B={B} H={H} KV={kv_len} D={head_dim} {dtype}")


@pytest.mark.parametrize("G", [1, 4])
def test_decode_head_dim_32_ragged(G):
    g = torch.Generator().manual_seed(G)
    B, Hkv, Smax, D = 6, 2, 700, 32
    lens = torch.tensor([1, 2, 255, 256, 257, 700], dtype=torch.int32)
    kc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hkv * G, D, generator=g).to(torch.bfloat16)
    o = ops.decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), lens.to(DEV)).cpu().float()
    ref = decode_attention_ref(q, kc, vc, lens).float()
    assert (o - ref).abs().max().item() <= 2e-2
