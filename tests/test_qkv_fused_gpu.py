"""Fused attention-block projection: q/k/v GEMM on packed weights with RoPE
and the KV append in the epilogue (lpc_qkv_rope_append).

Checks:
  * the "heads" packing is a pure byte permutation: bit-exact against a numpy
    restatement (per head, rows d and d + 64 interleaved 16 at a time);
  * bit-identical q, K cache and V cache to the two-kernel path on the same
    packed GEMM (packed_linear "store", then rope_kv_append /
    rope_kv_append_ragged): both accumulate the same products in the same
    order, and the epilogue rounds to the dtype before the same rotation;
  * against the fp32 oracle (projection in fp32, rounded, then the reference
    RoPE + scatter): within max(2e-2, 1 ulp);
  * skipped (negative) positions, flagged out-of-range rows, argument errors.
"""
import numpy as np
import pytest
import torch

from llama_pure_compute_b200 import _lib, ops
from llama_pure_compute_b200.model import precompute_freqs_cis
from llama_pure_compute_b200.packed_linear import PackedWeight, packed_linear
from oracle.ops_ref import rope_kv_append_ref

from test_wsgemm_gpu import _u16, half_ulp_bar, pack_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
D = 128


@pytest.fixture(autouse=True)
def _clean_status():
    yield
    assert _lib.device_status() == 0, "a kernel flagged a device-side error"


def tile_order_heads(w: np.ndarray) -> np.ndarray:
    """Rows of the "heads" tiles: tile row 32q + l is head dim 16q + l (l < 16)
    or 64 + 16q + (l - 16)."""
    n, k = w.shape
    r = np.arange(128)
    q, l = r // 32, r % 32
    d = np.where(l < 16, 16 * q + l, 64 + 16 * q + (l - 16))
    heads = w.reshape(n // 128, 128, k)
    return heads[:, d, :].reshape(n, k)


def tables(max_pos, dtype):
    cos, sin = precompute_freqs_cis(D, max_pos, theta=10000.0, device=DEV)
    return cos.to(dtype), sin.to(dtype)


def make(B, S, H, Hkv, dim, dtype, seed, Smax=64):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(B, S, dim, generator=g, device=DEV).to(dtype)
    w = (torch.randn((H + 2 * Hkv) * D, dim, generator=g, device=DEV) * dim ** -0.5).to(dtype)
    pos = torch.randint(0, Smax - S, (B, 1), generator=g, device=DEV) + torch.arange(S, device=DEV)
    return x, w, pos


def test_pack_heads_layout_bit_exact():
    g = torch.Generator().manual_seed(3)
    w = torch.randn(3 * 128, 192, generator=g).to(torch.bfloat16)
    pw = PackedWeight(w.to(DEV), layout="heads")
    assert np.array_equal(pw.data.cpu().numpy().view(np.uint16), pack_ref(tile_order_heads(_u16(w))))


@pytest.mark.parametrize("splits", [None, "1", "2", "3", "4"])
@pytest.mark.parametrize("B,S,H,Hkv,dim,dtype", [
    (32, 1, 8, 8, 512, torch.bfloat16), (5, 1, 8, 2, 256, torch.bfloat16),
    (3, 4, 4, 4, 320, torch.float16), (64, 1, 4, 1, 1024, torch.bfloat16),
    (1, 1, 32, 32, 4096, torch.bfloat16),
])
def test_fused_equals_two_kernel_path_dense(monkeypatch, splits, B, S, H, Hkv, dim, dtype):
    if splits is not None:
        monkeypatch.setenv("LPC_WSGEMM_SPLITS", splits)
    x, w, pos = make(B, S, H, Hkv, dim, dtype, B * 100 + H + dim)
    cos, sin = tables(64, dtype)
    Bmax, Smax = B + 1, 64
    kc0 = torch.randn(Bmax, Hkv, Smax, D, device=DEV).to(dtype)
    vc0 = torch.randn_like(kc0)
    kc1, vc1 = kc0.clone(), vc0.clone()
    q_fused = ops.qkv_rope_append(x, PackedWeight(w, layout="heads"), pos, cos, sin, kc0, vc0, H, Hkv)
    qkv = packed_linear(x, PackedWeight(w))
    q_two = ops.rope_kv_append(qkv, pos, cos, sin, kc1, vc1, H, Hkv)
    assert torch.equal(q_fused, q_two)
    assert torch.equal(kc0, kc1)
    assert torch.equal(vc0, vc1)


@pytest.mark.parametrize("H,Hkv", [(8, 8), (8, 2)])
def test_fused_equals_two_kernel_path_ragged(H, Hkv):
    dtype = torch.bfloat16
    caps = [9, 40, 17, 64]
    B, dim = len(caps), 512
    g = torch.Generator(device=DEV).manual_seed(H * 7 + Hkv)
    x = torch.randn(B, 1, dim, generator=g, device=DEV).to(dtype)
    w = (torch.randn((H + 2 * Hkv) * D, dim, generator=g, device=DEV) * dim ** -0.5).to(dtype)
    pos = torch.tensor([[c - 1] for c in caps], device=DEV)
    base, acc = [], 0
    for c in caps:
        base.append(acc)
        acc += c
    sb = torch.tensor(base, dtype=torch.int64, device=DEV)
    sc = torch.tensor(caps, dtype=torch.int32, device=DEV)
    cos, sin = tables(64, dtype)
    kc0 = torch.randn(Hkv, acc, D, device=DEV).to(dtype)
    vc0 = torch.randn_like(kc0)
    kc1, vc1 = kc0.clone(), vc0.clone()
    q_fused = ops.qkv_rope_append(x, PackedWeight(w, layout="heads"), pos, cos, sin, kc0, vc0, H,
                                  Hkv, seq_base=sb, seq_cap=sc)
    qkv = packed_linear(x, PackedWeight(w))
    q_two = ops.rope_kv_append_ragged(qkv, pos, cos, sin, kc1, vc1, sb, sc, H, Hkv)
    assert torch.equal(q_fused, q_two)
    assert torch.equal(kc0, kc1)
    assert torch.equal(vc0, vc1)


@pytest.mark.parametrize("B,S,H,Hkv,dim", [(16, 1, 8, 2, 512), (2, 3, 4, 4, 256)])
def test_fused_against_oracle(B, S, H, Hkv, dim):
    dtype = torch.bfloat16
    x, w, pos = make(B, S, H, Hkv, dim, dtype, 41 + B)
    cos, sin = tables(64, dtype)
    kc = torch.zeros(B, Hkv, 64, D, device=DEV, dtype=dtype)
    vc = torch.zeros_like(kc)
    q = ops.qkv_rope_append(x, PackedWeight(w, layout="heads"), pos, cos, sin, kc, vc, H, Hkv)
    qkv_ref = (x.float() @ w.float().t()).to(dtype)
    kr, vr = torch.zeros_like(kc), torch.zeros_like(vc)
    q_ref = rope_kv_append_ref(qkv_ref, pos, cos, sin, kr, vr, H, Hkv)
    half_ulp_bar(q, q_ref, dtype, "q")
    half_ulp_bar(kc, kr, dtype, "k cache")
    half_ulp_bar(vc, vr, dtype, "v cache")


def test_negative_positions_skipped_and_out_of_range_flagged():
    dtype = torch.bfloat16
    B, H, Hkv, dim = 4, 4, 2, 256
    x, w, _ = make(B, 1, H, Hkv, dim, dtype, 5)
    cos, sin = tables(64, dtype)
    pw = PackedWeight(w, layout="heads")
    kc = torch.zeros(B, Hkv, 32, D, device=DEV, dtype=dtype)
    vc = torch.zeros_like(kc)
    pos = torch.tensor([[3], [-1], [5], [-7]], device=DEV)
    ops.qkv_rope_append(x, pw, pos, cos, sin, kc, vc, H, Hkv)
    assert _lib.device_status() == 0
    assert kc[1].abs().sum() == 0 and kc[3].abs().sum() == 0 and vc[1].abs().sum() == 0
    assert kc[0, :, 3].abs().sum() > 0 and vc[2, :, 5].abs().sum() > 0
    before = kc.clone()
    ops.qkv_rope_append(x, pw, torch.tensor([[40]] * B, device=DEV), cos, sin, kc, vc, H, Hkv)
    assert _lib.device_status() & 0x2  # out-of-range position: bounds flag
    assert torch.equal(kc, before)


def test_fused_errors():
    dtype = torch.bfloat16
    x, w, pos = make(2, 1, 2, 2, 256, dtype, 1)
    cos, sin = tables(64, dtype)
    kc = torch.zeros(2, 2, 64, D, device=DEV, dtype=dtype)
    vc = torch.zeros_like(kc)
    with pytest.raises(ValueError):  # not a "heads" packing
        ops.qkv_rope_append(x, PackedWeight(w), pos, cos, sin, kc, vc, 2, 2)
    pw = PackedWeight(w, layout="heads")
    with pytest.raises(ValueError):  # head count mismatch
        ops.qkv_rope_append(x, pw, pos, cos, sin, kc, vc, 4, 1)
    with pytest.raises(TypeError):  # tables in another dtype
        ops.qkv_rope_append(x, pw, pos, cos.float(), sin.float(), kc, vc, 2, 2)
    with pytest.raises(ValueError):  # heads packing needs whole 128-row heads
        PackedWeight(torch.zeros(200, 64, device=DEV, dtype=dtype), layout="heads")
    with pytest.raises(ValueError):  # a heads packing is not a plain linear weight
        packed_linear(x, pw)
