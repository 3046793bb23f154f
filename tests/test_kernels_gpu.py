"""Parity of every sm_100a kernel with the CPU oracle (and, at sizes the CPU
oracle cannot finish quickly, with the same fp32 formulas evaluated by torch on
the GPU).  Tolerances are written next to each check:
  * copies and RoPE: bit-exact;
  * fp32: 1e-5 relative (+1e-5 absolute on O(1) data);
  * bf16 attention / SwiGLU: 2e-2 max-abs where the output scale allows it,
    plus the reference tests' rtol/atol band with its outlier fraction.
"""
import math

import numpy as np
import pytest
import torch

from llama_pure_compute_b200 import _lib, ops
from llama_pure_compute_b200.flash_attention import flash_attention_v2
from oracle.model_ref import rope_tables
from oracle.ops_ref import (attention_ref, decode_attention_ref, kv_append_ref, rmsnorm_ref,
                            rmsswiglu_ref, rope_kv_append_ref, rope_ref)

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _clean_status():
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    assert _lib.device_status() == 0, "a kernel flagged a device-side error"


def half_ulp_bar(out, ref, dtype, msg=""):
    """|out - ref| <= max(2e-2, one ulp of ref in `dtype`): the 2e-2 max-abs
    bar wherever the output dtype can represent it; at |ref| >= 4 (bf16) one
    ulp already exceeds 2e-2, so two once-rounded results may differ by it."""
    out, ref = out.float(), ref.float()
    mant = 7 if dtype == torch.bfloat16 else 10
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - mant)
    err = (out - ref).abs()
    bad = err > torch.maximum(torch.full_like(err, 2e-2), ulp)
    assert not bad.any(), f"{msg}: {int(bad.sum())} elements beyond max(2e-2, 1 ulp); worst {err.max().item()}"


def band_check(out, ref, rtol, atol, outlier_frac, msg=""):
    """tests/test_rmsswiglu_correctness.py:92-126: elements outside
    atol + rtol*|ref| may be at most `outlier_frac`, none beyond 10x the band."""
    out, ref = out.float(), ref.float()
    diff = (out - ref).abs()
    allowed = atol + rtol * ref.abs()
    bad = diff > allowed
    frac = bad.float().mean().item()
    worst = (diff[bad] / allowed[bad]).max().item() if bad.any() else 0.0
    assert frac <= outlier_frac and worst <= 10.0, f"{msg}: {frac:.5%} outside band, worst {worst:.2f}x"


# ---------------------------------------------------------------------------
# KV append: bit-exact
# ---------------------------------------------------------------------------
def test_kv_append_golden(golden):
    g = golden("kv_cache")
    kc = torch.zeros_like(g["k_cache"]).to(DEV)
    vc = torch.zeros_like(g["v_cache"]).to(DEV)
    ops.update_kv_cache(g["k_src"].to(DEV), g["v_src"].to(DEV), kc, vc, g["slots"].to(DEV))
    assert torch.equal(kc.cpu().view(torch.int16), g["k_cache"].view(torch.int16))
    assert torch.equal(vc.cpu().view(torch.int16), g["v_cache"].view(torch.int16))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 128, 40])
def test_kv_append_random_slots(dtype, head_dim):
    g = torch.Generator().manual_seed(5)
    Bmax, H, S = 6, 4, 33
    T = 50
    slots = torch.randperm(Bmax * S, generator=g)[:T].to(torch.int64)
    slots[::7] = -1
    k = torch.randn(T, H, head_dim, generator=g).to(dtype)
    v = torch.randn(T, H, head_dim, generator=g).to(dtype)
    kc = torch.randn(Bmax, H, S, head_dim, generator=g).to(dtype)
    vc = torch.randn(Bmax, H, S, head_dim, generator=g).to(dtype)
    kd, vd = kc.to(DEV), vc.to(DEV)
    ops.update_kv_cache(k.to(DEV), v.to(DEV), kd, vd, slots.to(DEV))
    it = torch.int32 if dtype == torch.float32 else torch.int16
    kn, vn = kc.view(it).numpy().copy(), vc.view(it).numpy().copy()
    kv_append_ref(k.view(it).numpy(), v.view(it).numpy(), kn, vn, slots.numpy())
    assert np.array_equal(kd.cpu().view(it).numpy(), kn)
    assert np.array_equal(vd.cpu().view(it).numpy(), vn)


@pytest.mark.parametrize("T,H,D,dtype", [(2000, 8, 128, torch.bfloat16), (10, 128, 128, torch.bfloat16),
                                         (700, 4, 128, torch.float32), (3000, 1, 64, torch.float16)])
def test_kv_append_token_runs(T, H, D, dtype):
    """Token counts and head counts that give runs of several tokens per CTA
    (a few heads), and runs longer than one batch of loads (128 heads)."""
    g = torch.Generator().manual_seed(T + H)
    Bmax, S = 8, (T + 7) // 8 + 3
    slots = torch.randperm(Bmax * S, generator=g)[:T].to(torch.int64)
    slots[::11] = -1
    k = torch.randn(T, H, D, generator=g).to(dtype)
    v = torch.randn(T, H, D, generator=g).to(dtype)
    kc = torch.randn(Bmax, H, S, D, generator=g).to(dtype)
    vc = torch.randn(Bmax, H, S, D, generator=g).to(dtype)
    kd, vd = kc.to(DEV), vc.to(DEV)
    ops.update_kv_cache(k.to(DEV), v.to(DEV), kd, vd, slots.to(DEV))
    it = torch.int32 if dtype == torch.float32 else torch.int16
    kn, vn = kc.view(it).numpy().copy(), vc.view(it).numpy().copy()
    kv_append_ref(k.view(it).numpy(), v.view(it).numpy(), kn, vn, slots.numpy())
    assert np.array_equal(kd.cpu().view(it).numpy(), kn)
    assert np.array_equal(vd.cpu().view(it).numpy(), vn)


def test_kv_append_default_slots_and_empty():
    k = torch.randn(3, 2, 128, device=DEV, dtype=torch.bfloat16)
    kc = torch.zeros(2, 2, 4, 128, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    ops.update_kv_cache(k, k, kc, vc, None)  # slot = token index: (0,0),(0,1),(0,2)
    assert torch.equal(kc[0, :, :3].transpose(0, 1), k)
    ops.update_kv_cache(k[:0], k[:0], kc, vc, torch.empty(0, dtype=torch.int64, device=DEV))


def test_kv_append_out_of_range_slot_is_flagged_not_written():
    k = torch.randn(2, 1, 128, device=DEV, dtype=torch.bfloat16)
    kc = torch.zeros(1, 1, 4, 128, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    ops.update_kv_cache(k, k, kc, vc, torch.tensor([1, 4], device=DEV))  # slot 4 = row 1: out of range
    assert _lib.device_status() & 0x2
    assert torch.equal(kc[0, 0, 1], k[0, 0]) and kc[0, 0, 2:].abs().sum() == 0


# ---------------------------------------------------------------------------
# RoPE: bit-exact against the oracle
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["model_f32", "model_bf16", "model_f16", "half_f32"])
def test_rope_golden_inputs(golden, name):
    g = golden("rope")[name]
    q, k = g["q"].to(DEV), g["k"].to(DEV)
    qo, ko = ops.rope_forward(q, k, g["cos"].to(DEV), g["sin"].to(DEV), g["pos"].to(DEV))
    qr, kr = rope_ref(g["q"], g["k"], g["cos"], g["sin"], g["pos"])
    assert torch.equal(qo.cpu(), qr) and torch.equal(ko.cpu(), kr)
    if name in ("model_f32", "half_f32"):  # the reference itself, fp32: exact too
        assert torch.equal(qo.cpu(), g["q_out"]) or torch.allclose(qo.cpu(), g["q_out"], 1e-6, 1e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H,Hkv", [(32, 32), (32, 8), (64, 8)])
@pytest.mark.parametrize("B,S", [(1, 1), (1, 128), (4, 512)])
def test_rope_shapes(dtype, H, Hkv, B, S):
    g = torch.Generator().manual_seed(B * 1000 + S)
    D = 128
    q = torch.randn(B, S, H, D, generator=g).to(dtype)
    k = torch.randn(B, S, Hkv, D, generator=g).to(dtype)
    cos, sin = rope_tables(D, 1024, 10000.0)
    half_c, half_s = cos[:, :64].contiguous().to(dtype), sin[:, :64].contiguous().to(dtype)
    pos = torch.randint(0, 1024, (B, S), generator=g)
    qo, ko = ops.rope_forward(q.to(DEV), k.to(DEV), half_c.to(DEV), half_s.to(DEV), pos.to(DEV))
    qr, kr = rope_ref(q, k, half_c, half_s, pos)
    assert torch.equal(qo.cpu(), qr) and torch.equal(ko.cpu(), kr)


def test_rope_in_place_and_no_position_ids():
    q = torch.randn(1, 16, 8, 128, device=DEV)
    k = torch.randn(1, 16, 2, 128, device=DEV)
    q0, k0 = q.cpu(), k.cpu()
    cos, sin = rope_tables(128, 256, 10000.0)
    c, s = cos[:, :64].contiguous(), sin[:, :64].contiguous()
    pq, pk = q.data_ptr(), k.data_ptr()
    qo, ko = ops.rope_forward(q, k, c.to(DEV), s.to(DEV), None)
    assert qo.data_ptr() == pq and ko.data_ptr() == pk
    qr, kr = rope_ref(q0, k0, c, s, None)
    assert torch.equal(qo.cpu(), qr) and torch.equal(ko.cpu(), kr)


def test_rope_position_out_of_table_is_flagged():
    q = torch.randn(1, 2, 1, 128, device=DEV)
    cos = torch.ones(4, 64, device=DEV)
    ops.rope_forward(q, q.clone(), cos, cos, torch.tensor([[1, 9]], device=DEV))
    assert _lib.device_status() & 0x2


@pytest.mark.parametrize("B,S,H,Hkv", [(3, 5, 4, 2), (64, 1, 32, 32), (2, 17, 8, 8), (4, 300, 4, 2),
                                       (2, 3, 128, 8), (1, 700, 32, 8)])
def test_rope_kv_append_bit_exact(B, S, H, Hkv):
    g = torch.Generator().manual_seed(7)
    D, Smax = 128, S + 35
    qkv = torch.randn(B, S, (H + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    start = torch.randint(0, Smax - S, (B, 1), generator=g)
    pos = start + torch.arange(S).unsqueeze(0)
    cos, sin = rope_tables(D, Smax + 24, 10000.0)
    cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
    kc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16)
    kd, vd = kc.to(DEV), vc.to(DEV)
    q = ops.rope_kv_append(qkv.to(DEV), pos.to(DEV), cos.to(DEV), sin.to(DEV), kd, vd, H, Hkv)
    qr = rope_kv_append_ref(qkv, pos, cos, sin, kc, vc, H, Hkv)
    assert torch.equal(q.cpu(), qr)
    assert torch.equal(kd.cpu(), kc) and torch.equal(vd.cpu(), vc)


@pytest.mark.parametrize("D,H,Hkv", [(64, 8, 2), (32, 16, 4), (96, 12, 4)])
def test_rope_kv_append_head_dims(D, H, Hkv):
    """Other head dims: 4, 2 and 6 chunks of 8 rotation pairs per head, so
    64, 128 and 42 heads per block step (a 252-thread block for 96)."""
    g = torch.Generator().manual_seed(D)
    B, S, Smax = 3, 37, 64
    qkv = torch.randn(B, S, (H + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, Smax - S, (B, 1), generator=g) + torch.arange(S).unsqueeze(0)
    pos[1, 5] = -1  # skipped token
    cos, sin = rope_tables(D, Smax, 10000.0)
    cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
    kc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16)
    kd, vd = kc.to(DEV), vc.to(DEV)
    q = ops.rope_kv_append(qkv.to(DEV), pos.to(DEV), cos.to(DEV), sin.to(DEV), kd, vd, H, Hkv)
    qr = rope_kv_append_ref(qkv, pos, cos, sin, kc, vc, H, Hkv)
    valid = (pos >= 0).view(B, 1, S, 1).expand_as(qr)
    assert torch.equal(q.cpu()[valid], qr[valid])
    assert torch.equal(kd.cpu(), kc) and torch.equal(vd.cpu(), vc)


# ---------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-6), (torch.bfloat16, 8e-3),
                                       (torch.float16, 1e-3)])
@pytest.mark.parametrize("rows,dim", [(1, 4096), (7, 4096), (300, 2048), (5, 1000), (3, 8192)])
def test_rmsnorm(dtype, tol, rows, dim):
    g = torch.Generator().manual_seed(rows + dim)
    x = (torch.randn(rows, dim, generator=g) * 2).to(dtype)
    w = (1 + 0.02 * torch.randn(dim, generator=g)).to(dtype)
    y = ops.rmsnorm_forward(x.to(DEV), w.to(DEV), 1e-5).cpu()
    torch.testing.assert_close(y.float(), rmsnorm_ref(x, w, 1e-5).float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("rows", [1, 150, 600, 1200, 2400, 5000])
@pytest.mark.parametrize("dim,xd,wd", [(4096, torch.bfloat16, torch.bfloat16),
                                       (4096, torch.bfloat16, torch.float32),
                                       (2048, torch.float32, torch.bfloat16),
                                       (1024, torch.float16, torch.float16),
                                       (8192, torch.bfloat16, torch.bfloat16)])
def test_rmsnorm_row_layouts(rows, dim, xd, wd):
    """Every rows-per-CTA choice (1-8 rows of one, two or four warps) and
    weight dtypes other than x's, against the oracle at the dtype's bar."""
    g = torch.Generator().manual_seed(rows * 7 + dim)
    x = (torch.randn(rows, dim, generator=g) * 2).to(xd)
    w = (1 + 0.02 * torch.randn(dim, generator=g)).to(wd)
    y = ops.rmsnorm_forward(x.to(DEV), w.to(DEV), 1e-5).cpu()
    tol = {torch.float32: 2e-6, torch.bfloat16: 8e-3, torch.float16: 1e-3}[xd]
    torch.testing.assert_close(y.float(), rmsnorm_ref(x, w, 1e-5).float(), rtol=tol, atol=tol)


def test_rmsnorm_golden(golden):
    for name, tol in (("f32", 2e-6), ("bf16", 8e-3)):
        gg = golden("rmsnorm")[name]
        y = ops.rmsnorm_forward(gg["x"].to(DEV), gg["w"].to(DEV), gg["eps"]).cpu()
        torch.testing.assert_close(y.float(), gg["y"].float(), rtol=tol, atol=tol)


# ---------------------------------------------------------------------------
# Fused RMSNorm + SwiGLU
# ---------------------------------------------------------------------------
def test_rmsswiglu_fp32_op_shape():
    """fp32 op shape: x [8, 4096] ~N(0,1), w ~N(1, 0.02), W ~N(0, 0.02), eps 1e-6, seed 0.
    Bar: fp32 within 1e-5 relative (atol 1e-5 on O(1) outputs) of the fp64
    evaluation of the same formula."""
    torch.manual_seed(0)
    x = torch.randn(8, 4096)
    w = 1 + 0.02 * torch.randn(4096)
    gw = 0.02 * torch.randn(11008, 4096)
    uw = 0.02 * torch.randn(11008, 4096)
    y = ops.rmsswiglu_forward(x.to(DEV), w.to(DEV), gw.to(DEV), uw.to(DEV), 1e-6).cpu()
    ref64 = rmsswiglu_ref(x.double(), w.double(), gw.double(), uw.double(), 1e-6, torch.float64)
    torch.testing.assert_close(y.double(), ref64, rtol=1e-5, atol=1e-5)
    ref32 = rmsswiglu_ref(x, w, gw, uw, 1e-6)  # the reference's fp32 CPU path
    torch.testing.assert_close(y, ref32, rtol=1e-5, atol=1e-5)


def test_rmsswiglu_golden(golden):
    gg = golden("rmsswiglu")["f32"]
    y = ops.rmsswiglu_forward(gg["x"].to(DEV), gg["w"].to(DEV), gg["gate"].to(DEV), gg["up"].to(DEV),
                              gg["eps"]).cpu()
    torch.testing.assert_close(y, gg["y"], rtol=1e-5, atol=1e-5)
    gb = golden("rmsswiglu")["bf16"]
    yb = ops.rmsswiglu_forward(gb["x"].to(DEV), gb["w"].to(DEV), gb["gate"].to(DEV), gb["up"].to(DEV),
                               gb["eps"]).cpu()
    band_check(yb, gb["y"], 1.5e-2, 1.5e-2, 0.002, "rmsswiglu golden bf16")
    half_ulp_bar(yb, rmsswiglu_ref(gb["x"], gb["w"], gb["gate"], gb["up"], gb["eps"],
                                   round_normed=True), torch.bfloat16, "rmsswiglu golden bf16")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,S", [(1, 1), (1, 128), (4, 512), (2, 2048)])
@pytest.mark.parametrize("D,I", [(4096, 11008), (2048, 5632)])
def test_rmsswiglu_tensor_core_shapes(dtype, B, S, D, I):
    """Shapes of tests/test_rmsswiglu_correctness.py:134-171 with its weight
    scaling (randn / sqrt(fan_in)); fp32 truth computed with torch on the GPU."""
    g = torch.Generator(device=DEV).manual_seed(42)
    x = torch.randn(B, S, D, device=DEV, generator=g).to(dtype)
    w = (1 + 0.02 * torch.randn(D, device=DEV, generator=g)).to(dtype)
    gw = (torch.randn(I, D, device=DEV, generator=g) / D ** 0.5).to(dtype)
    uw = (torch.randn(I, D, device=DEV, generator=g) / D ** 0.5).to(dtype)
    y = ops.rmsswiglu_forward(x, w, gw, uw, 1e-6)
    ref = rmsswiglu_ref(x, w, gw, uw, 1e-6)  # fp32 math on the GPU, rounded once
    ref_cuda = rmsswiglu_ref(x, w, gw, uw, 1e-6, round_normed=True)  # rmsswiglu.cu semantics
    assert y.shape == (B, S, I)
    half_ulp_bar(y, ref_cuda, dtype, "rmsswiglu")
    rt = 1.5e-2 if dtype == torch.bfloat16 else 1e-3
    band_check(y, ref, rt, rt, 0.002, "rmsswiglu")
    # pre-fused [2I, D] weight form gives the same result
    y2 = ops.rmsswiglu_forward(x, w, torch.cat([gw, uw], 0), torch.empty(0, device=DEV, dtype=dtype), 1e-6)
    assert torch.equal(y, y2)


def test_rmsswiglu_op_shape_bf16_distribution():
    """The fp32 op shape's distributions in bf16 (|out| reaches ~10): the
    reference band with its 0.2% outlier budget; max-abs bounded by the bf16
    spacing of the largest outputs."""
    torch.manual_seed(0)
    x = torch.randn(8, 4096).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(4096)).to(torch.bfloat16)
    gw = (0.02 * torch.randn(11008, 4096)).to(torch.bfloat16)
    uw = (0.02 * torch.randn(11008, 4096)).to(torch.bfloat16)
    y = ops.rmsswiglu_forward(x.to(DEV), w.to(DEV), gw.to(DEV), uw.to(DEV), 1e-6).cpu()
    ref = rmsswiglu_ref(x, w, gw, uw, 1e-6)
    band_check(y, ref, 1.5e-2, 1.5e-2, 0.002, "rmsswiglu bf16 op shape")
    half_ulp_bar(y, rmsswiglu_ref(x, w, gw, uw, 1e-6, round_normed=True), torch.bfloat16,
                 "rmsswiglu bf16 op shape")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_rmsswiglu_zero_large_ranks_and_repeatability(dtype):
    """As tests/test_rmsswiglu_correctness.py:174-263 of the reference: 1-D /
    2-D / 3-D inputs, all-zero rows (exact zeros out), inputs scaled by 1e3
    (the norm removes the scale), and bit-identical repeated calls (the split
    and pair reductions have a fixed order)."""
    g = torch.Generator(device=DEV).manual_seed(11)
    D, I = 1024, 640
    w = (1 + 0.02 * torch.randn(D, device=DEV, generator=g)).to(dtype)
    gw = (torch.randn(I, D, device=DEV, generator=g) / D ** 0.5).to(dtype)
    uw = (torch.randn(I, D, device=DEV, generator=g) / D ** 0.5).to(dtype)
    x = torch.randn(2, 160, D, device=DEV, generator=g).to(dtype)
    x[0, 5] = 0
    x[1, 77] = 0
    tol = (lambda y, r, what: torch.testing.assert_close(y, r, rtol=1e-5, atol=1e-5)) \
        if dtype == torch.float32 else (lambda y, r, what: half_ulp_bar(y, r, dtype, what))
    rnd = dtype != torch.float32
    y3 = ops.rmsswiglu_forward(x, w, gw, uw, 1e-6)
    assert y3.shape == (2, 160, I)
    tol(y3, rmsswiglu_ref(x, w, gw, uw, 1e-6, round_normed=rnd), "rmsswiglu 3-D")
    assert (y3[0, 5] == 0).all() and (y3[1, 77] == 0).all()
    y2 = ops.rmsswiglu_forward(x.reshape(-1, D), w, gw, uw, 1e-6)
    assert y2.shape == (320, I) and torch.equal(y2, y3.reshape(-1, I))
    y1 = ops.rmsswiglu_forward(x[1, 3], w, gw, uw, 1e-6)
    assert y1.shape == (I,)
    tol(y1, rmsswiglu_ref(x[1, 3:4], w, gw, uw, 1e-6, round_normed=rnd)[0], "rmsswiglu 1-D")
    big = (x.float() * 1e3).to(dtype)
    yb = ops.rmsswiglu_forward(big, w, gw, uw, 1e-6)
    assert torch.isfinite(yb.float()).all()
    tol(yb, rmsswiglu_ref(big, w, gw, uw, 1e-6, round_normed=rnd), "rmsswiglu x1e3")
    for xx in (x, x[:, :4]):
        assert torch.equal(ops.rmsswiglu_forward(xx, w, gw, uw, 1e-6),
                           ops.rmsswiglu_forward(xx, w, gw, uw, 1e-6))


@pytest.mark.parametrize("M", [1, 3, 127, 129, 300])
def test_rmsswiglu_ragged_token_counts(M):
    g = torch.Generator(device=DEV).manual_seed(M)
    D, I = 1024, 320
    x = torch.randn(M, D, device=DEV, generator=g).to(torch.bfloat16)
    w = torch.ones(D, device=DEV, dtype=torch.bfloat16)
    gw = (torch.randn(I, D, device=DEV, generator=g) / 32).to(torch.bfloat16)
    uw = (torch.randn(I, D, device=DEV, generator=g) / 32).to(torch.bfloat16)
    y = ops.rmsswiglu_forward(x, w, gw, uw, 1e-5)
    ref = rmsswiglu_ref(x, w, gw, uw, 1e-5, round_normed=True)
    half_ulp_bar(y, ref, torch.bfloat16, f"rmsswiglu M={M}")


@pytest.mark.parametrize("cfg", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("M,D,I,fused", [(1, 1024, 320, False), (129, 1024, 320, True),
                                         (256, 4096, 11008, False), (300, 512, 1024, True)])
def test_rmsswiglu_every_tile_config(monkeypatch, cfg, M, D, I, fused):
    """Every GEMM tile configuration (LPC_SWIGLU_CFG: 1 / 2 / 3 one-CTA tiles
    with 1, 2 or 1 token tiles, 4 / 5 CTA-pair tiles with 3- and 6-deep rings)
    against the oracle, and bit-identical to the default choice."""
    g = torch.Generator(device=DEV).manual_seed(M + I)
    x = torch.randn(M, D, device=DEV, generator=g).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(D, device=DEV, generator=g)).to(torch.bfloat16)
    gw = (torch.randn(I, D, device=DEV, generator=g) / D ** 0.5).to(torch.bfloat16)
    uw = (torch.randn(I, D, device=DEV, generator=g) / D ** 0.5).to(torch.bfloat16)
    args = (torch.cat([gw, uw]), torch.empty(0, device=DEV, dtype=torch.bfloat16)) if fused else (gw, uw)
    y_default = ops.rmsswiglu_forward(x, w, *args, 1e-5)
    monkeypatch.setenv("LPC_SWIGLU_CFG", str(cfg))
    y = ops.rmsswiglu_forward(x, w, *args, 1e-5)
    monkeypatch.delenv("LPC_SWIGLU_CFG")
    ref = rmsswiglu_ref(x, w, gw, uw, 1e-5, round_normed=True)
    half_ulp_bar(y, ref, torch.bfloat16, f"rmsswiglu cfg={cfg} M={M}")
    assert torch.equal(y, y_default), f"cfg {cfg} differs from the default tile choice"


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------
def test_attention_golden(golden):
    for name, g in golden("attention").items():
        q, k, v = (g[n].to(torch.bfloat16).to(DEV) for n in ("q", "k", "v"))
        o = flash_attention_v2(q, k, v, causal=g["causal"], sm_scale=128 ** -0.5).cpu().float()
        assert (o - g["out"]).abs().max().item() <= 2e-2, name
        torch.testing.assert_close(o, g["out"], rtol=2e-2, atol=2e-2, msg=name)


@pytest.mark.parametrize("B,H,S,causal", [(1, 8, 128, True), (4, 16, 512, True), (1, 8, 2048, True),
                                          (2, 4, 200, True), (1, 2, 1000, True), (1, 4, 333, False),
                                          (2, 8, 512, False)])
def test_flash_prefill(B, H, S, causal):
    g = torch.Generator(device=DEV).manual_seed(S)
    q, k, v = (torch.randn(B, H, S, 128, device=DEV, generator=g, dtype=torch.bfloat16)
               for _ in range(3))
    o = flash_attention_v2(q, k, v, causal=causal)
    ref = attention_ref(q, k, v, causal=causal).float()
    assert (o.float() - ref).abs().max().item() <= 2e-2
    torch.testing.assert_close(o.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("profile", ["plateau", "ramp", "drop"])
@pytest.mark.parametrize("causal", [True, False])
def test_flash_prefill_running_max_moves(profile, causal):
    """Scores whose row max moves across key tiles: later tiles a little above
    tile 0 everywhere (row sums of a tile far above 2^8 with the max grown by
    about 3 in log2 units), rising without bound (max grows by more than 8
    per tile), or far below tile 0."""
    B, H, S, D = 1, 2, 1024, 128
    g = torch.Generator(device=DEV).manual_seed(7)
    u = torch.ones(D, device=DEV) / math.sqrt(D)
    pos = torch.arange(S, device=DEV, dtype=torch.float32)
    if profile == "plateau":
        b = torch.where(pos < 128, 1.0, 2.5)
    elif profile == "ramp":
        b = 1.0 + pos / 32.0
    else:
        b = torch.where(pos < 128, 4.0, 0.25)
    noise = lambda s: s * torch.randn(B, H, S, D, device=DEV, generator=g)
    q = (16.0 * u + noise(0.05)).to(torch.bfloat16)
    k = (b[None, None, :, None] * u + noise(0.05)).to(torch.bfloat16)
    v = torch.randn(B, H, S, D, device=DEV, generator=g).to(torch.bfloat16)
    o = flash_attention_v2(q, k, v, causal=causal)
    ref = attention_ref(q, k, v, causal=causal).float()
    assert torch.isfinite(o.float()).all()
    assert (o.float() - ref).abs().max().item() <= 2e-2


def test_flash_prefill_op_shape():
    """Prefill op shape: Q,K,V [4, 32, 2048, 128] ~N(0,1) bf16, causal, scale 1/sqrt(128), seed 1."""
    torch.manual_seed(1)
    q, k, v = (torch.randn(4, 32, 2048, 128).to(torch.bfloat16).to(DEV) for _ in range(3))
    o = flash_attention_v2(q, k, v, causal=True, sm_scale=1 / math.sqrt(128))
    ref = torch.empty(4, 32, 2048, 128, device=DEV)
    for b in range(4):
        ref[b] = attention_ref(q[b:b + 1], k[b:b + 1], v[b:b + 1], causal=True)[0].float()
    assert (o.float() - ref).abs().max().item() <= 2e-2


@pytest.mark.parametrize("Sq,Skv", [(8, 40), (128, 300), (1, 77), (200, 1000)])
def test_flash_q_shorter_than_kv(Sq, Skv):
    g = torch.Generator(device=DEV).manual_seed(Sq * Skv)
    q = torch.randn(2, 4, Sq, 128, device=DEV, generator=g, dtype=torch.bfloat16)
    k = torch.randn(2, 4, Skv, 128, device=DEV, generator=g, dtype=torch.bfloat16)
    v = torch.randn(2, 4, Skv, 128, device=DEV, generator=g, dtype=torch.bfloat16)
    o = flash_attention_v2(q, k, v, causal=True)
    ref = attention_ref(q, k, v, causal=True).float()
    assert (o.float() - ref).abs().max().item() <= 2e-2


def test_flash_gqa_and_cache_slices():
    g = torch.Generator(device=DEV).manual_seed(9)
    B, H, Hkv, S, Smax = 2, 8, 2, 300, 512
    kc = torch.randn(4, Hkv, Smax, 128, device=DEV, generator=g, dtype=torch.bfloat16)
    vc = torch.randn(4, Hkv, Smax, 128, device=DEV, generator=g, dtype=torch.bfloat16)
    q = torch.randn(B, H, S, 128, device=DEV, generator=g, dtype=torch.bfloat16)
    k, v = kc[:B, :, :S], vc[:B, :, :S]
    o = flash_attention_v2(q, k, v, causal=True)
    ref = attention_ref(q, k.contiguous(), v.contiguous(), causal=True).float()
    assert (o.float() - ref).abs().max().item() <= 2e-2


def test_flash_api_errors():
    q = torch.randn(1, 2, 8, 128, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="Q_LEN cannot exceed KV_LEN"):
        flash_attention_v2(q, q[:, :, :4], q[:, :, :4])
    with pytest.raises(TypeError):
        flash_attention_v2(q.float(), q.float(), q.float())
    with pytest.raises(ValueError):
        flash_attention_v2(q.cpu(), q.cpu(), q.cpu())


@pytest.mark.parametrize("G", [1, 4])
def test_decode_ragged_small(G):
    g = torch.Generator().manual_seed(G)
    B, Hkv, Smax, D = 6, 2, 700, 128
    H = Hkv * G
    lens = torch.tensor([1, 2, 255, 256, 257, 700], dtype=torch.int32)
    kc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, Smax, D, generator=g).to(torch.bfloat16)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
    o = ops.decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), lens.to(DEV)).cpu().float()
    ref = decode_attention_ref(q, kc, vc, lens).float()
    assert (o - ref).abs().max().item() <= 2e-2


def test_decode_op_shape_ragged():
    """Decode op shape (seed 2): 64 sequences, L_i ~ U[128, 4096]; cache
    [64, 32, 4096+1, 128] ~N(0,1) bf16 up to L_i; q/k/v [64, 32, 128]; RoPE at
    position L_i, append, attend over L_i + 1 keys.  fp32 truth per sequence."""
    torch.manual_seed(2)
    B, H, D = 64, 32, 128
    L = torch.randint(128, 4097, (B,))
    Smax = 4097
    kc = torch.zeros(B, H, Smax, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    for b in range(B):
        kc[b, :, : L[b]] = torch.randn(H, int(L[b]), D).to(torch.bfloat16).to(DEV)
        vc[b, :, : L[b]] = torch.randn(H, int(L[b]), D).to(torch.bfloat16).to(DEV)
    qkv = torch.randn(B, 1, 3 * H * D).to(torch.bfloat16).to(DEV)
    cos, sin = rope_tables(D, Smax, 10000.0)
    cos, sin = cos.to(torch.bfloat16).to(DEV), sin.to(torch.bfloat16).to(DEV)
    pos = L.view(B, 1).to(DEV)
    q = ops.rope_kv_append(qkv, pos, cos, sin, kc, vc, H, H)
    # RoPE + append at this shape, bit-exact against the oracle: the rotated q
    # and the appended K/V row of every sequence (the oracle writes sequence
    # b's row into a small [B, H, B, D] cache at position b, rotating with the
    # table row of position L_b)
    qkv_c = qkv.cpu()
    kr = torch.zeros(B, H, B, D, dtype=torch.bfloat16)
    vr = torch.zeros_like(kr)
    q_ref = rope_kv_append_ref(qkv_c, torch.arange(B).view(B, 1), cos.cpu()[L], sin.cpu()[L],
                               kr, vr, H, H)
    assert torch.equal(q.cpu(), q_ref)
    idx = torch.arange(B)
    assert torch.equal(kc[idx.to(DEV), :, L.to(DEV)].cpu(), kr[idx, :, idx])
    assert torch.equal(vc[idx.to(DEV), :, L.to(DEV)].cpu(), vr[idx, :, idx])
    lens = (L + 1).to(torch.int32).to(DEV)
    o = ops.decode_attention(q.view(B, H, D), kc, vc, lens).float()
    worst = 0.0
    for b in range(B):
        n = int(L[b]) + 1
        kf, vf = kc[b, :, :n].float(), vc[b, :, :n].float()
        s = torch.einsum("hd,hnd->hn", q[b, :, 0].float(), kf) * D ** -0.5
        ref = torch.einsum("hn,hnd->hd", torch.softmax(s, -1), vf)
        worst = max(worst, (o[b] - ref).abs().max().item())
    assert worst <= 2e-2, worst


def test_decode_zero_length_gives_zeros():
    kc = torch.randn(2, 1, 300, 128, device=DEV, dtype=torch.bfloat16)
    q = torch.randn(2, 1, 128, device=DEV, dtype=torch.bfloat16)
    o = ops.decode_attention(q, kc, kc, torch.tensor([0, 3], dtype=torch.int32, device=DEV))
    assert o[0].abs().sum().item() == 0


@pytest.mark.parametrize("H,Hkv", [(8, 8), (8, 2)])
def test_decode_independent_of_workspace_contents(H, Hkv):
    """Every partial the combine step reads is written by the same call: a
    workspace full of 0xFF bytes (and a reused one) gives bit-identical
    outputs, and they match the oracle; a sequence with no keys gets zeros."""
    g = torch.Generator(device=DEV).manual_seed(H + Hkv)
    B, Smax, D = 6, 1300, 128
    lens = torch.tensor([1300, 0, 257, 256, 1, 900], dtype=torch.int32, device=DEV)
    kc = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    q = torch.randn(B, H, D, device=DEV, generator=g).to(torch.bfloat16)
    ws = ops.decode_attention_workspace(B, H, Smax, D, DEV)
    ws.fill_(255)
    o1 = ops.decode_attention(q, kc, vc, lens, workspace=ws)
    o2 = ops.decode_attention(q, kc, vc, lens, workspace=ws)
    ws.zero_()
    o3 = ops.decode_attention(q, kc, vc, lens, workspace=ws)
    assert torch.equal(o1, o2) and torch.equal(o1, o3)
    ref = decode_attention_ref(q.float().cpu(), kc.float().cpu(), vc.float().cpu(), lens.cpu(),
                               D ** -0.5)
    assert (o1.float().cpu() - ref).abs().max().item() <= 2e-2
    assert o1[1].abs().sum().item() == 0


def test_hbm_read_probe_runs_clean():
    """The read-rate probe the bench reports beside the copy peak: reads a
    256 MB buffer, returns 0 and leaves the device status clean."""
    buf = torch.zeros(256 << 20, dtype=torch.uint8, device=DEV)
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.lpc_hbm_read_probe(buf.data_ptr(), buf.numel(), st) == 0
    torch.cuda.synchronize()
    assert _lib.device_status() == 0


@pytest.mark.parametrize("B,Smax,lens", [
    # 64 x 32 (sequence, KV head) pairs, a cache of <= 1024 keys: one split
    # of up to 1024 keys per sequence, no combine launch
    (64, 1000, [1000, 0, 1, 31, 32, 33, 500, 999]),
    # 8 x 32 pairs, a 4096-key cache: 512-key splits
    (8, 4096, [4096, 4095, 513, 512, 511, 1, 0, 2000]),
])
def test_decode_split_lengths(B, Smax, lens):
    """The split length each launch picks from its grid (1024, 512 or 256
    keys): outputs against the oracle at lengths around the split and tile
    edges, zeros for an empty context (written by the split kernel when no
    combine kernel runs), the device status clean."""
    H = Hkv = 32
    D = 128
    g = torch.Generator(device=DEV).manual_seed(B)
    L = torch.tensor((lens * (B // len(lens) + 1))[:B], dtype=torch.int32)
    kc = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g).to(torch.bfloat16)
    q = torch.randn(B, H, D, device=DEV, generator=g).to(torch.bfloat16)
    o = ops.decode_attention(q, kc, vc, L.to(DEV)).float().cpu()
    ref = decode_attention_ref(q.float().cpu(), kc.float().cpu(), vc.float().cpu(), L,
                               D ** -0.5).float()
    assert (o - ref).abs().max().item() <= 2e-2
    assert o[L == 0].abs().sum().item() == 0
    assert _lib.device_status() == 0
