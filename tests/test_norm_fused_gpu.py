"""RMSNorm fused into the decode-sized GEMMs (lpc_wsgemm / lpc_qkv_rope_append
with norm_eps > 0).

The kernel reads the raw rows x, takes each row's sum of squares from the
activation tiles the tensor core consumes, and scales the accumulators by
rsqrt(mean(x^2) + eps); the norm weight w is folded into the packed weight
(W[n, k] * w[k], one rounding).  So the fused product is
epilogue(rsqrt(mean(x^2) + eps) * (x (W diag(w))^T)) -- the same function as
the reference's norm -> projection (triton_kernels/rmsnorm.py:58-96,
ops.py:45-59, model.py:125-168), with the normalised rows never rounded to
bf16.  Checked against the fp32 oracle of the unfused composition at the
bf16 output bar (max(2e-2, 1 ulp); for the rotated q/k rows, which are
rounded twice, one ulp of the rotated pair plus one of the result) and against the two-kernel form (row norm kernel, then the
unfused GEMM) at the same bar, with split-k (the partial sums of squares cross
the cluster) and without, for every epilogue.
"""
import pytest
import torch

from llama_pure_compute_b200 import _lib, ops
from llama_pure_compute_b200.packed_linear import PackedWeight, packed_linear
from oracle.model_ref import rope_tables
from oracle.ops_ref import rmsswiglu_ref, rope_kv_append_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
EPS = 1e-5


@pytest.fixture(autouse=True)
def _clean_status():
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    assert _lib.device_status() == 0, "a kernel flagged a device-side error"


def bar(out, ref, msg="", ulps=1):
    out, ref = out.float().cpu(), ref.float().cpu()
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - 7)
    err = (out - ref).abs()
    bad = err > torch.maximum(torch.full_like(err, 2e-2), ulps * ulp)
    assert not bad.any(), (f"{msg}: {int(bad.sum())} beyond max(2e-2, {ulps} ulp); "
                           f"worst {err.max().item()}")


def _data(seed, M, n, k, n2=None):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, k, generator=g) * 1.7).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    W = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    W2 = None if n2 is None else (torch.randn(n2, k, generator=g) * 0.02).to(torch.bfloat16)
    return x, w, W, W2


@pytest.mark.parametrize("M", [1, 7, 32, 64, 128])
def test_fused_norm_swiglu(M):
    I, k = 704, 1024
    x, w, Wg, Wu = _data(M, M, I, k, I)
    pw = PackedWeight(Wg.to(DEV), Wu.to(DEV), layout="swiglu", norm_weight=w.to(DEV))
    out = packed_linear(x.to(DEV), pw, "swiglu", norm_eps=EPS)
    ref = rmsswiglu_ref(x, w, Wg, Wu, EPS)  # fp32 normed rows, fp32 GEMM
    bar(out, ref, f"fused norm + SwiGLU M={M}")
    # the two-kernel form: row norm kernel, then the GEMM on unfolded weights
    xn = ops.rmsnorm_forward(x.to(DEV), w.to(DEV), EPS)
    two = packed_linear(xn, PackedWeight(Wg.to(DEV), Wu.to(DEV), layout="swiglu"), "swiglu")
    bar(out, two, f"fused vs two-kernel M={M}")


@pytest.mark.parametrize("M,n,k", [(16, 512, 4096), (64, 512, 4096), (128, 256, 2048),
                                   (32, 4096, 1024)])
def test_fused_norm_residual_split_k(M, n, k):
    """Few weight tiles (n = 256..512): the launch splits k over a cluster and
    the ranks' partial sums of squares are added through distributed shared
    memory; n = 4096 runs one CTA per tile."""
    x, w, W, _ = _data(M + n, M, n, k)
    r = (torch.randn(M, n, generator=torch.Generator().manual_seed(3))).to(torch.bfloat16)
    pw = PackedWeight(W.to(DEV), norm_weight=w.to(DEV))
    rd = r.to(DEV)
    out = packed_linear(x.to(DEV), pw, "residual", resid=rd, out=rd, norm_eps=EPS)
    xn = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + EPS) * w.float()
    ref = r.float() + xn @ W.float().t()
    bar(out, ref, f"fused norm + residual M={M} n={n} k={k}")
    st = packed_linear(x.to(DEV), pw, "store", norm_eps=EPS)
    bar(st, xn @ W.float().t(), f"fused norm + store M={M}")


def test_fused_norm_requires_folded_weight():
    x, w, W, _ = _data(1, 8, 128, 256)
    with pytest.raises(ValueError, match="norm_weight"):
        packed_linear(x.to(DEV), PackedWeight(W.to(DEV)), "store", norm_eps=EPS)
    with pytest.raises(ValueError, match="norm_weight"):
        packed_linear(x.to(DEV), PackedWeight(W.to(DEV), norm_weight=w.to(DEV)), "store")


@pytest.mark.parametrize("B,H,Hkv", [(8, 4, 4), (40, 8, 2), (128, 4, 4)])
def test_fused_norm_qkv_rope_append(B, H, Hkv):
    """Input RMSNorm + q/k/v projection + RoPE + KV append in one kernel,
    against the oracle composition rope_kv_append(rmsnorm(x) W^T) in fp32."""
    D, k, Smax = 128, 1024, 300
    g = torch.Generator().manual_seed(B * H)
    x = (torch.randn(B, 1, k, generator=g) * 1.3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    W = (torch.randn((H + 2 * Hkv) * D, k, generator=g) * 0.03).to(torch.bfloat16)
    pos = torch.randint(0, Smax, (B, 1), generator=g)
    cos, sin = rope_tables(D, Smax, 10000.0)
    cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
    kc = torch.zeros(B, Hkv, Smax, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kd, vd = kc.to(DEV), vc.to(DEV)
    pw = PackedWeight(W.to(DEV), layout="heads", norm_weight=w.to(DEV))
    q = ops.qkv_rope_append(x.to(DEV), pw, pos.to(DEV), cos.to(DEV), sin.to(DEV), kd, vd, H, Hkv,
                            norm_eps=EPS)
    xn = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + EPS) * w.float()
    qkv = (xn @ W.float().t()).to(torch.bfloat16)
    kr, vr = kc.clone(), vc.clone()
    q_ref = rope_kv_append_ref(qkv, pos, cos, sin, kr, vr, H, Hkv)
    # q and k are rounded twice: the projection, then the rotation of a pair
    # of projected values.  Projections one ulp apart move the rotated value
    # by up to one ulp of the larger of the pair (|cos|, |sin| <= 1), plus the
    # final rounding: the bar is one ulp of the pair plus one ulp of the result.
    def ulp(t):
        return torch.exp2(torch.floor(torch.log2(t.float().abs().clamp_min(1e-30))) - 7)

    def rot_bar(out, ref, pre, what):
        pair = torch.maximum(pre.float().abs(), pre.float().roll(D // 2, dims=-1).abs())
        lim = torch.maximum(torch.full_like(pair, 2e-2), ulp(pair) + ulp(ref))
        err = (out.float().cpu() - ref.float()).abs()
        assert bool((err <= lim).all()), f"{what}: worst {err.max().item()}"

    rot_bar(q.cpu(), q_ref, qkv[..., :H * D].reshape(B, 1, H, D).transpose(1, 2), "q")
    idx = torch.arange(B)
    k_rows = kd.cpu()[idx, :, pos[:, 0]]  # [B, Hkv, D]: the appended rows
    rot_bar(k_rows, kr[idx, :, pos[:, 0]], qkv[:, 0, H * D:(H + Hkv) * D].reshape(B, Hkv, D),
            "key cache")
    bar(vd, vr, "value cache")
    # rows that were not appended stay untouched
    written = torch.zeros(B, Smax, dtype=torch.bool)
    written[torch.arange(B), pos[:, 0]] = True
    assert kd.cpu()[~written.unsqueeze(1).expand(B, Hkv, Smax)].abs().sum().item() == 0


@pytest.mark.parametrize("M", [129, 256, 300, 2048])
@pytest.mark.parametrize("fused_weight", [False, True])
def test_folded_norm_swiglu_pair(M, fused_weight):
    """lpc_rmsswiglu_folded_forward: the CTA-pair kernel with the norm inside,
    on gate/up weights that carry the norm weight, against the fp32 oracle of
    norm -> SwiGLU and against the two-kernel op (rmsswiglu_forward)."""
    I, k = 1408, 1024
    x, w, Wg, Wu = _data(M + 11, M, I, k, I)
    fg = (Wg.float() * w.float()).to(torch.bfloat16)
    fu = (Wu.float() * w.float()).to(torch.bfloat16)
    if fused_weight:
        out = ops.rmsswiglu_folded_forward(x.to(DEV), torch.cat([fg, fu]).to(DEV), None, EPS)
    else:
        out = ops.rmsswiglu_folded_forward(x.to(DEV), fg.to(DEV), fu.to(DEV), EPS)
    bar(out, rmsswiglu_ref(x, w, Wg, Wu, EPS), f"folded norm + SwiGLU M={M}")
    two = ops.rmsswiglu_forward(x.to(DEV), w.to(DEV), Wg.to(DEV), Wu.to(DEV), EPS)
    bar(out, two, f"folded vs two-kernel M={M}")
