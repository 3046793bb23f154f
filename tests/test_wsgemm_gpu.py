"""Decode-sized projections on packed weights (lpc_pack_weights + lpc_wsgemm).

Checks:
  * packing is a pure byte permutation: bit-exact against a numpy restatement
    of the tile layout (128 rows x 64 k per 16 KB tile, 128-byte swizzle);
  * the GEMM against the fp32 product of the same bf16/fp16 inputs: within
    max(2e-2, 1 ulp) (fp32 accumulation, one rounding; accumulation order
    differs from torch's);
  * ragged n_out / token counts, residual add in place, SwiGLU from fused and
    separate gate/up weights against the rmsswiglu oracle.
"""
import numpy as np
import pytest
import torch

from llama_pure_compute_b200 import _lib
from llama_pure_compute_b200.packed_linear import PackedWeight, packed_linear
from oracle.ops_ref import rmsnorm_ref, rmsswiglu_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _clean_status():
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    assert _lib.device_status() == 0, "a kernel flagged a device-side error"


def half_ulp_bar(out, ref, dtype, msg=""):
    out, ref = out.float(), ref.float()
    mant = 7 if dtype == torch.bfloat16 else 10
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - mant)
    err = (out - ref).abs()
    bad = err > torch.maximum(torch.full_like(err, 2e-2), ulp)
    assert not bad.any(), f"{msg}: {int(bad.sum())} elements beyond max(2e-2, 1 ulp); worst {err.max().item()}"


def pack_ref(rows: np.ndarray) -> np.ndarray:
    """numpy restatement of the packed layout for a [n, k] uint16 matrix whose
    rows are already in tile order (n a multiple of 128): tile t, k-block b is
    16 KB at ((t * k/64) + b) * 16 KB; inside, row r's 16-byte chunk c sits at
    r * 128 + ((c ^ (r % 8)) * 16)."""
    n, k = rows.shape
    t = rows.reshape(n // 128, 128, k // 64, 8, 8)           # tile, row, kb, chunk, elem
    t = t.transpose(0, 2, 1, 3, 4)                          # tile, kb, row, chunk, elem
    r = np.arange(128)[:, None]
    c = np.arange(8)[None, :]
    out = np.empty_like(t)
    out[:, :, r, c ^ (r % 8), :] = t[:, :, r, c, :]
    return out.reshape(-1)


def tile_order_swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """Rows of the SwiGLU tiles: per 64 columns, 4 groups of (16 gate, 16 up)."""
    n, k = gate.shape
    n_pad = -(-n // 64) * 64
    g = np.zeros((n_pad, k), gate.dtype)
    u = np.zeros((n_pad, k), up.dtype)
    g[:n], u[:n] = gate, up
    g = g.reshape(n_pad // 16, 16, k)
    u = u.reshape(n_pad // 16, 16, k)
    return np.concatenate([g, u], axis=1).reshape(2 * n_pad, k)


def _u16(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("n,k", [(128, 64), (300, 192), (1024, 512)])
def test_pack_linear_layout_bit_exact(n, k):
    g = torch.Generator().manual_seed(n + k)
    w = torch.randn(n, k, generator=g).to(torch.bfloat16)
    pw = PackedWeight(w.to(DEV))
    n_pad = -(-n // 128) * 128
    rows = np.zeros((n_pad, k), np.uint16)
    rows[:n] = _u16(w)
    assert np.array_equal(pw.data.cpu().numpy().view(np.uint16), pack_ref(rows))


@pytest.mark.parametrize("fused", [True, False])
def test_pack_swiglu_layout_bit_exact(fused):
    g = torch.Generator().manual_seed(11)
    n, k = 200, 128
    gate = torch.randn(n, k, generator=g).to(torch.float16)
    up = torch.randn(n, k, generator=g).to(torch.float16)
    if fused:
        pw = PackedWeight(torch.cat([gate, up]).to(DEV), layout="swiglu")
    else:
        pw = PackedWeight(gate.to(DEV), up.to(DEV), layout="swiglu")
    rows = tile_order_swiglu(_u16(gate), _u16(up))
    assert np.array_equal(pw.data.cpu().numpy().view(np.uint16), pack_ref(rows))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tokens,n,k", [
    (1, 128, 64), (7, 300, 192), (16, 1024, 512), (33, 4096, 512),
    (100, 640, 4096),
    (256, 2048, 1024), (129, 96, 128), (256, 12288, 4096),
])
def test_wsgemm_store(dtype, tokens, n, k):
    g = torch.Generator().manual_seed(tokens * 7 + n)
    x = (torch.randn(tokens, k, generator=g) * 0.5).to(dtype).to(DEV)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype).to(DEV)
    pw = PackedWeight(w)
    out = packed_linear(x, pw)
    ref = x.float() @ w.float().t()
    half_ulp_bar(out, ref, dtype, f"store {tokens}x{n}x{k}")


@pytest.mark.parametrize("tokens,n,k", [(5, 4096, 4096), (64, 4096, 11008), (256, 4096, 11008),
                                        (12, 200, 320)])
def test_wsgemm_residual_in_place(tokens, n, k):
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(tokens + k)
    x = torch.randn(tokens, k, generator=g).to(dtype).to(DEV)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype).to(DEV)
    h = torch.randn(tokens, n, generator=g).to(dtype).to(DEV)
    ref = h.float() + x.float() @ w.float().t()
    pw = PackedWeight(w)
    out = packed_linear(x, pw, "residual", resid=h, out=h)
    assert out.data_ptr() == h.data_ptr()
    half_ulp_bar(h, ref, dtype, f"residual {tokens}x{n}x{k}")


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("tokens,D,I", [(1, 256, 512), (9, 512, 768), (128, 4096, 11008),
                                        (256, 4096, 11008), (40, 320, 200)])
def test_wsgemm_swiglu_matches_rmsswiglu_oracle(fused, tokens, D, I):
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(tokens + I)
    x = torch.randn(tokens, D, generator=g).to(dtype)
    rw = (1.0 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    gate = (torch.randn(I, D, generator=g) * D ** -0.5).to(dtype)
    up = (torch.randn(I, D, generator=g) * D ** -0.5).to(dtype)
    xd = x.to(DEV)
    normed = rmsnorm_ref(xd.float(), rw.to(DEV).float(), 1e-5).to(dtype)
    if fused:
        pw = PackedWeight(torch.cat([gate, up]).to(DEV), layout="swiglu")
    else:
        pw = PackedWeight(gate.to(DEV), up.to(DEV), layout="swiglu")
    out = packed_linear(normed, pw, "swiglu")
    ref = rmsswiglu_ref(xd, rw.to(DEV), gate.to(DEV), up.to(DEV), 1e-5, compute=torch.float32,
                        round_normed=True)
    half_ulp_bar(out, ref, dtype, f"swiglu {tokens}x{D}x{I}")


@pytest.mark.parametrize("splits", [2, 3, 4, 5, 7, 8])
@pytest.mark.parametrize("epilogue,tokens,n,k", [
    ("store", 32, 4096, 4096), ("residual", 64, 4096, 11008), ("store", 1, 300, 192),
    ("residual", 17, 1000, 1088), ("swiglu", 40, 320, 512), ("store", 128, 640, 4096),
    ("residual", 48, 384, 2048), ("swiglu", 80, 256, 1024), ("store", 112, 512, 960),
])
def test_wsgemm_split_k_cluster(monkeypatch, splits, epilogue, tokens, n, k):
    """Split-k clusters (partial tiles reduce-scattered through distributed
    shared memory); the split count is clamped to the k-blocks, to the shared
    memory that holds a partial tile and to a divisor of the 4-token column
    groups, so some cases run fewer splits."""
    monkeypatch.setenv("LPC_WSGEMM_SPLITS", str(splits))
    dtype = torch.bfloat16 if (splits + tokens) % 2 else torch.float16
    g = torch.Generator().manual_seed(splits * 1000 + tokens + n)
    x = (torch.randn(tokens, k, generator=g) * 0.5).to(dtype).to(DEV)
    if epilogue == "swiglu":
        gate = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype).to(DEV)
        up = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype).to(DEV)
        pw = PackedWeight(gate, up, layout="swiglu")
        out = packed_linear(x, pw, "swiglu")
        gf, uf = x.float() @ gate.float().t(), x.float() @ up.float().t()
        ref = torch.nn.functional.silu(gf) * uf
    else:
        w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype).to(DEV)
        pw = PackedWeight(w)
        ref = x.float() @ w.float().t()
        if epilogue == "residual":
            h = torch.randn(tokens, n, generator=g).to(dtype).to(DEV)
            ref = ref + h.float()
            out = packed_linear(x, pw, "residual", resid=h, out=h)
        else:
            out = packed_linear(x, pw)
    half_ulp_bar(out, ref, dtype, f"split {splits} {epilogue} {tokens}x{n}x{k}")
    if epilogue != "residual":
        again = packed_linear(x, pw, epilogue)
        assert torch.equal(out, again), "split-k reduction is not deterministic"


def test_wsgemm_errors():
    w = PackedWeight(torch.randn(128, 64, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        packed_linear(torch.randn(257, 64, device=DEV, dtype=torch.bfloat16), w)
    with pytest.raises(ValueError):
        packed_linear(torch.randn(4, 64, device=DEV, dtype=torch.bfloat16), w, "swiglu")
    with pytest.raises(ValueError):
        packed_linear(torch.randn(4, 64, device=DEV, dtype=torch.bfloat16), w, "residual")
    with pytest.raises(ValueError):
        PackedWeight(torch.randn(128, 96, device=DEV, dtype=torch.bfloat16))
    assert packed_linear(torch.empty(0, 64, device=DEV, dtype=torch.bfloat16), w).shape == (0, 128)
