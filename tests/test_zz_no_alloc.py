"""Allocation-free decode attention (lpc_decode_attention_noalloc).

This entry point exists for callers that cannot allocate device memory when
they run attention -- e.g. a plugin whose host application has reserved all of
HBM for itself, or a serving loop that must not call cudaMalloc mid-request.
It keeps the split partials in the library's own fixed scratch array instead
of a caller workspace.  Here it is called through the C ABI and compared with
the workspace entry point (lpc_decode_attention), two calls in a row.  Both
run the same split and combine kernels on the same inputs and differ only in
where the partials live, so the outputs must be bit-identical; the
attention-test bar (2e-2 max-abs) is kept for the check against the CPU
oracle.  The calls go from a shape with more splits to one with fewer and
different data, so a stale split left in the shared scratch would show.
This file is collected last on purpose; it must pass alone in a fresh
process too.
"""
import pytest
import torch

from llama_pure_compute_b200 import _lib
from oracle.ops_ref import decode_attention_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCRATCH_BYTES = 24 * 1024 * 1024  # LPC_NOALLOC_SCRATCH_BYTES in include/lpc_b200.h


def _inputs(seed, B, H, Hkv, Smax, D=128):
    g = torch.Generator(device=DEV).manual_seed(seed)
    kc = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g, dtype=torch.bfloat16)
    vc = torch.randn(B, Hkv, Smax, D, device=DEV, generator=g, dtype=torch.bfloat16)
    q = torch.randn(B, H, D, device=DEV, generator=g, dtype=torch.bfloat16)
    lens = torch.randint(1, Smax + 1, (B,), device=DEV, generator=g).to(torch.int32)
    lens[0] = Smax
    return q, kc, vc, lens


def _with_workspace(lib, q, kc, vc, lens, H, Hkv, Smax):
    B, D = q.shape[0], q.shape[-1]
    need = lib.lpc_decode_attention_workspace_bytes(B, H, Smax, D)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    out = torch.empty_like(q)
    rc = lib.lpc_decode_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(),
                                  out.data_ptr(), ws.data_ptr(), need, B, H, Hkv, D, B, Smax,
                                  D ** -0.5, 2, torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "decode_attention")
    return out


def _no_alloc(lib, q, kc, vc, lens, H, Hkv, Smax, out):
    B, D = q.shape[0], q.shape[-1]
    return lib.lpc_decode_attention_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                            lens.data_ptr(), out.data_ptr(), B, H, Hkv, D, B, Smax,
                                            D ** -0.5, 2, torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    lib = _lib.load()
    # first call: 16 sequences of up to 1300 keys (6 splits); second call: 5
    # sequences of up to 777 keys (4 splits), GQA, other data
    for seed, (B, H, Hkv, Smax) in ((1, (16, 8, 8, 1300)), (2, (5, 8, 2, 777))):
        q, kc, vc, lens = _inputs(seed, B, H, Hkv, Smax)
        ref = _with_workspace(lib, q, kc, vc, lens, H, Hkv, Smax)
        out = torch.full_like(q, float("nan"))
        _lib.check(_no_alloc(lib, q, kc, vc, lens, H, Hkv, Smax, out), "decode_attention_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        orc = decode_attention_ref(q.cpu(), kc.cpu(), vc.cpu(), lens.cpu(), 128 ** -0.5)
        assert (out.cpu().float() - orc.float()).abs().max().item() <= 2e-2
    assert _lib.device_status() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    B, H, Smax, D = 64, 32, 4097, 128  # 18 MB of partials fits; 4x the batch does not
    assert lib.lpc_decode_attention_workspace_bytes(B, H, Smax, D) <= SCRATCH_BYTES
    assert lib.lpc_decode_attention_workspace_bytes(4 * B, H, Smax, D) > SCRATCH_BYTES
    rc = lib.lpc_decode_attention_noalloc(None, None, None, None, None, 4 * B, H, H, D, 4 * B,
                                          Smax, 1.0, 2, None)
    assert rc == _lib.LPC_ERR_INVALID
    assert b"static scratch holds" in lib.lpc_last_error()
