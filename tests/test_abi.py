"""C-ABI library: builds, loads without a GPU, exports every declared symbol,
and rejects bad arguments on the host (no kernel is launched in these tests)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from llama_pure_compute_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "lpc_b200.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"LPC_API\s+[\w\s\*]+?\b(lpc_\w+)\s*\(", text)))


def test_header_declares_all_bound_symbols():
    assert set(declared()) == set(_lib.exported_symbols())


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\bT (lpc_\w+)", out))
    for name in declared():
        assert name in exported, name
        assert getattr(lib, name) is not None


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.lpc_version() >= 100
    assert isinstance(lib.lpc_last_error(), bytes)


def test_host_validation_without_gpu():
    lib = _lib.load()
    # negative sizes / bad eps are rejected before any CUDA call
    assert lib.lpc_rmsnorm_forward(None, None, None, -1, 16, 1e-5, 2, 2, None) == _lib.LPC_ERR_INVALID
    assert b"invalid sizes" in lib.lpc_last_error()
    assert lib.lpc_rmsnorm_forward(None, None, None, 4, 16, 0.0, 2, 2, None) == _lib.LPC_ERR_INVALID
    assert lib.lpc_rmsswiglu_forward(None, None, None, None, None, None, 0, 4, 64, 64, -1.0, 2, 2,
                                     None) == _lib.LPC_ERR_INVALID
    assert b"eps must be strictly positive" in lib.lpc_last_error()
    assert lib.lpc_update_kv_cache(None, None, None, None, None, 4, 64, 1, 64, 1, 8, 3,
                                   None) == _lib.LPC_ERR_UNSUPPORTED
    assert lib.lpc_flash_attention(None, None, None, None, 1, 2, 2, 8, 4, 128, 0, 0, 1, 1.0, 2,
                                   None) == _lib.LPC_ERR_INVALID
    assert b"Q_LEN cannot exceed KV_LEN" in lib.lpc_last_error()
    assert lib.lpc_decode_attention(None, None, None, None, None, None, 0, 2, 3, 2, 128, 4, 64, 1.0,
                                    2, None) == _lib.LPC_ERR_INVALID
    # packed decode GEMM / fused q/k/v projection: sizes, layouts, dtypes, head_dim
    assert lib.lpc_packed_weight_bytes(300, 100, 0) == 0          # k not a multiple of 64
    assert lib.lpc_packed_weight_bytes(200, 128, 2) == 0          # heads layout: whole heads only
    assert lib.lpc_packed_weight_bytes(256, 128, 2) == 2 * 2 * 16384
    assert lib.lpc_pack_weights(None, None, None, None, 128, 64, 3, 2, None) == _lib.LPC_ERR_INVALID
    assert lib.lpc_wsgemm(None, None, None, None, 257, 128, 64, 0, 2, 0.0, None) == _lib.LPC_ERR_INVALID
    assert lib.lpc_wsgemm(None, None, None, None, 8, 128, 64, 1, 2, 0.0, None) == _lib.LPC_ERR_INVALID
    assert b"residual needs resid" in lib.lpc_last_error()
    qkv = lib.lpc_qkv_rope_append
    # head_dim other than 128
    assert qkv(None, None, None, None, None, 64, None, None, None, None, None, 2, 1, 4, 4, 64, 256,
               2, 64, 0, 2, 2, 0.0, None) == _lib.LPC_ERR_UNSUPPORTED
    # cos/sin tables in another dtype than the data
    assert qkv(None, None, None, None, None, 64, None, None, None, None, None, 2, 1, 4, 4, 128, 256,
               2, 64, 0, 2, 0, 0.0, None) == _lib.LPC_ERR_UNSUPPORTED
    # more than 256 tokens
    assert qkv(None, None, None, None, None, 64, None, None, None, None, None, 300, 1, 4, 4, 128, 256,
               300, 64, 0, 2, 2, 0.0, None) == _lib.LPC_ERR_INVALID
    # dense cache smaller than the batch
    assert qkv(None, None, None, None, None, 64, None, None, None, None, None, 4, 1, 4, 4, 128, 256,
               2, 64, 0, 2, 2, 0.0, None) == _lib.LPC_ERR_INVALID
    assert b"max_batch" in lib.lpc_last_error()
    # zero-sized work is a no-op
    assert lib.lpc_update_kv_cache(None, None, None, None, None, 0, 64, 1, 64, 1, 8, 2, None) == 0


def test_workspace_queries():
    lib = _lib.load()
    assert lib.lpc_rmsswiglu_workspace_bytes(256, 4096, 2) == 256 * 4096 * 2
    assert lib.lpc_rmsswiglu_workspace_bytes(8, 4096, 0) == 0
    n = lib.lpc_decode_attention_workspace_bytes(64, 32, 4097, 128)
    assert n == 64 * 32 * 17 * 130 * 4


def test_decode_split_keys_rule():
    """The split length decode attention picks from its grid (host only):
    1024 keys from 2048 (sequence, KV head) pairs up or when whole 1024-key
    splits of the capacity give 2048 CTAs, 512 when whole 512-key splits do,
    else 256; the launch count follows (one kernel when a split covers the
    cache length)."""
    lib = _lib.load()
    sk = lib.lpc_decode_attention_split_keys
    assert sk(256, 32, 616, 0) == 1024 and sk(64, 32, 616, 0) == 1024   # 8192 / 2048 pairs
    assert sk(32, 32, 616, 0) == 256 and sk(16, 32, 616, 0) == 256     # 608 / 1216 CTAs at 1024 / 512
    assert sk(32, 32, 1064, 0) == 512                                  # 32 x 66 whole 512-key splits
    assert sk(8, 32, 4096, 0) == 512 and sk(4, 32, 8232, 0) == 512     # 32 x 64 whole 512-key splits
    assert sk(8, 32, 8232, 0) == 1024 and sk(16, 32, 8192, 0) == 1024  # 32 x 64 / 128 whole 1024
    assert sk(1, 32, 4096, 0) == 256
    # ragged: the rows per KV head stand for the capacity, not batch * max_seq_len
    assert sk(8, 32, 8448, 39000) == 512 and sk(8, 32, 8448, 66000) == 1024
    assert sk(0, 32, 600, 0) == 0 and sk(4, 0, 600, 0) == 0 and sk(4, 32, 0, 0) == 0
    assert _lib.decode_kernels(256, 32, 616) == 1 and _lib.decode_kernels(256, 32, 1025) == 2
    assert _lib.decode_kernels(32, 32, 616) == 2 and _lib.decode_kernels(0, 32, 616) == 0


def test_decode_split_keys_override():
    """LPC_DECODE_CHUNK forces the split length (read once per process, so
    each case runs in a fresh interpreter); values that are not a multiple of
    32 in [256, 65536] are ignored."""
    import os
    import sys
    code = ("from llama_pure_compute_b200 import _lib; "
            "print(_lib.load().lpc_decode_attention_split_keys(256, 32, 616, 0))")
    for forced, want in (("512", 512), ("2048", 2048), ("300", 1024), ("128", 1024)):
        env = dict(os.environ, LPC_DECODE_CHUNK=forced)
        out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                             cwd=Path(__file__).resolve().parents[1], timeout=120)
        assert out.returncode == 0, out.stderr[-500:]
        assert int(out.stdout.strip().splitlines()[-1]) == want, forced


def test_read_probe_validates_on_the_host():
    lib = _lib.load()
    assert lib.lpc_hbm_read_probe(None, 131072, None) == _lib.LPC_ERR_INVALID
    assert lib.lpc_hbm_read_probe(16, 1000, None) == _lib.LPC_ERR_INVALID
    assert b"multiple of 131072" in lib.lpc_last_error()


def test_decode_sizes_that_would_overflow_are_rejected_on_the_host():
    """Sizes beyond the split grid (65535 splits of 256 keys, 65535 sequences)
    are refused before any size arithmetic: no wrapped, negative workspace
    size can slip past a scratch or workspace check."""
    lib = _lib.load()
    big = 2**63 - 1
    assert lib.lpc_decode_attention_workspace_bytes(1, 32, big, 128) == 0
    assert lib.lpc_decode_attention_workspace_bytes(big, 32, 4096, 128) == 0
    assert lib.lpc_decode_attention_workspace_bytes(1, 32, 65535 * 256 + 1, 128) == 0
    assert lib.lpc_decode_attention_workspace_bytes(1, 1, 65535 * 256, 128) > 0
    for b, s in ((1, big), (big, 4096), (65536, 4096), (1, 65535 * 256 + 1)):
        rc = lib.lpc_decode_attention_noalloc(None, None, None, None, None, b, 32, 32, 128, b, s,
                                              1.0, 2, None)
        assert rc == _lib.LPC_ERR_INVALID, (b, s)
        assert b"invalid sizes" in lib.lpc_last_error()
    rc = lib.lpc_decode_attention(None, None, None, None, None, None, 0, 1, 32, 32, 128, 1, big,
                                  1.0, 2, None)
    assert rc != _lib.LPC_OK


def test_error_translation():
    lib = _lib.load()
    lib.lpc_rmsnorm_forward(None, None, None, -1, 16, 1e-5, 2, 2, None)
    with pytest.raises(ValueError):
        _lib.check(_lib.LPC_ERR_INVALID, "x")
    with pytest.raises(TypeError):
        _lib.check(_lib.LPC_ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.LPC_ERR_CUDA, "x")


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(_lib.BackendUnavailable):
        _lib.load(tmp_path / "nope.so")


def test_ops_refuse_cpu_tensors():
    import torch
    from llama_pure_compute_b200 import ops
    q = torch.zeros(1, 2, 128)
    with pytest.raises(ValueError, match="must be on CUDA device"):
        ops.rope_forward(q, q, torch.zeros(4, 64), torch.zeros(4, 64))
    with pytest.raises(ValueError):
        ops.rmsswiglu_forward(torch.zeros(2, 64), torch.ones(64), torch.zeros(64, 64),
                              torch.zeros(64, 64))
    with pytest.raises(ValueError, match="must be on CUDA device"):
        ops.qkv_rope_append(torch.zeros(1, 1, 64), None, torch.zeros(1, 1, dtype=torch.long),
                            torch.zeros(4, 128), torch.zeros(4, 128), torch.zeros(1, 1, 4, 128),
                            torch.zeros(1, 1, 4, 128), 1, 1)
