"""Generates the golden vectors in this directory by running the REFERENCE
implementation (Llama_Pure_Compute, Python/PyTorch CPU path) on seeded inputs.

Run where the reference source tree is present (not on GPU boxes):

    python tests/golden/make_golden.py [--ref /root/reference]

The reference package does not import as shipped (merge-conflict markers in
triton_kernels/flash_attention.py); the shim below registers a bare package
object pointing at the reference sources plus an empty flash-attention module,
so ops.py, rmsnorm.py, model.py and the reference tests' own inline reference
functions import and run on the CPU.  Nothing from the reference is copied:
this script only calls it and stores inputs/outputs.

Fixtures written (torch.save dicts of small tensors):
  rope.pt       ops._rope_forward_pytorch (ops.py:27-42) with model tables, and the
                half-table convention of tests/test_rope_correctness.py:6-63
  rmsnorm.pt    triton_kernels/rmsnorm.py:88-96 (_rmsnorm_pytorch_fallback)
  rmsswiglu.pt  ops._rmsswiglu_forward_pytorch (ops.py:45-59), fp32 and the
                fp32-upcast ground truth of tests/test_rmsswiglu_correctness.py:35-54
  kv_cache.pt   ops._update_kv_cache_pytorch (ops.py:62-91) on a flat slot-major
                cache, with the slots of tests/test_kv_cache.py:85-118
  attention.pt  reference_attention (tests/test_attention_correctness.py:10-76)
  model.pt      LlamaForCausalLM (model.py:408-477) greedy tokens, full recompute
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle.model_ref import make_state_dict  # noqa: E402

MODEL_CFGS = {
    "mha": dict(vocab_size=512, dim=256, inter_dim=512, num_layers=2, num_heads=2, num_kv_heads=2,
                max_seq_len=64, rms_norm_eps=1e-5, rope_theta=10000.0),
    "gqa": dict(vocab_size=384, dim=512, inter_dim=768, num_layers=2, num_heads=4, num_kv_heads=2,
                max_seq_len=64, rms_norm_eps=1e-5, rope_theta=10000.0),
}
MODEL_SEED = 1234


def install_shim(ref_root: Path):
    src = ref_root / "src" / "llama_pure_compute"
    pkg = types.ModuleType("llama_pure_compute")
    pkg.__path__ = [str(src)]
    sys.modules["llama_pure_compute"] = pkg
    tk = types.ModuleType("llama_pure_compute.triton_kernels")
    tk.__path__ = [str(src / "triton_kernels")]
    sys.modules["llama_pure_compute.triton_kernels"] = tk
    fa = types.ModuleType("llama_pure_compute.triton_kernels.flash_attention")
    fa.flash_attention_v2 = None  # model.py:17-25 then uses SDPA
    sys.modules["llama_pure_compute.triton_kernels.flash_attention"] = fa


def load_test_module(ref_root: Path, name: str):
    path = ref_root / "tests" / f"{name}.py"
    spec = importlib.util.spec_from_file_location(f"_ref_tests_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def gen_rope(ops, model_mod, ref_tests):
    g = torch.Generator().manual_seed(11)
    out = {}
    B, S, H, Hkv, D = 2, 4, 4, 2, 128
    cos_t, sin_t = model_mod.precompute_freqs_cis(D, 64, theta=10000.0)
    pos = torch.randint(0, 64, (B, S), generator=g)
    for name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16), ("f16", torch.float16)):
        q = torch.randn(B, S, H, D, generator=g).to(dt)
        k = torch.randn(B, S, Hkv, D, generator=g).to(dt)
        c = cos_t.to(dt)[pos].unsqueeze(2)
        s = sin_t.to(dt)[pos].unsqueeze(2)
        qo, ko = ops._rope_forward_pytorch(q, k, c, s, pos)
        out[f"model_{name}"] = dict(q=q, k=k, cos=c, sin=s, pos=pos, q_out=qo, k_out=ko)
    # half-table convention of the reference CUDA kernel and its test
    cos_h, sin_h = ref_tests.generate_rope_freqs(128, D, device="cpu")
    pid = torch.randint(0, 128, (B, S), generator=g)
    q = torch.randn(B, S, H, D, generator=g)
    k = torch.randn(B, S, Hkv, D, generator=g)
    qo, ko = ref_tests.reference_rope(q, k, cos_h, sin_h, position_ids=pid)
    out["half_f32"] = dict(q=q, k=k, cos=cos_h, sin=sin_h, pos=pid, q_out=qo, k_out=ko)
    return out


def gen_rmsnorm(rms_mod):
    g = torch.Generator().manual_seed(12)
    out = {}
    for name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        x = (torch.randn(4, 256, generator=g) * 3).to(dt)
        w = (1 + 0.02 * torch.randn(256, generator=g)).to(dt)
        out[name] = dict(x=x, w=w, eps=1e-5, y=rms_mod._rmsnorm_pytorch_fallback(x, w, 1e-5))
    return out


def gen_rmsswiglu(ops, ref_tests):
    g = torch.Generator().manual_seed(13)
    out = {}
    x = torch.randn(3, 256, generator=g)
    w = 1 + 0.02 * torch.randn(256, generator=g)
    gw = 0.02 * torch.randn(192, 256, generator=g)
    uw = 0.02 * torch.randn(192, 256, generator=g)
    out["f32"] = dict(x=x, w=w, gate=gw, up=uw, eps=1e-6,
                      y=ops._rmsswiglu_forward_pytorch(x, w, gw, uw, 1e-6))
    xb, wb, gb, ub = (t.to(torch.bfloat16) for t in (x, w, gw, uw))
    out["bf16"] = dict(x=xb, w=wb, gate=gb, up=ub, eps=1e-6,
                       y=ref_tests.torch_rms_swiglu_fused(xb, wb, gb, ub, eps=1e-6))
    return out


def gen_kv(ops):
    g = torch.Generator().manual_seed(14)
    Bmax, Smax, H, D = 4, 16, 2, 64
    slots = torch.tensor([12, 45, -1, 3, 63, 16], dtype=torch.int64)
    k = torch.randn(len(slots), H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(len(slots), H, D, generator=g).to(torch.bfloat16)
    # flat slot-major cache [Bmax*Smax, H, D]: the layout the fallback indexes correctly
    kf = torch.zeros(Bmax * Smax, H, D, dtype=torch.bfloat16)
    vf = torch.zeros(Bmax * Smax, H, D, dtype=torch.bfloat16)
    ops._update_kv_cache_pytorch(k, v, kf, vf, slots)
    kc = kf.view(Bmax, Smax, H, D).permute(0, 2, 1, 3).contiguous()
    vc = vf.view(Bmax, Smax, H, D).permute(0, 2, 1, 3).contiguous()
    return dict(k_src=k, v_src=v, slots=slots, k_cache=kc, v_cache=vc, max_batch=Bmax, max_seq=Smax)


def gen_attention(att_tests):
    g = torch.Generator().manual_seed(15)
    out = {}
    cases = {"prefill_causal": (1, 2, 40, 40, True), "chunk_causal": (1, 2, 8, 40, True),
             "decode": (2, 2, 1, 40, True), "prefill_full": (1, 2, 24, 24, False)}
    for name, (B, H, Sq, Skv, causal) in cases.items():
        q = torch.randn(B, H, Sq, 128, generator=g).to(torch.bfloat16).float()
        k = torch.randn(B, H, Skv, 128, generator=g).to(torch.bfloat16).float()
        v = torch.randn(B, H, Skv, 128, generator=g).to(torch.bfloat16).float()
        o = att_tests.reference_attention(q, k, v, causal=causal, sm_scale=128 ** -0.5)
        out[name] = dict(q=q, k=k, v=v, causal=causal, out=o)
    return out


def gen_model(model_mod, config_mod):
    out = {}
    for name, cfgd in MODEL_CFGS.items():
        cfg = config_mod.LlamaModelConfig(**cfgd)
        model = model_mod.LlamaForCausalLM(cfg).float().eval()
        sd = make_state_dict(cfgd, MODEL_SEED)
        missing, unexpected = model.load_state_dict(sd, strict=False)
        assert not missing and not unexpected, (missing, unexpected)
        g = torch.Generator().manual_seed(16)
        prompt = torch.randint(0, cfgd["vocab_size"], (2, 12), generator=g)
        toks = prompt.clone()
        steps = 10
        with torch.no_grad():
            for _ in range(steps):
                logits = model(toks)  # full recompute, model-built causal mask
                nxt = logits[:, -1].argmax(-1, keepdim=True)
                toks = torch.cat([toks, nxt], 1)
            last = model(toks[:, :-1])[:, -1]
        out[name] = dict(cfg=cfgd, seed=MODEL_SEED, prompt=prompt, tokens=toks[:, 12:],
                         last_logits=last,
                         weight_checksum=float(sum(v.double().sum() for v in sd.values())))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    args = ap.parse_args()
    ref = Path(args.ref)
    install_shim(ref)
    from llama_pure_compute import config as config_mod
    from llama_pure_compute import model as model_mod
    from llama_pure_compute import ops
    from llama_pure_compute.triton_kernels import rmsnorm as rms_mod

    rope_tests = load_test_module(ref, "test_rope_correctness")
    swiglu_tests = load_test_module(ref, "test_rmsswiglu_correctness")
    att_tests = load_test_module(ref, "test_attention_correctness")

    torch.save(gen_rope(ops, model_mod, rope_tests), HERE / "rope.pt")
    torch.save(gen_rmsnorm(rms_mod), HERE / "rmsnorm.pt")
    torch.save(gen_rmsswiglu(ops, swiglu_tests), HERE / "rmsswiglu.pt")
    torch.save(gen_kv(ops), HERE / "kv_cache.pt")
    torch.save(gen_attention(att_tests), HERE / "attention.pt")
    torch.save(gen_model(model_mod, config_mod), HERE / "model.pt")
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
