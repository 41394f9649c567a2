"""Folded-RMSNorm GEMM epilogues (residual+norm stats, RoPE + KV append, scaled SiLU / fp32) vs PyTorch fp32."""

from __future__ import annotations

import pytest
import torch

from conftest import mod

pytestmark = pytest.mark.gpu


def _ops():
    return mod("ops.cuda_ops").shared_ops(torch.device("cuda", 0))


def _ref_norm(h, g, eps=1e-5):
    return h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps) * g.float()


@pytest.mark.parametrize("n", [1, 5, 16, 40, 130])
def test_embed_norm_and_scaled_gemms(n):
    ops = _ops()
    H, F, V = 1024, 2048, 512
    g = torch.Generator(device="cuda").manual_seed(n)
    table = (torch.randn(V, H, device="cuda", generator=g) * 0.5).half()
    tok = torch.randint(0, V, (n,), device="cuda", generator=g, dtype=torch.int32)
    h, hb, ss = ops.embed_norm(tok, table)
    ref_h = table[tok.long()].float()
    torch.testing.assert_close(h, ref_h)
    torch.testing.assert_close(ss, ref_h.pow(2).reshape(n, H // 128, 128).sum(-1).t(), rtol=1e-5, atol=1e-4)
    llama = mod("models.llama")
    gate = torch.randn(F, H, device="cuda", generator=g) * 0.03
    up = torch.randn(F, H, device="cuda", generator=g) * 0.03
    wgu = llama.interleave_gate_up(gate, up).half()
    act = ops.gate_up_silu_norm(hb, wgu, ss, 1e-5)
    x = _ref_norm(ref_h, torch.ones(H, device="cuda")).half().float()
    ref = torch.nn.functional.silu(x @ gate.half().float().t()) * (x @ up.half().float().t())
    torch.testing.assert_close(act.float(), ref, rtol=2e-2, atol=2e-2)
    lm = (torch.randn(V, H, device="cuda", generator=g) * 0.03).half()
    logits = ops.lm_head_norm(hb, lm, ss, 1e-5)
    torch.testing.assert_close(logits, x @ lm.float().t(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("n", [1, 12, 33])
def test_residual_norm_epilogue(n):
    ops = _ops()
    H, K = 1024, 2048
    g = torch.Generator(device="cuda").manual_seed(7 + n)
    w = (torch.randn(H, K, device="cuda", generator=g) * 0.02).half()
    x = torch.randn(n, K, device="cuda", generator=g).half()
    h = torch.randn(n, H, device="cuda", generator=g)
    h0 = h.clone()
    hb = torch.empty(n, H, device="cuda", dtype=torch.half)
    ss = torch.empty(H // 128, n, device="cuda")
    ops.linear_residual_norm(x, w, h, hb, ss)
    ops.check()
    ref = h0 + x.float() @ w.float().t()
    torch.testing.assert_close(h, ref, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(hb, ref.half(), rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(ss, ref.pow(2).reshape(n, H // 128, 128).sum(-1).t(), rtol=1e-3, atol=1e-2)


@pytest.mark.parametrize("n", [1, 9, 40])
def test_qkv_rope_epilogue(n):
    ops = _ops()
    llama = mod("models.llama")
    cfg = llama.LlamaConfig("t", 1, 512, 8, 2, 128, 1024, 4096)
    H, hq, hkv = 512, 8, 2
    g = torch.Generator(device="cuda").manual_seed(11 + n)
    hres = torch.randn(n, H, device="cuda", generator=g)
    hb = hres.half()
    ss = hres.pow(2).reshape(n, H // 128, 128).sum(-1).t().contiguous()
    wqkv = (torch.randn(cfg.qkv_size, H, device="cuda", generator=g) * 0.05).half()
    table = llama.rope_table(cfg, 256, device="cuda")
    pos = torch.randint(0, 256, (n,), device="cuda", generator=g, dtype=torch.int32)
    ps, pages = 16, 8
    slots = torch.randperm(pages * ps, device="cuda", generator=g)[:n].to(torch.int32)
    kv = torch.zeros(pages, 2, hkv, ps, 128, device="cuda", dtype=torch.half)
    q = ops.qkv_rope(hb, wqkv, ss, 1e-5, table, pos, slots, kv, hq, hkv)
    ops.check()
    x = _ref_norm(hb.float(), torch.ones(H, device="cuda"))
    qkv = (x * 1.0) @ wqkv.float().t()
    # the kernel scales the product of the unnormalized hb by rstd; same math
    qr = llama.apply_rope(qkv[:, :hq * 128].reshape(n, hq, 128), table, pos)
    kr = llama.apply_rope(qkv[:, hq * 128:(hq + hkv) * 128].reshape(n, hkv, 128), table, pos)
    vr = qkv[:, (hq + hkv) * 128:].reshape(n, hkv, 128)
    torch.testing.assert_close(q.float(), qr, rtol=2e-2, atol=2e-2)
    pg, off = (slots // ps).long(), (slots % ps).long()
    torch.testing.assert_close(kv[pg, 0, :, off].float(), kr, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(kv[pg, 1, :, off].float(), vr, rtol=2e-2, atol=2e-2)


def test_engine_with_nonunit_norm_gains_matches_reference():
    llama = mod("models.llama")
    engine = mod("runtime.engine")
    cfg = llama.get_config("small-target")
    w = llama.random_weights(cfg, seed=3, dtype=torch.float16, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(0)
    for lw in w.layers:
        lw.attn_norm.copy_((torch.rand(cfg.hidden_size, device="cuda", generator=g) + 0.5).half())
        lw.mlp_norm.copy_((torch.rand(cfg.hidden_size, device="cuda", generator=g) + 0.5).half())
    w.final_norm.copy_((torch.rand(cfg.hidden_size, device="cuda", generator=g) + 0.5).half())
    toks = list(range(100, 150))
    ref = llama.reference_forward(w, toks)
    e = engine.LlamaEngine(w, num_pages=32, page_size=16, max_positions=256)
    assert e.fused_norm
    out = e.prefill_sequence(torch.tensor(toks, dtype=torch.int32, device="cuda"), start_pos=0,
                             slots=torch.arange(50, dtype=torch.int32, device="cuda"),
                             pages=torch.arange(4, dtype=torch.int32, device="cuda"), chunk_size=64)
    e.ops.check()
    torch.testing.assert_close(out, ref[-1], rtol=3e-2, atol=3e-2)
