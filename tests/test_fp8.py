"""Block-scaled fp8: quantizer semantics on CPU; tcgen05 fp8 GEMM and engine numerics on GPU."""

from __future__ import annotations

import pytest
import torch

from conftest import mod


def test_blockwise_quantization_round_trip():
    fp8 = mod("models.fp8")
    g = torch.Generator().manual_seed(0)
    w = torch.randn(300, 256, generator=g)
    t = fp8.quantize_blockwise(w)
    assert t.q.dtype == torch.float8_e4m3fn and t.scale.shape == (3, 2)
    # e4m3 keeps 3 mantissa bits: relative error per element below 2^-4 of the block max.
    err = (t.dequantize() - w).abs()
    bmax = w.abs().reshape(-1)[...].max()
    assert float(err.max()) <= float(bmax) * 2 ** -4
    xq, sa = fp8.quantize_activations(w[:5])
    assert sa.shape == (2, 5)
    assert float(xq.float().abs().max()) <= 448.0


def test_fp8_engine_cpu_matches_reference():
    fp8 = mod("models.fp8")
    llama = mod("models.llama")
    eng = mod("runtime.engine_fp8")
    cfg = llama.LlamaConfig("t8", 2, 256, 4, 2, 64, 512, 1024, rope_theta=10000.0, rope_scaling=None)
    w = fp8.random_weights_fp8(cfg, seed=3, dtype=torch.float32)
    toks = list(range(10, 30))
    ref = fp8.fp8_reference_forward(w, toks)
    for chunk in (64, 7):
        e = eng.Fp8LlamaEngine(w, num_pages=64, page_size=4, max_positions=64)
        out = e.prefill_sequence(torch.tensor(toks, dtype=torch.int32), start_pos=0,
                                 slots=torch.arange(20, dtype=torch.int32), pages=torch.arange(8, dtype=torch.int32),
                                 chunk_size=chunk)
        if chunk == 64:
            torch.testing.assert_close(out, ref[-1], rtol=1e-4, atol=1e-4)
        else:
            # Chunking changes fp32 summation order upstream of the per-token quantizer, which can
            # move a value across an e4m3 rounding boundary: compare at fp8 resolution.
            assert float((out - ref[-1]).abs().max()) < 0.03 * float(ref[-1].abs().max())


# ------------------------------------------------------------------ GPU
def _ops():
    return mod("ops.cuda_ops").shared_ops(torch.device("cuda", 0))


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(256, 1, 512), (384, 12, 1024), (4096, 48, 4096), (1000, 64, 2048),
                                   (8192, 9, 28672 // 4), (512, 40, 9216)])
def test_gemm_fp8_store_matches_reference(m, n, k):
    fp8 = mod("models.fp8")
    ops = _ops()
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    w = fp8.quantize_blockwise(torch.randn(m, k, device="cuda", generator=g) * 0.02)
    x = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    xq, sa = ops.quant_fp8(x)
    out = torch.empty((n, m), dtype=torch.float32, device="cuda")
    ops.gemm_fp8(xq, sa, w, out, ops.ext.EPI_F32)
    ops.check()
    # The GEMM alone: the kernel's own quantized activations, dequantized, times the weights.
    ref = fp8.dequantize_activations(xq, sa) @ w.dequantize().t()
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-4 * float(ref.abs().max()))



@pytest.mark.gpu
def test_quantizers_match_reference():
    fp8 = mod("models.fp8")
    ops = _ops()
    x = torch.randn(7, 1024, device="cuda").to(torch.bfloat16)
    xq, sa = ops.quant_fp8(x)
    rq, rs = fp8.quantize_activations(x.float())
    # Same scale up to one fp32 ulp; e4m3 codes agree except where a value sits on a rounding boundary.
    torch.testing.assert_close(sa[:, :7], rs, rtol=2.5e-7, atol=0)
    assert float((xq.view(torch.uint8) != rq.view(torch.uint8)).float().mean()) < 1e-3
    h = torch.randn(5, 1024, device="cuda")
    gamma = (torch.rand(1024, device="cuda") + 0.5).to(torch.bfloat16)
    nq, ns = ops.rmsnorm_fp8(h, gamma, 1e-5)
    xn = mod("models.llama").rmsnorm_ref(h, gamma, 1e-5)
    rq, rs = fp8.quantize_activations(xn)
    torch.testing.assert_close(ns[:, :5], rs, rtol=1e-5, atol=0)
    assert float((nq.view(torch.uint8) != rq.view(torch.uint8)).float().mean()) < 1e-2


@pytest.mark.gpu
@pytest.mark.parametrize("n", [3, 16, 40])
def test_gemm_fp8_residual_and_silu(n):
    fp8 = mod("models.fp8")
    llama = mod("models.llama")
    ops = _ops()
    k, h, f = 1024, 512, 1024
    g = torch.Generator(device="cuda").manual_seed(n)
    gate = torch.randn(f, k, device="cuda", generator=g) * 0.03
    up = torch.randn(f, k, device="cuda", generator=g) * 0.03
    wgu = fp8.quantize_blockwise(llama.interleave_gate_up(gate, up))
    x = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    xq, sa = ops.quant_fp8(x)
    act = torch.empty((n, f), dtype=torch.bfloat16, device="cuda")
    ops.gemm_fp8(xq, sa, wgu, act, ops.ext.EPI_SILU)
    gu = fp8.fp8_matmul_ref(x.float(), wgu).reshape(n, -1, 2, 64)
    ref = torch.nn.functional.silu(gu[:, :, 0].reshape(n, -1)) * gu[:, :, 1].reshape(n, -1)
    torch.testing.assert_close(act.float(), ref, rtol=2e-2, atol=2e-2 * float(ref.abs().max()))
    wd = fp8.quantize_blockwise(torch.randn(h, f, device="cuda", generator=g) * 0.03)
    resid = torch.randn(n, h, device="cuda")
    r0 = resid.clone()
    aq, sa2 = ops.quant_fp8(act)
    ops.gemm_fp8(aq, sa2, wd, resid, ops.ext.EPI_RESIDUAL)
    ops.check()
    ref2 = r0 + fp8.dequantize_activations(aq, sa2) @ wd.dequantize().t()
    torch.testing.assert_close(resid, ref2, rtol=1e-3, atol=1e-4 * float(ref2.abs().max()))


@pytest.mark.gpu
def test_fp8_engine_matches_reference_forward():
    fp8 = mod("models.fp8")
    llama = mod("models.llama")
    eng = mod("runtime.engine_fp8")
    cfg = llama.get_config("small-target")
    w = fp8.random_weights_fp8(cfg, seed=4, dtype=torch.bfloat16, device="cuda")
    toks = list(range(100, 160))
    ref = fp8.fp8_reference_forward(w, toks)
    e = eng.Fp8LlamaEngine(w, num_pages=64, page_size=16, max_positions=256)
    out = e.prefill_sequence(torch.tensor(toks, dtype=torch.int32, device="cuda"), start_pos=0,
                             slots=torch.arange(60, dtype=torch.int32, device="cuda"),
                             pages=torch.arange(4, dtype=torch.int32, device="cuda"), chunk_size=64)
    e.ops.check()
    assert float((out - ref[-1]).abs().max()) < 0.05 * float(ref[-1].abs().max()) + 1e-3
    assert int(out.argmax()) == int(ref[-1].argmax())
