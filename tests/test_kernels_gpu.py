"""Numerics of every sm_100a kernel against the PyTorch fp32 reference of the same op."""

from __future__ import annotations

import math

import pytest
import torch

from conftest import mod

pytestmark = pytest.mark.gpu

DT = [torch.float16, torch.bfloat16]


@pytest.fixture(scope="module")
def ops():
    cuda_ops = mod("ops.cuda_ops")
    return cuda_ops.CudaOps(device=torch.device("cuda"))


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("m,k,n", [(256, 128, 3), (6144, 4096, 12), (4096, 14336, 9), (1024, 2048, 1),
                                   (512, 512, 300), (384, 1024, 64), (2048, 4096, 33)])
def test_gemm_store(ops, dtype, m, k, n):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    w = (torch.randn(m, k, device="cuda", generator=g) * 0.05).to(dtype)
    x = torch.randn(n, k, device="cuda", generator=g).to(dtype)
    out = ops.linear(x, w)
    ref = x.float() @ w.float().t()
    torch.cuda.synchronize()
    ops.check()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("m,k,n", [(4096, 4096, 5), (2048, 8192, 48), (1024, 256, 200)])
def test_gemm_residual_and_f32(ops, dtype, m, k, n):
    g = torch.Generator(device="cuda").manual_seed(n)
    w = (torch.randn(m, k, device="cuda", generator=g) * 0.05).to(dtype)
    x = torch.randn(n, k, device="cuda", generator=g).to(dtype)
    resid = torch.randn(n, m, device="cuda", generator=g)
    ref = resid + x.float() @ w.float().t()
    out = ops.linear_residual(x, w, resid.clone())
    logits = ops.lm_head(x, w)
    torch.cuda.synchronize()
    ops.check()
    assert rel_err(out, ref) < 1e-2
    assert rel_err(logits, x.float() @ w.float().t()) < 1e-2


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("f,k,n", [(1024, 512, 4), (14336, 4096, 12), (512, 256, 270)])
def test_gemm_silu(ops, dtype, f, k, n):
    torch_ops = mod("ops.torch_ops")
    g = torch.Generator(device="cuda").manual_seed(f)
    wgu = (torch.randn(2 * f, k, device="cuda", generator=g) * 0.05).to(dtype)
    x = torch.randn(n, k, device="cuda", generator=g).to(dtype)
    out = ops.gate_up_silu(x, wgu)
    ref = torch_ops.gate_up_silu(x.float(), wgu.float())
    torch.cuda.synchronize()
    ops.check()
    assert rel_err(out, ref) < 1e-2


def test_gemm_deterministic_across_batch(ops):
    """A row's result does not depend on the other rows of the batch (same tile bucket)."""
    g = torch.Generator(device="cuda").manual_seed(3)
    w = (torch.randn(4096, 4096, device="cuda", generator=g) * 0.05).half()
    x = torch.randn(12, 4096, device="cuda", generator=g).half()
    full = ops.linear(x, w)
    one = ops.linear(x[5:6].contiguous(), w)
    torch.cuda.synchronize()
    assert torch.equal(full[5:6], one)


@pytest.mark.parametrize("dtype", DT)
def test_rmsnorm_embed(ops, dtype):
    torch_ops = mod("ops.torch_ops")
    g = torch.Generator(device="cuda").manual_seed(1)
    table = torch.randn(1000, 4096, device="cuda", generator=g).to(dtype)
    tok = torch.tensor([3, 999, 0, 17], dtype=torch.int32, device="cuda")
    h = ops.embed(tok, table)
    assert torch.equal(h, table[tok.long()].float())
    w = torch.rand(4096, device="cuda", generator=g).to(dtype)
    out = ops.rmsnorm(h, w, 1e-5, dtype)
    ref = torch_ops.rmsnorm(h, w, 1e-5, torch.float32)
    assert rel_err(out, ref) < 5e-3


def _paged_setup(dtype, *, pages=64, layers=2, hkv=2, ps=16, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kv = torch.randn(layers, pages, 2, hkv, ps, 128, device="cuda", generator=g).to(dtype)
    return kv, g


@pytest.mark.parametrize("dtype", DT)
def test_rope_append(ops, dtype):
    torch_ops = mod("ops.torch_ops")
    llama = mod("models.llama")
    cfg = llama.get_config("llama-8b")
    table = llama.rope_table(cfg, 4096, device="cuda")
    kv, g = _paged_setup(dtype)
    hq, hkv = 8, 2
    qkv = torch.randn(5, (hq + 2 * hkv) * 128, device="cuda", generator=g).to(dtype)
    pos = torch.tensor([0, 7, 100, 1000, 4095], dtype=torch.int32, device="cuda")
    slots = torch.tensor([3, 17, 40, 200, 1023], dtype=torch.int32, device="cuda")
    kv_ref = kv.clone()
    q = ops.rope_qkv_append(qkv, table, pos, slots, kv[1], hq, hkv)
    q_ref = torch_ops.rope_qkv_append(qkv.float(), table, pos, slots, kv_ref[1], hq, hkv)
    torch.cuda.synchronize()
    ops.check()
    assert rel_err(q, q_ref) < 5e-3
    assert rel_err(kv, kv_ref) < 5e-3


def _drafter_desc(prefix_pages, shared_len, tails, lens, ps):
    attn_desc = mod("ops.attn_desc")
    m = lens.numel()
    return attn_desc.AttnDesc(
        prefix_pages=prefix_pages,
        n_shared_pages=shared_len // ps,
        shared_len=shared_len,
        mask_base=shared_len,
        row_full=lens,
        row_len=lens,
        row_mask=torch.full((m, 1), -1, dtype=torch.int64, device="cuda"),
        tail_pages=tails,
    )


@pytest.fixture(params=[True, False], ids=["fused_merge", "two_kernels"])
def merge_path(request, ops):
    """Run an attention test with the splits merged inside the kernel (clusters) and with the separate merge kernel."""
    old = ops.fused_merge
    ops.fused_merge = request.param
    yield request.param
    ops.fused_merge = old


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("shared_len", [0, 5, 37, 300, 999])
def test_attention_drafter_rows(ops, merge_path, dtype, shared_len):
    """Rows share the prefix pages; each row has private tail pages after it."""
    torch_ops = mod("ops.torch_ops")
    engine_mod = mod("runtime.engine")
    ps, hkv, hq = 16, 2, 8
    kv, g = _paged_setup(dtype, pages=128, hkv=hkv)
    ops.engine = type("E", (), {"kv": kv})()
    n_pf = shared_len // ps
    prefix_pages = torch.randperm(100, generator=torch.Generator().manual_seed(1))[: n_pf + 1].to(torch.int32).cuda()
    m = 9
    tails = torch.arange(100, 100 + 2 * m, dtype=torch.int32, device="cuda").reshape(m, 2)
    lens = torch.tensor([shared_len + 1 + (i % 5) for i in range(m)], dtype=torch.int32, device="cuda")
    desc = _drafter_desc(prefix_pages, shared_len, tails, lens, ps)
    q = torch.randn(m, hq, 128, device="cuda", generator=g).to(dtype)
    out = ops.attention(q, kv[1], desc)
    ref = torch_ops.attention(q.float(), kv[1].float(), desc)
    torch.cuda.synchronize()
    ops.check()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("prefix,nodes", [(64, 7), (1000, 12), (4096, 48), (33, 70), (2100, 13)])
def test_attention_tree_mask(ops, merge_path, dtype, prefix, nodes):
    torch_ops = mod("ops.torch_ops")
    attn_desc = mod("ops.attn_desc")
    ps, hkv, hq = 16, 8, 32
    npages = (prefix + nodes + ps - 1) // ps
    kv, g = _paged_setup(dtype, pages=npages + 4, hkv=hkv, layers=1)
    ops.engine = type("E", (), {"kv": kv})()
    pages = torch.randperm(npages + 4, generator=torch.Generator().manual_seed(2))[:npages].to(torch.int32).cuda()
    parents = [-1] + [int(torch.randint(0, i, (1,), generator=torch.Generator().manual_seed(i)).item()) if i % 4 else -1
                      for i in range(1, nodes)]
    words = (nodes + 63) // 64
    masks = torch.zeros(nodes, words, dtype=torch.int64)
    for i in range(nodes):
        a = i
        while a >= 0:
            masks[i, a // 64] |= (1 << (a % 64)) if a % 64 < 63 else -(1 << 63)
            a = parents[a]
    lens = torch.full((nodes,), prefix + nodes, dtype=torch.int32, device="cuda")
    full = torch.full((nodes,), prefix, dtype=torch.int32, device="cuda")
    desc = attn_desc.single_sequence_desc(pages, lens, shared_len=prefix, mask_base=prefix, masks=masks.cuda(), full=full)
    q = torch.randn(nodes, hq, 128, device="cuda", generator=g).to(dtype)
    out = ops.attention(q, kv[0], desc)
    ref = torch_ops.attention(q.float(), kv[0].float(), desc)
    torch.cuda.synchronize()
    ops.check()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8, 16])
def test_attention_fused_merge_any_cluster_size(ops, splits):
    """The in-kernel merge for every cluster size up to the largest the device allows, against fp32."""
    if splits > ops.max_cluster(torch.float16):
        pytest.skip(f"this device allows clusters of at most {ops.max_cluster(torch.float16)} CTAs")
    torch_ops = mod("ops.torch_ops")
    attn_desc = mod("ops.attn_desc")
    ps, hkv, hq, prefix, nodes = 16, 8, 32, 3000, 12
    npages = (prefix + nodes + ps - 1) // ps
    kv, g = _paged_setup(torch.float16, pages=npages + 4, hkv=hkv, layers=1)
    ops.engine = type("E", (), {"kv": kv})()
    pages = torch.randperm(npages + 4, generator=torch.Generator().manual_seed(3))[:npages].to(torch.int32).cuda()
    masks = torch.tensor([[(1 << (i + 1)) - 1] for i in range(nodes)], dtype=torch.int64)
    lens = torch.full((nodes,), prefix + nodes, dtype=torch.int32, device="cuda")
    full = torch.full((nodes,), prefix, dtype=torch.int32, device="cuda")
    desc = attn_desc.single_sequence_desc(pages, lens, shared_len=prefix, mask_base=prefix, masks=masks.cuda(),
                                          full=full)
    q = torch.randn(nodes, hq, 128, device="cuda", generator=g).to(torch.float16)
    old = ops.fused_merge
    ops.fused_merge = True
    try:
        out = ops.attention(q, kv[0], desc, splits=splits)
        again = ops.attention(q, kv[0], desc, splits=splits)
    finally:
        ops.fused_merge = old
    ref = torch_ops.attention(q.float(), kv[0].float(), desc)
    torch.cuda.synchronize()
    ops.check()
    assert rel_err(out, ref) < 1e-2
    assert torch.equal(out, again)  # split order is fixed: the merge is deterministic


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("start,chunk", [(0, 40), (48, 300), (512, 17)])
def test_attention_causal_prefill(ops, dtype, start, chunk):
    torch_ops = mod("ops.torch_ops")
    attn_desc = mod("ops.attn_desc")
    ps, hkv, hq = 16, 8, 32
    total = start + chunk
    npages = (total + ps - 1) // ps
    kv, g = _paged_setup(dtype, pages=npages, hkv=hkv, layers=1)
    ops.engine = type("E", (), {"kv": kv})()
    pages = torch.arange(npages, dtype=torch.int32, device="cuda").flip(0).contiguous()
    pos = torch.arange(start, total, dtype=torch.int32, device="cuda")
    desc = attn_desc.single_sequence_desc(pages, pos + 1, shared_len=start)
    q = torch.randn(chunk, hq, 128, device="cuda", generator=g).to(dtype)
    out = ops.attention_causal(q, kv[0], desc, start)
    ref = torch_ops.attention(q.float(), kv[0].float(), desc)
    torch.cuda.synchronize()
    ops.check()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("dtype", DT)
def test_kv_copy_and_move(ops, dtype):
    torch_ops = mod("ops.torch_ops")
    kv, _ = _paged_setup(dtype, pages=32, layers=3)
    ref = kv.clone()
    plan = torch.tensor([[1, 5, 7], [2, 6, 15], [3, 7, 1]], dtype=torch.int32)
    ops.kv_copy_pages(kv, plan)
    torch_ops.kv_copy_pages(ref, plan)
    src = torch.tensor([16 * 4 + 3, 16 * 4 + 5, 16 * 9 + 1], dtype=torch.int32)
    dst = torch.tensor([16 * 4 + 1, 16 * 4 + 3, 16 * 4 + 2], dtype=torch.int32)
    ops.kv_move_slots(kv, src, dst)
    torch_ops.kv_move_slots(ref, src, dst)
    torch.cuda.synchronize()
    ops.check()
    assert torch.equal(kv, ref)


def test_topk_greedy_and_sampled(ops):
    sampling = mod("runtime.sampling")
    g = torch.Generator(device="cuda").manual_seed(5)
    logits = torch.randn(9, 128256, device="cuda", generator=g) * 3
    lp, ids = ops.topk_logprobs(logits, 4)
    rlp, rids = torch.topk(torch.log_softmax(logits, -1), 4)
    assert torch.equal(ids, rids)
    assert torch.allclose(lp, rlp, atol=1e-4)
    keys = torch.tensor([11, 2**62 + 5, 7, 8, 9, 10, 12, 13, 14], dtype=torch.int64, device="cuda")
    lp2, ids2 = ops.topk_logprobs(logits, 3, keys, 0.7)
    noise = sampling.gumbel_from_uniform(sampling.keyed_uniform(keys, logits.shape[1]))
    rids2 = torch.topk(logits / 0.7 + noise, 3).indices
    agree = (ids2 == rids2).float().mean().item()
    assert agree > 0.95
    assert torch.allclose(lp2, torch.log_softmax(logits, -1).gather(-1, ids2), atol=1e-4)


def test_gather_logprobs(ops):
    g = torch.Generator(device="cuda").manual_seed(6)
    logits = torch.randn(13, 5000, device="cuda", generator=g)
    rows = torch.tensor([0, 3, 12, 5], device="cuda")
    toks = torch.tensor([1, 4999, 0, 77], device="cuda")
    out = ops.gather_logprobs(logits, rows, toks)
    ref = torch.log_softmax(logits, -1)[rows, toks]
    assert torch.allclose(out, ref, atol=1e-4)


@pytest.mark.parametrize("dtype", DT)
def test_engine_matches_oracle(dtype):
    """A small hd-128 model: paged CUDA forward vs the fp32 oracle, prefill + tree verify."""
    llama = mod("models.llama")
    engine_mod = mod("runtime.engine")
    target_mod = mod("runtime.target")
    cfg = llama.LlamaConfig("gpu-small", 2, 512, 8, 2, 128, 1024, 4096)
    w32 = llama.random_weights(cfg, seed=3, dtype=torch.float32, device="cuda")
    w = llama.weights_to(w32, dtype=dtype)
    eng = engine_mod.LlamaEngine(w, num_pages=256, page_size=16, max_positions=2048)
    tv = target_mod.TargetVerifier(eng, k=3, d=3)
    prompt = torch.randint(0, 4096, (90,), generator=torch.Generator().manual_seed(0)).tolist()
    tv.prefill(prompt)
    ref_prefix = llama.reference_forward(llama.weights_to(w, dtype=torch.float32), prompt)[-1]
    assert rel_err(tv.prefix_logits, ref_prefix) < 3e-2
    paths = [(5, 6, 7), (5, 6, 8), (9, 6, 7)]
    out = tv.run_tree(paths)
    toks = [5, 6, 7, 8, 9, 6, 7]
    parents = [-1, 0, 1, 1, -1, 4, 5]
    depth = [0, 1, 2, 2, 0, 1, 2]
    p = len(prompt)
    t = p + 7
    vis = torch.zeros(t, t, dtype=torch.bool, device="cuda")
    vis[:p, :p] = torch.tril(torch.ones(p, p, dtype=torch.bool, device="cuda"))
    for i in range(7):
        vis[p + i, :p] = True
        a = i
        while a >= 0:
            vis[p + i, p + a] = True
            a = parents[a]
    lo = llama.reference_forward(llama.weights_to(w, dtype=torch.float32), prompt + toks,
                                 positions=list(range(p)) + [p + x for x in depth], visible=vis)[p:]
    assert rel_err(out["logits"], lo) < 3e-2
    eng.ops.check()


@pytest.mark.parametrize("rows", [3, 9, 12])
def test_graph_replay_matches_eager(rows):
    """A captured row-bucket graph gives bit-identical logits to the eager forward."""
    llama = mod("models.llama")
    engine_mod = mod("runtime.engine")
    import numpy as np

    cfg = llama.LlamaConfig("gpu-small", 2, 512, 8, 2, 128, 1024, 4096)
    w = llama.random_weights(cfg, seed=4, dtype=torch.float16, device="cuda")
    eng = engine_mod.LlamaEngine(w, num_pages=128, page_size=16, max_positions=2048)
    pages = torch.arange(100, dtype=torch.int32, device="cuda")
    g = np.random.default_rng(rows)
    fields = dict(
        tokens=g.integers(0, 4096, rows), positions=np.arange(300, 300 + rows), slots=np.arange(300, 300 + rows),
        shared_len=300, n_shared_pages=100, mask_base=300, row_full=np.full(rows, 300),
        row_len=np.full(rows, 300 + rows), row_mask=np.array([(1 << (i + 1)) - 1 for i in range(rows)])[:, None],
    )
    eng.kv.normal_()
    out_graph = [eng.run_rows(engine_mod.row_bucket(rows), prefix_pages=pages, **fields) for _ in range(2)]
    eng.use_graphs = False
    out_eager = eng.run_rows(engine_mod.row_bucket(rows), prefix_pages=pages, **fields)
    torch.cuda.synchronize()
    eng.ops.check()
    assert torch.equal(out_graph[0], out_graph[1])
    assert torch.equal(out_graph[1], out_eager)


def _causal_oracle(w, tokens, q_chunk: int = 2048) -> torch.Tensor:
    """fp32 causal forward with query-chunked attention (long contexts); returns the final hidden rows."""
    llama = mod("models.llama")
    cfg = w.config
    toks = torch.as_tensor(tokens, dtype=torch.long, device=w.device)
    t = int(toks.numel())
    pos = torch.arange(t, device=w.device)
    table = llama.rope_table(cfg, t, device=w.device)
    hd = cfg.head_dim
    x = w.embed[toks].float()
    for lw in w.layers:
        a = llama.rmsnorm_ref(x, lw.attn_norm, cfg.rms_eps)
        qkv = a @ lw.wqkv.float().t()
        q = llama.apply_rope(qkv[:, : cfg.q_size].reshape(t, cfg.num_heads, hd), table, pos)
        k = llama.apply_rope(qkv[:, cfg.q_size: cfg.q_size + cfg.kv_size].reshape(t, cfg.num_kv_heads, hd), table, pos)
        v = qkv[:, cfg.q_size + cfg.kv_size:].reshape(t, cfg.num_kv_heads, hd)
        k = k.repeat_interleave(cfg.group, dim=1).transpose(0, 1)
        v = v.repeat_interleave(cfg.group, dim=1).transpose(0, 1)
        o = torch.empty(t, cfg.num_heads, hd, device=w.device)
        for c0 in range(0, t, q_chunk):
            c1 = min(t, c0 + q_chunk)
            s = torch.einsum("qhd,hkd->hqk", q[c0:c1], k[:, :c1]) / math.sqrt(hd)
            s = s.masked_fill(torch.arange(c1, device=w.device)[None, None, :] > pos[c0:c1][None, :, None],
                              float("-inf"))
            o[c0:c1] = torch.einsum("hqk,hkd->qhd", torch.softmax(s, -1), v[:, :c1])
        x = x + o.reshape(t, cfg.q_size) @ lw.wo.float().t()
        m = llama.rmsnorm_ref(x, lw.mlp_norm, cfg.rms_eps)
        gate, up = llama.split_gate_up(lw.wgu.float())
        x = x + (torch.nn.functional.silu(m @ gate.t()) * (m @ up.t())) @ lw.wd.float().t()
    return x


@pytest.mark.parametrize("prefill_chunk", [8192, 4096])
def test_long_context_prefill_and_verify(prefill_chunk):
    """A 16K-token prompt prefilled in chunks, then a tree verified on top of it (split-KV attention path)."""
    llama = mod("models.llama")
    engine_mod = mod("runtime.engine")
    target_mod = mod("runtime.target")
    cfg = llama.LlamaConfig("gpu-small", 2, 512, 8, 2, 128, 1024, 4096)
    w32 = llama.random_weights(cfg, seed=11, dtype=torch.float32, device="cuda")
    w = llama.weights_to(w32, dtype=torch.bfloat16)
    p = 16384 + 37
    eng = engine_mod.LlamaEngine(w, num_pages=p // 16 + 64, page_size=16, max_positions=p + 64)
    tv = target_mod.TargetVerifier(eng, k=2, d=3, prefill_chunk_size=prefill_chunk)
    prompt = torch.randint(0, 4096, (p,), generator=torch.Generator().manual_seed(5)).tolist()
    tv.prefill(prompt)
    paths = [(5, 6, 7), (5, 8, 9)]
    out = tv.run_tree(paths)
    wf = llama.weights_to(w, dtype=torch.float32)
    nodes = {(5, 6, 7): [0, 1, 2], (5, 8, 9): [0, 3, 4]}
    for path in paths:
        hid = _causal_oracle(wf, prompt + list(path))[p - 1:]
        lo = llama.rmsnorm_ref(hid, wf.final_norm, cfg.rms_eps) @ wf.lm_head.float().t()
        assert rel_err(tv.prefix_logits, lo[0]) < 3e-2
        assert rel_err(out["logits"][nodes[path]], lo[1:]) < 3e-2
    eng.ops.check()


@pytest.mark.parametrize("hq,hkv", [(64, 8), (8, 8), (16, 8)])
@pytest.mark.parametrize("m", [1, 5, 40])
def test_attention_gqa_groups(ops, hq, hkv, m):
    """GQA groups other than 4 (70B: 8 query heads per kv head; MHA: 1; 2) against fp32, with
    rows past one 128-row tile when the group is large."""
    torch_ops = mod("ops.torch_ops")
    attn_desc = mod("ops.attn_desc")
    ps, prefix = 16, 700
    npages = (prefix + m + ps - 1) // ps
    kv, g = _paged_setup(torch.bfloat16, pages=npages + 2, hkv=hkv, layers=1)
    ops.engine = type("E", (), {"kv": kv})()
    pages = torch.randperm(npages + 2, generator=torch.Generator().manual_seed(7))[:npages].to(torch.int32).cuda()
    words = (m + 63) // 64
    masks = torch.zeros(m, words, dtype=torch.int64)
    for i in range(m):  # a chain: node i sees nodes 0..i
        for a in range(i + 1):
            masks[i, a // 64] |= (1 << (a % 64)) if a % 64 < 63 else -(1 << 63)
    lens = torch.full((m,), prefix + m, dtype=torch.int32, device="cuda")
    full = torch.full((m,), prefix, dtype=torch.int32, device="cuda")
    desc = attn_desc.single_sequence_desc(pages, lens, shared_len=prefix, mask_base=prefix, masks=masks.cuda(), full=full)
    q = torch.randn(m, hq, 128, device="cuda", generator=g).to(torch.bfloat16)
    out = ops.attention(q, kv[0], desc)
    ref = torch_ops.attention(q.float(), kv[0].float(), desc)
    torch.cuda.synchronize()
    ops.check()
    assert rel_err(out, ref) < 1e-2
