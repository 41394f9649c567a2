"""PyTorch implementations of every kernel's semantics on the paged KV layout.

These run the CPU configuration (fp32 tiny models) and serve as the
per-kernel numerics reference for the CUDA kernels.  KV cache layout for all
paths: ``[layers, pages, 2 (k, v), kv_heads, page_size, head_dim]``.

Reference counterparts of the op semantics: the manual Llama layer around FlashInfer
(src/atlas_0709/flashinfer_full_verify.py:1183-1231), its suffix KV write (:1027-1044),
``topk_logprobs`` (src/atlas_0709/flashinfer_paged/utils.py:11-25) and the tail-page
copy-on-write of the route pool (src/atlas_0709/flashinfer_paged/sglang_runtime.py:708-798).
"""

from __future__ import annotations

import math

import torch

from ..models.llama import GU_BLOCK
from .attn_desc import AttnDesc


def check() -> None:
    """The CUDA op table's error-flag check; PyTorch ops raise where they fail, so there is nothing to read."""
    return None


def embed(tokens: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    return table[tokens.long()].float()


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out_dtype: torch.dtype) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(out_dtype)


def linear(x: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    y = x.float() @ w.float().t()
    return y.to(out_dtype or x.dtype)


def linear_residual(x: torch.Tensor, w: torch.Tensor, resid: torch.Tensor) -> torch.Tensor:
    return resid + x.float() @ w.float().t()


def gate_up_silu(x: torch.Tensor, wgu: torch.Tensor) -> torch.Tensor:
    y = x.float() @ wgu.float().t()  # [M, 2F] interleaved in blocks
    m = y.shape[0]
    y = y.reshape(m, -1, 2, GU_BLOCK)
    act = torch.nn.functional.silu(y[:, :, 0]) * y[:, :, 1]
    return act.reshape(m, -1).to(x.dtype)


def _slot_to_page(slots: torch.Tensor, page_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    s = slots.long()
    return s // page_size, s % page_size


def rope_qkv_append(
    qkv: torch.Tensor,
    table: torch.Tensor,
    positions: torch.Tensor,
    slots: torch.Tensor,
    kv_layer: torch.Tensor,
    num_heads: int,
    num_kv_heads: int,
) -> torch.Tensor:
    """Rotate q/k, write k and v into the paged cache at ``slots``; return rotated q [M, Hq, hd]."""
    m = qkv.shape[0]
    hd = kv_layer.shape[-1]
    ps = kv_layer.shape[-2]
    q = qkv[:, : num_heads * hd].reshape(m, num_heads, hd)
    k = qkv[:, num_heads * hd: (num_heads + num_kv_heads) * hd].reshape(m, num_kv_heads, hd)
    v = qkv[:, (num_heads + num_kv_heads) * hd:].reshape(m, num_kv_heads, hd)
    half = hd // 2
    cs = table[positions.long()]
    cos, sin = cs[:, None, :half], cs[:, None, half:]

    def rot(x: torch.Tensor) -> torch.Tensor:
        x1, x2 = x[..., :half].float(), x[..., half:].float()
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)

    qr = rot(q).to(qkv.dtype)
    kr = rot(k).to(kv_layer.dtype)
    page, off = _slot_to_page(slots, ps)
    kv_layer[page, 0, :, off] = kr
    kv_layer[page, 1, :, off] = v.to(kv_layer.dtype)
    return qr


def _row_positions(desc: AttnDesc, r: int, page_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Visible key positions of row r and their physical slots."""
    n = int(desc.row_len[r])
    pos = torch.arange(n, device=desc.row_len.device)
    full = int(desc.row_full[r])
    vis = pos < full
    if n > full:
        rel = (pos - desc.mask_base).clamp(min=0)
        words = desc.row_mask[r]
        word = words[(rel // 64).clamp(max=words.numel() - 1)]
        bit = torch.bitwise_and(torch.bitwise_right_shift(word, rel % 64), 1).bool()
        vis = vis | ((pos >= full) & bit)
    pos = pos[vis]
    j = pos // page_size
    shared = (j < desc.n_shared_pages) | (pos < desc.shared_len)
    pages = torch.empty_like(j)
    pages[shared] = desc.prefix_pages.long()[j[shared]]
    if (~shared).any():
        pages[~shared] = desc.tail_pages[r].long()[j[~shared] - desc.n_shared_pages]
    return pos, pages * page_size + pos % page_size


def attention(q: torch.Tensor, kv_layer: torch.Tensor, desc: AttnDesc, scale: float | None = None) -> torch.Tensor:
    """Paged GQA attention per the descriptor; returns [M, Hq * hd] in q's dtype."""
    m, hq, hd = q.shape
    hkv, ps = kv_layer.shape[2], kv_layer.shape[3]
    group = hq // hkv
    scale = 1.0 / math.sqrt(hd) if scale is None else scale
    flat_k = kv_layer[:, 0].permute(0, 2, 1, 3).reshape(-1, hkv, hd)  # [pages*ps, Hkv, hd]
    flat_v = kv_layer[:, 1].permute(0, 2, 1, 3).reshape(-1, hkv, hd)
    out = torch.empty(m, hq, hd, dtype=torch.float32, device=q.device)
    for r in range(m):
        _, slots = _row_positions(desc, r, ps)
        k = flat_k[slots.long()].float().repeat_interleave(group, dim=1)  # [n, Hq, hd]
        v = flat_v[slots.long()].float().repeat_interleave(group, dim=1)
        s = torch.einsum("hd,nhd->hn", q[r].float(), k) * scale
        p = torch.softmax(s, dim=-1)
        out[r] = torch.einsum("hn,nhd->hd", p, v)
    return out.reshape(m, hq * hd).to(q.dtype)


def lm_head(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return x.float() @ w.float().t()


def kv_copy_pages(kv: torch.Tensor, copies: torch.Tensor) -> None:
    """For each (src page, dst page, ntok): copy the first ntok slots in every layer."""
    for src, dst, n in copies.tolist():
        kv[:, dst, :, :, :n] = kv[:, src, :, :, :n]


def kv_move_slots(kv: torch.Tensor, src_slots: torch.Tensor, dst_slots: torch.Tensor) -> None:
    """Move slot contents (all layers, k and v); sources are read before any write."""
    ps = kv.shape[-2]
    sp, so = _slot_to_page(src_slots, ps)
    dp, do = _slot_to_page(dst_slots, ps)
    vals = kv[:, sp, :, :, so].clone()  # [L, n, 2, Hkv, hd]
    kv[:, dp, :, :, do] = vals


def topk_logprobs(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    lp = torch.log_softmax(logits.float(), dim=-1)
    return torch.topk(lp, k=k, dim=-1)
