"""CUDA op table: the engine's ops backed by the sm_100a kernels of ``atlas_cuda``.

Each engine owns one ``CudaOps`` with persistent device buffers: the split-KV
attention partials and an error flag (the GEMM reduces its K splits inside a
thread-block cluster and needs no workspace; ``ws``/``counters`` are unused
placeholders kept for the binding signature).  The error flag is set by kernels instead of trapping (bad index, bounded wait that
timed out).  ``check()`` reads the flag.  If the extension cannot be loaded on
a GPU machine, construction raises -- there is no silent fallback.

The reference reaches the same operations through SGLang, FlashInfer, cuBLAS and torch
(drafter: src/atlas_0709/flashinfer_paged/frontier.py:128-307 and sglang_runtime.py:708-798,
1031-1092; target: src/atlas_0709/target_runtime.py:144-321, 767-851, 873-920).
"""

from __future__ import annotations

import math
import os

import torch

from . import _native
from ..utils import counters
from ..utils.transfer import ERROR_NAMES, KernelError  # noqa: F401  (re-exported)
from .attn_desc import AttnDesc

_FLAGS: dict[int, torch.Tensor] = {}


def device_error_flag(device: torch.device) -> torch.Tensor:
    """The device's error flag (int32[1]), shared by every op table and TP group on it.

    Kernels record a code here instead of trapping; one read of this flag (packed
    into a result copy the serving path makes anyway) covers every kernel that
    ran on the device before it.
    """
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    flag = _FLAGS.get(idx)
    if flag is None:
        flag = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _FLAGS[idx] = flag
    return flag


def _ext():
    return _native.cuda()


class CudaOps:
    def __init__(self, engine=None, *, device: torch.device | None = None) -> None:
        self.ext = _ext()
        self.engine = engine
        self.device = engine.device if engine is not None else (device or torch.device("cuda"))
        dev = self.device
        self.err = device_error_flag(dev)
        self.ws = torch.empty(0, dtype=torch.float32, device=dev)
        self.counters = torch.empty(0, dtype=torch.int32, device=dev)
        self.part_o = torch.empty(0, dtype=torch.float32, device=dev)
        self.part_ml = torch.empty(0, dtype=torch.float32, device=dev)
        self.num_sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.last_gemm_config: list[int] | None = None
        # Split merge inside the attention kernel (thread-block clusters, ATLAS_ATTN_FUSED_MERGE=1) or the
        # separate merge kernel (default, faster in the serving round as measured); cluster size capped
        # by ATLAS_ATTN_MAX_CLUSTER.
        self.fused_merge = os.environ.get("ATLAS_ATTN_FUSED_MERGE", "0") == "1"
        self.cluster_cap = int(os.environ.get("ATLAS_ATTN_MAX_CLUSTER", "16"))
        self._max_cluster: dict[bool, int] = {}

    # ----------------------------------------------------------- errors
    def check(self) -> None:
        code = int(self.err.item())
        if code:
            self.err.zero_()
            raise KernelError(code)

    # ------------------------------------------------------------- GEMM
    def _gemm(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, epi: int) -> torch.Tensor:
        self.last_gemm_config = self.ext.gemm(w, x, out, epi, self.ws, self.counters, self.err, 0)
        counters.launches(1)
        return out

    def linear(self, x: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        out = torch.empty((x.shape[0], w.shape[0]), dtype=w.dtype, device=x.device)
        return self._gemm(x, w, out, self.ext.EPI_STORE)

    def linear_residual(self, x: torch.Tensor, w: torch.Tensor, resid: torch.Tensor) -> torch.Tensor:
        return self._gemm(x, w, resid, self.ext.EPI_RESIDUAL)

    def gate_up_silu(self, x: torch.Tensor, wgu: torch.Tensor) -> torch.Tensor:
        out = torch.empty((x.shape[0], wgu.shape[0] // 2), dtype=wgu.dtype, device=x.device)
        return self._gemm(x, wgu, out, self.ext.EPI_SILU)

    def lm_head(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        out = torch.empty((x.shape[0], w.shape[0]), dtype=torch.float32, device=x.device)
        return self._gemm(x, w, out, self.ext.EPI_F32)

    # ------------------------------------------------ folded-norm GEMMs
    # RMSNorm is folded into the GEMMs: the B operand is the residual h in the
    # activation dtype (``hb``), the norm gain lives in the weight rows, and
    # the epilogue scales each token column by rstd computed from ``ss``, the
    # per-128-feature sums of h^2 written by the previous residual epilogue.
    def embed_norm(self, tokens: torch.Tensor, table: torch.Tensor):
        m, hdim = tokens.numel(), table.shape[1]
        h = torch.empty((m, hdim), dtype=torch.float32, device=table.device)
        hb = torch.empty((m, hdim), dtype=table.dtype, device=table.device)
        ss = torch.empty((hdim // 128, m), dtype=torch.float32, device=table.device)
        self.ext.embed_norm(tokens.to(torch.int32), table, h, hb, ss, self.err)
        counters.launches(1)
        return h, hb, ss

    def _fused(self, w, x, out, epi, *, ss=None, eps=0.0, ss_out=None, hb=None, rope=None):
        table = pos = slots = kv = q = None
        hq = hkv = 0
        if rope is not None:
            table, pos, slots, kv, q, hq, hkv = rope
        self.last_gemm_config = self.ext.gemm_fused(w, x, out, epi, self.err, ss, float(eps), ss_out, hb, table, pos,
                                                    slots, kv, q, hq, hkv)
        counters.launches(1)

    def qkv_rope(self, hb, w, ss, eps, table, positions, slots, kv_layer, num_heads, num_kv_heads):
        q = torch.empty((hb.shape[0], num_heads, 128), dtype=hb.dtype, device=hb.device)
        self._fused(w, hb, None, self.ext.EPI_ROPE, ss=ss, eps=eps,
                    rope=(table, positions.to(torch.int32), slots.to(torch.int32), kv_layer, q, num_heads,
                          num_kv_heads))
        return q

    def linear_residual_norm(self, x, w, h, hb, ss_out) -> None:
        self._fused(w, x, h, self.ext.EPI_RESIDUAL_NORM, ss_out=ss_out, hb=hb)

    def gate_up_silu_norm(self, hb, wgu, ss, eps):
        out = torch.empty((hb.shape[0], wgu.shape[0] // 2), dtype=wgu.dtype, device=hb.device)
        self._fused(wgu, hb, out, self.ext.EPI_SILU, ss=ss, eps=eps)
        return out

    def lm_head_norm(self, hb, w, ss, eps):
        out = torch.empty((hb.shape[0], w.shape[0]), dtype=torch.float32, device=hb.device)
        self._fused(w, hb, out, self.ext.EPI_F32, ss=ss, eps=eps)
        return out

    # -------------------------------------------------------------- fp8
    @staticmethod
    def _scale_ld(n: int) -> int:
        return (n + 3) // 4 * 4

    def quant_fp8(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        n, k = x.shape
        xq = torch.empty((n, k), dtype=torch.float8_e4m3fn, device=x.device)
        sa = torch.empty((k // 128, self._scale_ld(n)), dtype=torch.float32, device=x.device)
        self.ext.quant_fp8(x.contiguous(), xq, sa)
        counters.launches(1)
        return xq, sa

    def rmsnorm_fp8(self, h: torch.Tensor, w: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
        n, k = h.shape
        xq = torch.empty((n, k), dtype=torch.float8_e4m3fn, device=h.device)
        sa = torch.empty((k // 128, self._scale_ld(n)), dtype=torch.float32, device=h.device)
        self.ext.rmsnorm_fp8(h.contiguous(), w, xq, sa, float(eps))
        counters.launches(1)
        return xq, sa

    def gemm_fp8(self, xq: torch.Tensor, sa: torch.Tensor, w, out: torch.Tensor, epi: int) -> torch.Tensor:
        self.last_gemm_config = self.ext.gemm_fp8(w.q, w.scale, xq, sa, out, epi, self.err)
        counters.launches(1)
        return out

    # ------------------------------------------------------ elementwise
    def embed(self, tokens: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
        out = torch.empty((tokens.numel(), table.shape[1]), dtype=torch.float32, device=table.device)
        self.ext.embed(tokens.to(torch.int32), table, out, self.err)
        counters.launches(1)
        return out

    def rmsnorm(self, x: torch.Tensor, w: torch.Tensor, eps: float, out_dtype: torch.dtype) -> torch.Tensor:
        out = torch.empty(x.shape, dtype=w.dtype, device=x.device)
        self.ext.rmsnorm(x.contiguous(), w, out, float(eps))
        counters.launches(1)
        return out

    def rope_qkv_append(self, qkv, table, positions, slots, kv_layer, num_heads, num_kv_heads):
        hd = kv_layer.shape[-1]
        q = torch.empty((qkv.shape[0], num_heads, hd), dtype=qkv.dtype, device=qkv.device)
        self.ext.rope_append(
            qkv, table, positions.to(torch.int32), slots.to(torch.int32), kv_layer, q, num_heads, num_kv_heads, self.err
        )
        counters.launches(1)
        return q

    # -------------------------------------------------------- attention
    def _layer_index(self, kv_layer: torch.Tensor) -> tuple[torch.Tensor, int]:
        kv = self.engine.kv
        per = kv[0].numel() * kv.element_size()
        off = kv_layer.data_ptr() - kv.data_ptr()
        if off % per or not 0 <= off // per < kv.shape[0]:
            raise ValueError("kv_layer must be a layer view of the engine cache")
        return kv, off // per

    def _dparams(self, desc: AttnDesc) -> torch.Tensor:
        cached = getattr(desc, "_dparams", None)
        if cached is None:
            cached = torch.tensor(
                [desc.shared_len, desc.n_shared_pages, desc.mask_base], dtype=torch.int32
            ).to(self.device, non_blocking=True)
            desc._dparams = cached  # type: ignore[attr-defined]
        return cached

    def attention_splits(self, rows: int, hq: int, hkv: int, shared_len: int, page_size: int) -> int:
        g = hq // hkv
        row_tiles = max(1, math.ceil(rows * g / 128))
        chunks = max(1, math.ceil(math.ceil(shared_len / page_size) / (64 // page_size)))
        return int(max(1, min(64, self.num_sms // (hkv * row_tiles), chunks)))

    def reserve_attention_workspace(self, max_rows: int, hq: int, hkv: int, max_context: int, page_size: int) -> None:
        """Allocate split partials for every row count up to ``max_rows`` once (graphs keep the address)."""
        need_o = need_ml = 0
        for m in range(1, max_rows + 1):
            sp = self.attention_splits(m, hq, hkv, max_context, page_size)
            need_o = max(need_o, sp * m * hq * 128)
            need_ml = max(need_ml, 2 * sp * m * hq)
        self._ensure_parts_exact(need_o, need_ml)

    def _ensure_parts_exact(self, need_o: int, need_ml: int) -> None:
        if self.part_o.numel() < need_o:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("attention workspace must be reserved before graph capture")
            self.part_o = torch.empty(need_o, dtype=torch.float32, device=self.device)
        if self.part_ml.numel() < need_ml:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("attention workspace must be reserved before graph capture")
            self.part_ml = torch.empty(need_ml, dtype=torch.float32, device=self.device)

    def _ensure_parts(self, splits: int, m: int, hq: int) -> None:
        self._ensure_parts_exact(splits * m * hq * 128, 2 * splits * m * hq)

    def attention(self, q: torch.Tensor, kv_layer: torch.Tensor, desc: AttnDesc, scale: float | None = None,
                  *, splits: int | None = None, stages: tuple[bool, bool] = (True, True)) -> torch.Tensor:
        kv, layer = self._layer_index(kv_layer)
        m, hq, hd = q.shape
        scale = 1.0 / math.sqrt(hd) if scale is None else scale
        out = torch.empty((m, hq * hd), dtype=q.dtype, device=q.device)
        run_tc = desc.shared_len > 0 and stages[0]
        sp = splits or getattr(desc, "_splits", None) or self.attention_splits(m, hq, kv.shape[3], desc.shared_len,
                                                                                kv.shape[4])
        if run_tc and stages[1] and self.fused_merge:
            # One launch: the splits of a head form one cluster and merge (plus the rows' tail keys)
            # over distributed shared memory; no split workspace.
            c = min(int(sp), self.max_cluster(q.dtype))
            self.ext.attention(
                q.contiguous(), kv, layer, out, self._dparams(desc), desc.prefix_pages, desc.row_full, desc.row_len,
                desc.row_mask, desc.tail_pages, self.part_o, self.part_ml, self.err, c, True, True, False,
                float(scale), True,
            )
            counters.launches(1)
            return out
        if run_tc:
            self._ensure_parts(sp, m, hq)
        self.ext.attention(
            q.contiguous(), kv, layer, out, self._dparams(desc), desc.prefix_pages, desc.row_full, desc.row_len,
            desc.row_mask, desc.tail_pages, self.part_o, self.part_ml, self.err, sp, run_tc, stages[1], False,
            float(scale), False,
        )
        counters.launches(int(run_tc) + int(stages[1]))
        return out

    def max_cluster(self, dtype: torch.dtype) -> int:
        key = dtype == torch.bfloat16
        if key not in self._max_cluster:
            self._max_cluster[key] = int(self.ext.attention_max_cluster(key))
        return max(1, min(self._max_cluster[key], self.cluster_cap))

    def attention_causal(self, q, kv_layer, desc: AttnDesc, causal_start: int, scale: float | None = None):
        kv, layer = self._layer_index(kv_layer)
        m, hq, hd = q.shape
        scale = 1.0 / math.sqrt(hd) if scale is None else scale
        out = torch.empty((m, hq * hd), dtype=q.dtype, device=q.device)
        # All rows of a prefill chunk read one page list; limits are pos + 1 (row_full).
        total = int(causal_start) + m
        dp = getattr(desc, "_causal_dparams", None)
        if dp is None:
            dp = torch.tensor([total, desc.n_shared_pages, 0], dtype=torch.int32).to(self.device)
            desc._causal_dparams = dp  # type: ignore[attr-defined]
        self.ext.attention(
            q.contiguous(), kv, layer, out, dp, desc.prefix_pages, desc.row_full, desc.row_len,
            desc.row_mask, desc.tail_pages, self.part_o, self.part_ml, self.err, 1, True, False, True, float(scale),
            False,
        )
        counters.launches(1)
        return out

    # --------------------------------------------------------- KV cache
    def kv_copy_pages(self, kv: torch.Tensor, copies: torch.Tensor) -> None:
        self.ext.kv_copy_pages(kv, copies.to(self.device, torch.int32).contiguous(), self.err)
        counters.launches(1)

    def kv_copy_pages_counted(self, kv: torch.Tensor, plan: torch.Tensor, count: torch.Tensor) -> None:
        """Copy-on-write of ``count[0]`` rows of ``plan`` [max, 3] (both read on the device)."""
        self.ext.kv_copy_pages_counted(kv, plan, count, self.err)
        counters.launches(1)

    def kv_move_slots(self, kv: torch.Tensor, src: torch.Tensor, dst: torch.Tensor) -> None:
        self.ext.kv_move_slots(kv, src.to(self.device, torch.int32), dst.to(self.device, torch.int32), self.err)
        counters.launches(1)

    # ----------------------------------------------------------- vocab
    def topk_logprobs(self, logits: torch.Tensor, k: int, keys: torch.Tensor | None = None, temperature: float = 1.0):
        b = logits.shape[0]
        lp = torch.empty((b, k), dtype=torch.float32, device=logits.device)
        ids = torch.empty((b, k), dtype=torch.int64, device=logits.device)
        self.ext.topk(logits.float().contiguous(), k, keys, 1.0 / float(temperature), lp, ids)
        counters.launches(1)
        return lp, ids

    def gather_logprobs(self, logits: torch.Tensor, rows: torch.Tensor, toks: torch.Tensor) -> torch.Tensor:
        lse = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device)
        out = torch.empty(rows.numel(), dtype=torch.float32, device=logits.device)
        self.ext.gather_logprobs(
            logits.contiguous(), rows.to(logits.device, torch.int32), toks.to(logits.device, torch.int32), lse, out,
            self.err,
        )
        counters.launches(2)
        return out


_SHARED: dict[int, CudaOps] = {}


def shared_ops(device: torch.device | None = None) -> CudaOps:
    """Process-wide op table for model-independent kernels (top-k, gathers)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _SHARED:
        _SHARED[idx] = CudaOps(device=torch.device("cuda", idx))
    return _SHARED[idx]
