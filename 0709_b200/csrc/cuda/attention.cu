// Paged attention for decode, tree verify and prefill on sm_100a.
//
// Key positions [0, A_r) with A_r = min(row_full[r], shared_len) are read
// through the shared page list by `attn_shared_tc`: per (kv head, split,
// 128-row tile) one CTA streams K/V pages with TMA (one 16-token page per
// box, 128B swizzle) into a 4-stage ring, computes S = Q K^T with
// tcgen05.mma into TMEM (M = 128 query rows = tokens x GQA group, N = 64 keys),
// does the online softmax in registers (one thread per row), writes P to
// shared memory and issues O_chunk = P V (V read MN-major straight from the
// page layout).  Each chunk's O is accumulated in registers.
//
// The rest of each row -- route-private tail pages (drafter) or the
// ancestor-masked node region (target tree) -- is handled by
// `attn_combine_tail`, which also merges the splits' (m, l, O) partials in
// split order (deterministic).  Causal prefill uses the tensor-core kernel
// alone with row limits pos + 1 and writes normalized output directly.
//
// Parity: replaces FlashInfer BatchDecodeWithPagedKVCache (drafter decode,
// reference fp/sglang_page_attention.py:151-209) and BatchPrefillWithPaged-
// KVCache with a custom mask (target verify, reference
// src/atlas_0709/flashinfer_full_verify.py:953-985).

#include "attention.h"
#include "common.cuh"
#include "launch.h"

namespace atlas {

namespace {
constexpr int kChunkKeys = 64;
constexpr int kStages = 4;
constexpr int kHd = 128;
constexpr int kQBytes = 2 * 128 * 128;                     // 2 halves x 128 rows x 128 B
constexpr int kKVHalfBytes = kChunkKeys * 128;             // 64 keys x 128 B
constexpr int kStageBytes = 4 * kKVHalfBytes;              // K (2 halves) + V (2 halves)
constexpr int kPBytes = 128 * 128;                         // 128 rows x 64 keys x 2 B
constexpr int kSmemBytes = kQBytes + kStages * kStageBytes + kPBytes + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;
}  // namespace

template <typename T>
__global__ void __launch_bounds__(160, 1)
    attn_shared_tc(const __grid_constant__ CUtensorMap kvmap, AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;
  uint8_t* kv_s = q_s + kQBytes;
  uint8_t* p_s = kv_s + kStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(p_s + kPBytes);
  uint64_t* empty = full + kStages;
  uint64_t* s_bar = empty + kStages;
  uint64_t* o_bar = s_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_bar + 1);
  int* s_int = reinterpret_cast<int*>(tmem_slot + 1);  // [0] tile max A, [1] ok

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int h = blockIdx.x;
  const int split = blockIdx.y;
  const int G = p.Hq / p.Hkv;
  const int shared_len = p.dparams[0];
  const int ps = p.page_size;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(s_bar, 1);
    mbar_init(o_bar, 1);
    fence_barrier_init();
    s_int[0] = 0;
    s_int[1] = 1;
    tma_prefetch_desc(&kvmap);
  }
  if (warp == 0) tmem_alloc(tmem_slot, 256);
  // Zero the K/V ring so rows past a partial chunk hold finite data.
  for (int i = tid; i < kStages * kStageBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(kv_s)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  pdl_trigger();
  pdl_wait();

  // ---- load the Q tile (row rho = token * G + g of this kv head) and row limits
  const int rho = tid;
  const int grow = blockIdx.z * 128 + rho;
  const int m = grow / G;
  const int hq = h * G + (grow % G);
  int a_lim = 0;
  if (tid < 128) {
    const bool valid = m < p.M;
    if (valid) a_lim = min(p.row_full[m], shared_len);
    const T* qrow = static_cast<const T*>(p.q) + (static_cast<int64_t>(m) * p.Hq + hq) * kHd;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (valid) v = *reinterpret_cast<const uint4*>(qrow + c * 8);
      *reinterpret_cast<uint4*>(q_s + (c >> 3) * (128 * 128) + sw128_offset(rho, c & 7)) = v;
    }
    fence_proxy_async_smem();
    atomicMax(&s_int[0], a_lim);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int tile_max = s_int[0];

  const int np_total = (shared_len + ps - 1) / ps;
  const int pps = (np_total + p.splits - 1) / max(p.splits, 1);
  const int pb = split * pps;
  const int pe = min(min(np_total, pb + pps), (tile_max + ps - 1) / ps);
  const int cp = kChunkKeys / ps;  // pages per chunk
  const int nchunks = pe > pb ? (pe - pb + cp - 1) / cp : 0;

  if (warp == 4) {
    if (tid == 128) {
      bool ok = true;
      for (int c = 0; c < nchunks && ok; ++c) {
        const int s = c % kStages;
        if (c >= kStages) ok = mbar_wait(&empty[s], ((c / kStages) - 1) & 1, p.err);
        if (!ok) break;
        const int p0 = pb + c * cp;
        const int npg = min(cp, pe - p0);
        uint8_t* st = kv_s + s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(npg * ps * 128 * 4));
        for (int i = 0; i < npg; ++i) {
          int page = p.prefix_pages[p0 + i];
          if (page < 0 || page >= p.num_pages) {
            set_error(p.err, kErrBadIndex);
            page = 0;
          }
          const int zc = p.layer * p.num_pages + page;
          const int roff = i * ps * 128;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            tma_load_5d(st + half * kKVHalfBytes + roff, &kvmap, &full[s], half * 64, 0, h, 0, zc);
            tma_load_5d(st + (2 + half) * kKVHalfBytes + roff, &kvmap, &full[s], half * 64, 0, h, 1, zc);
          }
        }
      }
      if (!ok) s_int[1] = 0;
    }
  } else {
    // ---- softmax / MMA warps (rows 0..127)
    const bool is_bf16 = p.bf16 != 0;
    const uint32_t idesc_s = umma_idesc_f16(128, kChunkKeys, is_bf16, false, false);
    const uint32_t idesc_o = umma_idesc_f16(128, kHd, is_bf16, false, true);
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem;        // columns [0, 64)
    const uint32_t tO = tmem + 64;   // columns [64, 192)
    float acc[kHd];
#pragma unroll
    for (int i = 0; i < kHd; ++i) acc[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    const float sl2 = p.scale * kLog2e;
    const int lim = min(a_lim, pe * ps);  // keys of later splits / stale ring rows are masked
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % kStages;
      const uint32_t st = smem_u32(kv_s + s * kStageBytes);
      if (tid == 0) {
        ok = mbar_wait(&full[s], (c / kStages) & 1, p.err);
        tc_fence_after();
        if (ok) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t qa = smem_u32(q_s) + (kk >> 2) * (128 * 128) + (kk & 3) * 32;
            const uint32_t kb = st + (kk >> 2) * kKVHalfBytes + (kk & 3) * 32;
            umma_f16_ss(tS, umma_desc_sw128(qa, 16, 1024), umma_desc_sw128(kb, 16, 1024), idesc_s, kk > 0);
          }
        }
        umma_commit(s_bar);
      }
      __syncwarp();
      ok = mbar_wait(s_bar, c & 1, p.err) && ok;
      tc_fence_after();
      float sv[kChunkKeys];
      tmem_ld32(tS + lane_base, sv);
      tmem_ld32(tS + lane_base + 32, sv + 32);
      const int x0 = (pb + c * cp) * ps;
      float cmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < kChunkKeys; ++j) {
        const int x = x0 + j;
        sv[j] = (x < lim) ? sv[j] * sl2 : -INFINITY;
        cmax = fmaxf(cmax, sv[j]);
      }
      const float m_new = fmaxf(m_run, cmax);
      const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m_run - m_new);
      float psum = 0.f;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        T pk[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float pv = (m_new == -INFINITY) ? 0.f : exp2f(sv[cc * 8 + e] - m_new);
          psum += pv;
          pk[e] = from_f32<T>(pv);
        }
        *reinterpret_cast<uint4*>(p_s + sw128_offset(rho, cc)) = *reinterpret_cast<uint4*>(pk);
      }
      l_run = l_run * alpha + psum;
      m_run = m_new;
      fence_proxy_async_smem();
      tc_fence_before();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (tid == 0) {
        tc_fence_after();
        if (ok) {
          const uint32_t pa = smem_u32(p_s);
          const uint32_t vb = st + 2 * kKVHalfBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_f16_ss(tO, umma_desc_sw128(pa + kk * 32, 16, 1024),
                        umma_desc_sw128(vb + kk * 2048, kKVHalfBytes, 1024), idesc_o, kk > 0);
          }
        }
        umma_commit(o_bar);
        umma_commit(&empty[s]);
      }
      __syncwarp();
      ok = mbar_wait(o_bar, c & 1, p.err) && ok;
      tc_fence_after();
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        float ov[32];
        tmem_ld32(tO + lane_base + q4 * 32, ov);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[q4 * 32 + i] = acc[q4 * 32 + i] * alpha + ov[i];
      }
      tc_fence_before();
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
    if (!ok) s_int[1] = 0;
    // ---- write results
    if (m < p.M) {
      const int64_t rowi = static_cast<int64_t>(m) * p.Hq + hq;
      if (p.direct_out) {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        T* o = static_cast<T*>(p.out) + rowi * kHd;
#pragma unroll
        for (int c8 = 0; c8 < kHd / 8; ++c8) {
          T pk[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) pk[e] = from_f32<T>(acc[c8 * 8 + e] * inv);
          *reinterpret_cast<uint4*>(o + c8 * 8) = *reinterpret_cast<uint4*>(pk);
        }
      } else {
        float* po = p.part_o + (static_cast<int64_t>(split) * p.M * p.Hq + rowi) * kHd;
#pragma unroll
        for (int i = 0; i < kHd; i += 4) *reinterpret_cast<float4*>(po + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
        p.part_ml[static_cast<int64_t>(split) * p.M * p.Hq + rowi] = make_float2(m_run, l_run);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// One warp per (row, q head): merge split partials, then the row's tail keys.
template <typename T>
__global__ void __launch_bounds__(128) attn_combine_tail(AttnParams p) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t pair = static_cast<int64_t>(blockIdx.x) * 4 + warp;
  if (pair >= static_cast<int64_t>(p.M) * p.Hq) return;
  const int m = static_cast<int>(pair / p.Hq);
  const int hq = static_cast<int>(pair % p.Hq);
  const int G = p.Hq / p.Hkv;
  const int h = hq / G;
  const int shared_len = p.dparams[0];
  const int n_shared_pages = p.dparams[1];
  const int mask_base = p.dparams[2];
  const int ps = p.page_size;
  const float sl2 = p.scale * kLog2e;

  float mx = -INFINITY, l = 0.f;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < p.splits; ++s) {
    const float2 ml = p.part_ml[static_cast<int64_t>(s) * p.M * p.Hq + pair];
    if (!(ml.y > 0.f)) continue;
    const float4 ov = *reinterpret_cast<const float4*>(p.part_o + (static_cast<int64_t>(s) * p.M * p.Hq + pair) * kHd + lane * 4);
    const float nm = fmaxf(mx, ml.x);
    const float a = exp2f(mx - nm), b = exp2f(ml.x - nm);
    o[0] = o[0] * a + ov.x * b;
    o[1] = o[1] * a + ov.y * b;
    o[2] = o[2] * a + ov.z * b;
    o[3] = o[3] * a + ov.w * b;
    l = l * a + ml.y * b;
    mx = nm;
  }
  const T* qp = static_cast<const T*>(p.q) + pair * kHd + lane * 4;
  const float q0 = to_f32(qp[0]), q1 = to_f32(qp[1]), q2 = to_f32(qp[2]), q3 = to_f32(qp[3]);
  const int full = p.row_full[m];
  const int rlen = p.row_len[m];
  const int start = min(full, shared_len);
  const int64_t kv_head = static_cast<int64_t>(ps) * kHd;
  for (int x = start; x < rlen; ++x) {
    bool vis = x < full;
    if (!vis) {
      const int b = x - mask_base;
      if (b >= 0 && b < 64 * p.mask_words) {
        const uint64_t w = static_cast<uint64_t>(p.row_mask[static_cast<int64_t>(m) * p.mask_words + (b >> 6)]);
        vis = (w >> (b & 63)) & 1ull;
      }
    }
    if (!vis) continue;
    const int j = x / ps;
    int page = j < n_shared_pages ? p.prefix_pages[j] : p.tail_pages[static_cast<int64_t>(m) * p.tail_stride + (j - n_shared_pages)];
    if (page < 0 || page >= p.num_pages) {
      set_error(p.err, kErrBadIndex);
      continue;
    }
    const int64_t base = ((static_cast<int64_t>(p.layer) * p.num_pages + page) * 2 * p.Hkv + h) * kv_head + (x % ps) * kHd + lane * 4;
    const T* kp = static_cast<const T*>(p.kv) + base;
    const T* vp = kp + static_cast<int64_t>(p.Hkv) * kv_head;
    float sc = q0 * to_f32(kp[0]) + q1 * to_f32(kp[1]) + q2 * to_f32(kp[2]) + q3 * to_f32(kp[3]);
    sc = warp_sum(sc) * sl2;
    const float nm = fmaxf(mx, sc);
    const float a = exp2f(mx - nm), w = exp2f(sc - nm);
    o[0] = o[0] * a + w * to_f32(vp[0]);
    o[1] = o[1] * a + w * to_f32(vp[1]);
    o[2] = o[2] * a + w * to_f32(vp[2]);
    o[3] = o[3] * a + w * to_f32(vp[3]);
    l = l * a + w;
    mx = nm;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* op = static_cast<T*>(p.out) + pair * kHd + lane * 4;
  op[0] = from_f32<T>(o[0] * inv);
  op[1] = from_f32<T>(o[1] * inv);
  op[2] = from_f32<T>(o[2] * inv);
  op[3] = from_f32<T>(o[3] * inv);
}

template <typename T>
static void launch_typed(const CUtensorMap& kvmap, const AttnParams& p, bool run_tc, bool run_combine, int row_tiles,
                         cudaStream_t st) {
  if (run_tc) {
    static bool configured = false;
    if (!configured) {
      cudaFuncSetAttribute(attn_shared_tc<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      configured = true;
    }
    dim3 grid(p.Hkv, p.splits, row_tiles);
    launch_k(attn_shared_tc<T>, grid, dim3(160), kSmemBytes, st, kvmap, p);
  }
  if (run_combine) {
    const int64_t pairs = static_cast<int64_t>(p.M) * p.Hq;
    launch_k(attn_combine_tail<T>, dim3(static_cast<unsigned>((pairs + 3) / 4)), dim3(128), 0, st, p);
  }
}

void launch_attention(const CUtensorMap& kvmap, const AttnParams& p, bool run_tc, bool run_combine, int row_tiles,
                      cudaStream_t st) {
  if (p.bf16)
    launch_typed<__nv_bfloat16>(kvmap, p, run_tc, run_combine, row_tiles, st);
  else
    launch_typed<__half>(kvmap, p, run_tc, run_combine, row_tiles, st);
}

}  // namespace atlas
