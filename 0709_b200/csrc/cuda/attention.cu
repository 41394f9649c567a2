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
constexpr int kPBytes = 128 * 128;                         // 128 rows x 64 keys x 2 B (one buffer)
constexpr int kSmemBytes = kQBytes + kStages * kStageBytes + 2 * kPBytes + 1024 + 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 256 between rescales
constexpr int kThreadsTC = 192;            // warps 0-3 softmax, 4 TMA, 5 MMA
}  // namespace

// 2^x for x <= 0 (softmax weights): the PTX approximate base-2 exponential, subnormal results flushed.
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two fp32 values as one packed pair of T (a in the low half).
template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Profiling stamp k of this CTA (SM clock), when a phase buffer is set.
__device__ __forceinline__ void phase_stamp(const AttnParams& p, int k) {
  if (p.phases != nullptr) {
    const int64_t cta = (static_cast<int64_t>(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    p.phases[cta * kAttnPhases + k] = clock64();
  }
}

// Element offset of key x of row m (kv head h) in the cache, or -1 when x is not visible to the row.
__device__ __forceinline__ int64_t resolve_key(const AttnParams& p, int m, int h, int x, int full, int rlen,
                                               int shared_len, int n_shared_pages, int mask_base) {
  if (x >= rlen) return -1;
  bool vis = x < full;
  if (!vis) {
    const int b = x - mask_base;
    if (b >= 0 && b < 64 * p.mask_words) {
      const uint64_t w = static_cast<uint64_t>(p.row_mask[static_cast<int64_t>(m) * p.mask_words + (b >> 6)]);
      vis = (w >> (b & 63)) & 1ull;
    }
  }
  if (!vis) return -1;
  const int ps = p.page_size;
  const int j = x / ps;
  const bool in_shared = j < n_shared_pages || x < shared_len;
  const int page = in_shared ? p.prefix_pages[j]
                             : p.tail_pages[static_cast<int64_t>(m) * p.tail_stride + (j - n_shared_pages)];
  if (page < 0 || page >= p.num_pages) {
    set_error(p.err, kErrBadIndex);
    return -1;
  }
  return ((static_cast<int64_t>(p.layer) * p.num_pages + page) * 2 * p.Hkv + h) * (static_cast<int64_t>(ps) * kHd) +
         (x % ps) * kHd;
}

// One warp folds keys [start, rlen) of row m (kv head h) into its running
// (mx, l, o), keys in position order; lane t holds dimensions 4t..4t+3 and
// q[0..3] are the row's query values at those dimensions.  `first` is the
// cache offset of key start + lane when the caller resolved it already (so
// the address chain runs before the PDL wait), or -2 to resolve it here.
template <typename T>
__device__ __forceinline__ void fold_tail_keys(const AttnParams& p, int m, int h, int lane, const float* q, int start,
                                               int rlen, int full, int shared_len, int n_shared_pages, int mask_base,
                                               int64_t first, float& mx, float& l, float* o) {
  const float sl2 = p.scale * kLog2e;
  const int64_t kv_head = static_cast<int64_t>(p.page_size) * kHd;
  for (int t0 = start; t0 < rlen; t0 += 32) {
    const int64_t base = (t0 == start && first != -2)
                             ? first
                             : resolve_key(p, m, h, t0 + lane, full, rlen, shared_len, n_shared_pages, mask_base);
    const int cnt = min(32, rlen - t0);
    for (int j0 = 0; j0 < cnt; j0 += 8) {
      int64_t bj[8];
      float2 kh[8], vh[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        bj[u] = (j0 + u < cnt) ? __shfl_sync(0xffffffffu, base, j0 + u) : -1;
        if (bj[u] >= 0) {  // L2 loads: the merge kernel issues them before its PDL wait
          const T* kp = static_cast<const T*>(p.kv) + bj[u] + lane * 4;
          kh[u] = __ldcg(reinterpret_cast<const float2*>(kp));
          vh[u] = __ldcg(reinterpret_cast<const float2*>(kp + static_cast<int64_t>(p.Hkv) * kv_head));
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (bj[u] < 0) continue;  // warp-uniform
        const T* ke = reinterpret_cast<const T*>(&kh[u]);
        const T* ve = reinterpret_cast<const T*>(&vh[u]);
        float sc = q[0] * to_f32(ke[0]) + q[1] * to_f32(ke[1]) + q[2] * to_f32(ke[2]) + q[3] * to_f32(ke[3]);
        sc = warp_sum(sc) * sl2;
        const float nm = fmaxf(mx, sc);
        const float a = exp2f(mx - nm), w = exp2f(sc - nm);
        o[0] = o[0] * a + w * to_f32(ve[0]);
        o[1] = o[1] * a + w * to_f32(ve[1]);
        o[2] = o[2] * a + w * to_f32(ve[2]);
        o[3] = o[3] * a + w * to_f32(ve[3]);
        l = l * a + w;
        mx = nm;
      }
    }
  }
}

// One warp folds row m's keys beyond the shared range -- route-private tail pages
// (drafter) or ancestor-masked nodes (tree verify) -- into its running (mx, l, o).
template <typename T>
__device__ __forceinline__ void row_tail(const AttnParams& p, int m, int h, int64_t pair, int lane, float& mx,
                                         float& l, float* o) {
  const int shared_len = p.dparams[0];
  const int full = p.row_full[m];
  const int rlen = p.row_len[m];
  const int start = min(full, shared_len);
  if (start >= rlen) return;
  const T* qp = static_cast<const T*>(p.q) + pair * kHd + lane * 4;
  const float q[4] = {to_f32(qp[0]), to_f32(qp[1]), to_f32(qp[2]), to_f32(qp[3])};
  fold_tail_keys<T>(p, m, h, lane, q, start, rlen, full, shared_len, p.dparams[1], p.dparams[2], -2, mx, l, o);
}

// Fused-merge epilogue: the p.splits CTAs of one (kv head, row tile) are one cluster,
// each has staged its partial (max, sum) per row in ml_s and its O rows in o_s.  CTA r
// of the cluster owns an equal share of the tile's valid rows; one warp per row reads
// the partials of every split over distributed shared memory in split order
// (deterministic), adds the row's tail keys and writes the normalized output.
template <typename T>
__device__ void merge_rows_and_tails(const AttnParams& p, const float* o_s, const float2* ml_s, int h, int warp,
                                     int lane) {
  const int G = p.Hq / p.Hkv;
  const int C = p.splits;
  const int tile0 = static_cast<int>(blockIdx.z) * 128;
  const int rows_valid = min(128, p.M * G - tile0);
  const int per = (rows_valid + C - 1) / C;
  const int r0 = static_cast<int>(cluster_ctarank()) * per;
  const int r1 = min(rows_valid, r0 + per);
  for (int row = r0 + warp; row < r1; row += kThreadsTC / 32) {
    const int grow = tile0 + row;
    const int m = grow / G;
    const int hq = h * G + grow % G;
    const int64_t pair = static_cast<int64_t>(m) * p.Hq + hq;
    float2 ml = make_float2(-INFINITY, 0.f);
    if (lane < C) ml = ld_dsmem_f2(ml_s + row, static_cast<uint32_t>(lane));
    if (!(ml.y > 0.f)) ml.x = -INFINITY;
    float mx = warp_max(ml.x);
    float l = 0.f;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    if (mx > -INFINITY) {
      const float w = ml.x > -INFINITY ? exp2f(ml.x - mx) : 0.f;
      l = warp_sum(w * ml.y);
      const float* src = o_s + row * kHd + ((lane ^ (row & 31)) * 4);
      for (int s = 0; s < C; ++s) {
        const float ws = __shfl_sync(0xffffffffu, w, s);
        if (ws > 0.f) {  // warp-uniform
          const float4 v = ld_dsmem_f4(src, static_cast<uint32_t>(s));
          o[0] += ws * v.x;
          o[1] += ws * v.y;
          o[2] += ws * v.z;
          o[3] += ws * v.w;
        }
      }
    }
    row_tail<T>(p, m, h, pair, lane, mx, l, o);
    const float inv = l > 0.f ? 1.f / l : 0.f;
    T* op = static_cast<T*>(p.out) + pair * kHd + lane * 4;
    op[0] = from_f32<T>(o[0] * inv);
    op[1] = from_f32<T>(o[1] * inv);
    op[2] = from_f32<T>(o[2] * inv);
    op[3] = from_f32<T>(o[3] * inv);
  }
}

// Warp-specialized flash attention over the shared key range.
//   warp 4  TMA producer: K/V pages of each 64-key chunk into a 4-stage ring
//           (non-causal: the first stages are issued before the PDL wait --
//           they read only committed prefix KV);
//   warp 5  MMA issuer: loads the Q tile by TMA right after the PDL wait, then
//           S(c) = Q K(c)^T into TMEM buffer c%2 and, once the softmax warps
//           publish P(c-1), O += P(c-1) V(c-1) into TMEM;
//   warps 0-3  one thread per query row: online softmax with lazy rescaling
//           (O in TMEM is rescaled only when a row's max grows by more than
//           2^8), P written to a double-buffered shared tile.
template <typename T>
__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_shared_tc(const __grid_constant__ CUtensorMap kvmap, const __grid_constant__ CUtensorMap qmap, AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;
  uint8_t* kv_s = q_s + kQBytes;
  uint8_t* p_s = kv_s + kStages * kStageBytes;  // two P buffers
  uint64_t* full = reinterpret_cast<uint64_t*>(p_s + 2 * kPBytes);
  uint64_t* empty = full + kStages;
  uint64_t* s_full = empty + kStages;  // [2]
  uint64_t* p_full = s_full + 2;       // [2], 128 arrivals
  uint64_t* pv_done = p_full + 2;      // [2]
  uint64_t* fin = pv_done + 2;
  uint64_t* q_full = fin + 1;  // the Q tile (TMA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_full + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int h = blockIdx.x;
  const int split = blockIdx.y;
  const int G = p.Hq / p.Hkv;
  const int ps = p.page_size;
  const bool causal = p.direct_out != 0;
  // Stamps (thread 0 = row 0 unless noted): 0 entry, 1 set up, 2 after the PDL wait, 3 Q staged,
  // 4/6 S(0)/S(1) ready, 5/7 P(0)/P(1) published, 8 O final, 9 partials stored, 10 exit;
  // 11 MMA thread past its first full stage, 12 MMA thread done; 13/14 producer's first / last
  // load issued; 15 global timer (ns) at entry.
  if (tid == 0 && p.phases != nullptr) {
    phase_stamp(p, 0);
    const int64_t cta = (static_cast<int64_t>(blockIdx.z) * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    p.phases[cta * kAttnPhases + 15] = global_timer_ns();
  }

  // Key range of this split, its first page ids and the row limits: graph inputs written
  // before the chain started, so they are safe to read before the wait, and read first so
  // that their latency overlaps the set-up.  The Q tile needs the previous kernel's output.
  const int shared_len = p.dparams[0];
  const int np_total = (shared_len + ps - 1) / ps;
  const int pps = max((np_total + p.splits - 1) / max(p.splits, 1), causal ? 1 : p.min_pages_per_split);
  const int pb = split * pps;
  const int cp = kChunkKeys / ps;  // pages per chunk
  const int rho = tid;
  const int grow = blockIdx.z * 128 + rho;
  const int m = grow / G;
  const int hq = h * G + (grow % G);
  const int pe0 = min(np_total, pb + pps);
  const int nch_loaded = pe0 > pb ? (pe0 - pb + cp - 1) / cp : 0;
  int first_page = -1;  // producer lane i: page pb + i
  if (warp == 4 && pb + (tid & 31) < pe0) first_page = p.prefix_pages[pb + (tid & 31)];
  int row_full_m = 0;
  if (warp < 4 && m < p.M) row_full_m = p.row_full[m];
  // Largest shared-range limit over the tile's tokens (every warp computes the same value, so
  // no warp waits for another to learn how many chunks the tile needs).
  const int tok_per_tile = 128 / G;
  const int m_lo = static_cast<int>(blockIdx.z) * tok_per_tile;
  int tile_max = 0;
  for (int j = tid & 31; j < tok_per_tile; j += 32) {
    const int mm = m_lo + j;
    if (mm < p.M) tile_max = max(tile_max, min(p.row_full[mm], shared_len));
  }

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
      mbar_init(&pv_done[b], 1);
    }
    mbar_init(fin, 1);
    mbar_init(q_full, 1);
    fence_barrier_init();
    tma_prefetch_desc(&kvmap);
    tma_prefetch_desc(&qmap);
  }
  if (warp == 0) tmem_alloc(tmem_slot, 256);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) phase_stamp(p, 1);
  tile_max = __reduce_max_sync(0xffffffffu, tile_max);
  const int pe = min(pe0, (tile_max + ps - 1) / ps);
  const int nchunks = pe > pb ? (pe - pb + cp - 1) / cp : 0;
  // The Q tile (tokens m_lo.., this head's G query heads, two 64-dimension halves) by TMA:
  // rows land 128B-swizzled like the K/V stages, rows past the last token are zero-filled.
  // Issued once the previous kernel (which wrote Q) is complete; only by a CTA that loads keys.
  auto load_q = [&]() {
    mbar_arrive_expect_tx(q_full, static_cast<uint32_t>(kQBytes));
    tma_load_3d(q_s, &qmap, q_full, 0, h * G, m_lo);
    tma_load_3d(q_s + kQBytes / 2, &qmap, q_full, 64, h * G, m_lo);
  };

  int a_lim = 0;
  if (warp == 4) {
    // Producer warp: lane i holds page id pb + i (read before the set-up; the next 32 are read
    // when a split has more), lane 0 streams the chunks.  Pages past the split's end repeat a
    // valid page: finite data that the softmax masks to P = 0.  It never joins a block barrier
    // before the end (the MMA warp frees its ring stages).
    const int lane = tid & 31;
    if (causal) pdl_wait();  // causal prefill reads keys the previous kernel wrote
    bool ok = true;
    int pid = first_page, pid_base = pb;
    for (int c = 0; c < nch_loaded && ok; ++c) {
      const int p0 = pb + c * cp;
      const int npg = min(cp, pe0 - p0);
      if (p0 + cp > pid_base + 32) {
        pid_base = p0;
        pid = p0 + lane < pe0 ? p.prefix_pages[p0 + lane] : -1;
      }
      int pg[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) pg[i] = __shfl_sync(0xffffffffu, pid, (p0 - pid_base + (i < npg ? i : 0)) & 31);
      if (lane == 0) {
        const int s = c % kStages;
        if (c >= kStages) ok = mbar_wait(&empty[s], ((c / kStages) - 1) & 1, p.err);
        if (ok) {
          uint8_t* st = kv_s + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(cp * ps * 128 * 4));
          for (int i = 0; i < cp; ++i) {
            int page = pg[i];
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
        if (c == 0) phase_stamp(p, 13);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
    if (lane == 0) phase_stamp(p, 14);
  } else {
    if (warp < 4) {
      pdl_wait();
      // The successor (the merge/tail kernel) may start now: it reads the queries and the
      // tail keys before its own wait, which the kernel this wait covered has written.
      pdl_trigger();
      if (tid == 0) phase_stamp(p, 2);
      if (m < p.M) a_lim = min(row_full_m, shared_len);
    }
  }

  if (warp == 5) {
    if (tid == 160) {
      const bool is_bf16 = p.bf16 != 0;
      const uint32_t idesc_s = umma_idesc_f16(128, kChunkKeys, is_bf16, false, false);
      const uint32_t idesc_o = umma_idesc_f16(128, kHd, is_bf16, false, true);
      const uint32_t tO = tmem + 128;
      // The Q tile: loaded (once the kernel that wrote Q is complete) by every CTA that loads
      // keys, and waited for even when this tile needs none of them, so no copy into shared
      // memory outlives the CTA.
      bool ok = true;
      if (nch_loaded > 0) {
        pdl_wait();
        load_q();
        ok = mbar_wait(q_full, 0, p.err);
      }
      for (int c = 0; c <= nchunks && ok; ++c) {
        if (c < nchunks) {
          const int s = c % kStages;
          ok = mbar_wait(&full[s], (c / kStages) & 1, p.err);
          if (!ok) break;
          if (c == 0) phase_stamp(p, 11);
          tc_fence_after();
          const uint32_t st = smem_u32(kv_s + s * kStageBytes);
          const uint32_t tS = tmem + (c & 1) * 64;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t qa = smem_u32(q_s) + (kk >> 2) * (128 * 128) + (kk & 3) * 32;
            const uint32_t kb = st + (kk >> 2) * kKVHalfBytes + (kk & 3) * 32;
            umma_f16_ss(tS, umma_desc_sw128(qa, 16, 1024), umma_desc_sw128(kb, 16, 1024), idesc_s, kk > 0);
          }
          umma_commit(&s_full[c & 1]);
        }
        if (c >= 1) {
          const int pc = c - 1;
          ok = mbar_wait(&p_full[pc & 1], (pc >> 1) & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t pa = smem_u32(p_s + (pc & 1) * kPBytes);
          const uint32_t vb = smem_u32(kv_s + (pc % kStages) * kStageBytes) + 2 * kKVHalfBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_f16_ss(tO, umma_desc_sw128(pa + kk * 32, 16, 1024),
                        umma_desc_sw128(vb + kk * 2048, kKVHalfBytes, 1024), idesc_o, (pc > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&pv_done[pc & 1]);
          umma_commit(&empty[pc % kStages]);
        }
      }
      // Release the stages the producer filled beyond this tile's chunks.
      for (int c = nchunks; c < nch_loaded && ok; ++c) {
        ok = mbar_wait(&full[c % kStages], (c / kStages) & 1, p.err);
        if (ok) mbar_arrive(&empty[c % kStages]);
      }
      umma_commit(fin);
      phase_stamp(p, 12);
    }
  } else if (warp < 4) {
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tO = tmem + 128 + lane_base;
    float m_run = -INFINITY, l_run = 0.f;
    const float sl2 = p.scale * kLog2e;
    const int lim = min(a_lim, pe * ps);
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      ok = mbar_wait(&s_full[c & 1], (c >> 1) & 1, p.err) && ok;
      if (tid == 0 && c < 2) phase_stamp(p, 4 + 2 * c);
      tc_fence_after();
      float sv[kChunkKeys];
      tmem_ld32(tmem + (c & 1) * 64 + lane_base, sv);
      tmem_ld32(tmem + (c & 1) * 64 + lane_base + 32, sv + 32);
      const int x0 = (pb + c * cp) * ps;
      if (x0 + kChunkKeys > lim) {  // the row sees this chunk only in part (or not at all)
#pragma unroll
        for (int j = 0; j < kChunkKeys; ++j)
          if (x0 + j >= lim) sv[j] = -INFINITY;
      }
      // Row maximum (a tree; the scale is positive, so it is applied after the max) in log2 units.
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        mx8[i] = fmaxf(fmaxf(fmaxf(sv[i], sv[i + 8]), fmaxf(sv[i + 16], sv[i + 24])),
                       fmaxf(fmaxf(sv[i + 32], sv[i + 40]), fmaxf(sv[i + 48], sv[i + 56])));
      const float cmax = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * sl2;
      const bool grow_max = cmax > m_run + kRescaleThreshold || (m_run == -INFINITY && cmax > -INFINITY);
      float alpha = 1.f;
      if (grow_max) {
        alpha = m_run == -INFINITY ? 0.f : exp2f(m_run - cmax);
        l_run *= alpha;
        m_run = cmax;
      }
      if (c > 0 && __any_sync(0xffffffffu, grow_max)) {
        // O must hold P(c-1) V(c-1) before it is rescaled.
        ok = mbar_wait(&pv_done[(c - 1) & 1], ((c - 1) >> 1) & 1, p.err) && ok;
        tc_fence_after();
#pragma unroll 1
        for (int q4 = 0; q4 < 4; ++q4) {
          float ov[32];
          tmem_ld32(tO + q4 * 32, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= alpha;
          tmem_st32(tO + q4 * 32, ov);
        }
      }
      // P buffer c%2 is free once PV(c-2) completed.
      if (c >= 2) ok = mbar_wait(&pv_done[c & 1], ((c - 2) >> 1) & 1, p.err) && ok;
      uint8_t* pbuf = p_s + (c & 1) * kPBytes;
      // P = 2^(s * scale * log2(e) - m): one FMA and one ex2 per key.  A row that has seen
      // no key yet has m = -inf and every s = -inf, so P = 0.
      const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
      float psum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = exp2_approx(fmaf(sv[cc * 8 + 2 * e], sl2, neg_m));
          const float p1 = exp2_approx(fmaf(sv[cc * 8 + 2 * e + 1], sl2, neg_m));
          psum4[e] += p0 + p1;
          w[e] = pack_pair<T>(p0, p1);
        }
        *reinterpret_cast<uint4*>(pbuf + sw128_offset(rho, cc)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l_run += (psum4[0] + psum4[1]) + (psum4[2] + psum4[3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[c & 1]);
      if (tid == 0 && c < 2) phase_stamp(p, 5 + 2 * c);
    }
    ok = mbar_wait(fin, 0, p.err) && ok;
    if (tid == 0) phase_stamp(p, 8);
    tc_fence_after();
    float acc[kHd];
    if (nchunks > 0) {
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tmem_ld32(tO + q4 * 32, acc + q4 * 32);
    } else {
#pragma unroll
      for (int i = 0; i < kHd; ++i) acc[i] = 0.f;
    }
    if (p.fused_merge) {
      // Stage this split's (max, sum) and unnormalized O rows for the cluster merge: O over the
      // drained K/V ring (every TMA load landed and every MMA finished before `fin`), 16-byte
      // chunks XOR-swizzled by row so the 128 row threads do not share banks.
      float* o_s = reinterpret_cast<float*>(kv_s);
      float2* ml_s = reinterpret_cast<float2*>(p_s);
      ml_s[rho] = make_float2(l_run > 0.f ? m_run : -INFINITY, l_run);
      if (l_run > 0.f) {
#pragma unroll
        for (int c4 = 0; c4 < kHd / 4; ++c4)
          *reinterpret_cast<float4*>(o_s + rho * kHd + ((c4 ^ (rho & 31)) * 4)) =
              make_float4(acc[c4 * 4], acc[c4 * 4 + 1], acc[c4 * 4 + 2], acc[c4 * 4 + 3]);
      }
    } else if (m < p.M) {
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
        // A split that saw no key of this row leaves (m, l) = (-inf, 0); the
        // merge gives it weight 0 and never reads its O.
        if (l_run > 0.f) {
          float* po = p.part_o + (static_cast<int64_t>(split) * p.M * p.Hq + rowi) * kHd;
#pragma unroll
          for (int i = 0; i < kHd; i += 4)
            *reinterpret_cast<float4*>(po + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
        }
        p.part_ml[static_cast<int64_t>(split) * p.M * p.Hq + rowi] = make_float2(m_run, l_run);
      }
    }
  }
  if (tid == 0) phase_stamp(p, 9);
  tc_fence_before();
  __syncthreads();
  if (tid == 0) phase_stamp(p, 10);
  if (warp == 0) tmem_dealloc(tmem, 256);
  if (p.fused_merge) {
    cluster_sync();  // every split of the cluster has staged its partials
    merge_rows_and_tails<T>(p, reinterpret_cast<const float*>(kv_s), reinterpret_cast<const float2*>(p_s), h, warp,
                            tid & 31);
    cluster_sync();  // the other CTAs are done reading this CTA's shared memory
  }
}

// One warp per (row, q head): the row's tail keys and the merge of the split partials.
// Latency-bound, so the dependent round trips after the PDL wait are cut to one: the
// tensor-core kernel triggers this launch only after its own wait returned (the kernel
// that wrote the queries and the tail keys is complete), so the whole tail -- key
// addresses, K/V loads and the online softmax over those keys -- runs before this
// kernel's wait, overlapping the split pass.  After the wait the split records and the
// split partials are loaded together and merged in split order, then folded with the
// tail's partial (a fixed order, independent of timing).
template <typename T>
__global__ void __launch_bounds__(128) attn_combine_tail(AttnParams p) {
  constexpr int kBatch = 24;  // split partials loaded in the first round trip
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t pair = static_cast<int64_t>(blockIdx.x) * 4 + warp;
  if (pair >= static_cast<int64_t>(p.M) * p.Hq) {
    pdl_trigger();
    return;
  }
  const int m = static_cast<int>(pair / p.Hq);
  const int hq = static_cast<int>(pair % p.Hq);
  const int G = p.Hq / p.Hkv;
  const int h = hq / G;
  const int64_t stride_split = static_cast<int64_t>(p.M) * p.Hq;

  // ---- before the wait: the tail keys [start, rlen) of this row
  const int shared_len = p.dparams[0];
  const int full = p.row_full[m];
  const int rlen = p.row_len[m];
  const int start = min(full, shared_len);
  float mt = -INFINITY, lt = 0.f;
  float ot[4] = {0.f, 0.f, 0.f, 0.f};
  if (start < rlen) {
    const uint2 qraw = __ldcg(reinterpret_cast<const uint2*>(static_cast<const T*>(p.q) + pair * kHd + lane * 4));
    const T* qe = reinterpret_cast<const T*>(&qraw);
    const float q[4] = {to_f32(qe[0]), to_f32(qe[1]), to_f32(qe[2]), to_f32(qe[3])};
    fold_tail_keys<T>(p, m, h, lane, q, start, rlen, full, shared_len, p.dparams[1], p.dparams[2], -2, mt, lt, ot);
  }

  pdl_wait();
  pdl_trigger();

  // ---- split records and partials in one round trip (lane s holds records s and s + 32; splits <= 64)
  const int S = p.splits;
  float2 ml0 = make_float2(-INFINITY, 0.f), ml1 = make_float2(-INFINITY, 0.f);
  if (lane < S) ml0 = __ldcg(p.part_ml + lane * stride_split + pair);
  if (lane + 32 < S) ml1 = __ldcg(p.part_ml + (lane + 32) * stride_split + pair);
  const float* po = p.part_o + pair * kHd + lane * 4;
  float4 ov[kBatch];
#pragma unroll
  for (int j = 0; j < kBatch; ++j)
    ov[j] = j < S ? __ldcg(reinterpret_cast<const float4*>(po + j * stride_split * kHd)) : make_float4(0.f, 0.f, 0.f, 0.f);

  float mx = -INFINITY, l = 0.f;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  if (!(ml0.y > 0.f)) ml0.x = -INFINITY;  // a split that saw no key of this row left no O
  if (!(ml1.y > 0.f)) ml1.x = -INFINITY;
  mx = warp_max(fmaxf(ml0.x, ml1.x));
  if (mx > -INFINITY) {
    const float w0 = ml0.x > -INFINITY ? exp2f(ml0.x - mx) : 0.f;
    const float w1 = ml1.x > -INFINITY ? exp2f(ml1.x - mx) : 0.f;
    l = warp_sum(w0 * ml0.y + w1 * ml1.y);
    auto weight = [&](int sidx) {
      return sidx < 32 ? __shfl_sync(0xffffffffu, w0, sidx & 31) : __shfl_sync(0xffffffffu, w1, sidx & 31);
    };
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const float w = j < S ? weight(j) : 0.f;
      if (w > 0.f) {  // warp-uniform; unwritten partials are never read into the sum
        o[0] += w * ov[j].x;
        o[1] += w * ov[j].y;
        o[2] += w * ov[j].z;
        o[3] += w * ov[j].w;
      }
    }
    for (int s0 = kBatch; s0 < S; s0 += 16) {
      float4 v[16];
      float wv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int sidx = s0 + j;
        wv[j] = sidx < S ? weight(sidx) : 0.f;
        v[j] = wv[j] > 0.f ? __ldcg(reinterpret_cast<const float4*>(po + sidx * stride_split * kHd))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[0] += wv[j] * v[j].x;
        o[1] += wv[j] * v[j].y;
        o[2] += wv[j] * v[j].z;
        o[3] += wv[j] * v[j].w;
      }
    }
  }

  // ---- fold in the tail's partial
  const float M = fmaxf(mx, mt);
  const float a = mx > -INFINITY ? exp2f(mx - M) : 0.f;
  const float b = mt > -INFINITY ? exp2f(mt - M) : 0.f;
  l = l * a + lt * b;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* op = static_cast<T*>(p.out) + pair * kHd + lane * 4;
  op[0] = from_f32<T>((o[0] * a + ot[0] * b) * inv);
  op[1] = from_f32<T>((o[1] * a + ot[1] * b) * inv);
  op[2] = from_f32<T>((o[2] * a + ot[2] * b) * inv);
  op[3] = from_f32<T>((o[3] * a + ot[3] * b) * inv);
}

template <typename T>
static void configure_tc() {
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(attn_shared_tc<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    cudaFuncSetAttribute(attn_shared_tc<T>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured = true;
  }
}

template <typename T>
static void launch_typed(const CUtensorMap& kvmap, const CUtensorMap& qmap, const AttnParams& p, bool run_tc,
                         bool run_combine, int row_tiles, cudaStream_t st) {
  if (p.fused_merge) {
    // Splits of one head = one cluster; the merge and the tails run in the same kernel.
    configure_tc<T>();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.Hkv, p.splits, row_tiles);
    cfg.blockDim = dim3(kThreadsTC);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = p.splits;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, attn_shared_tc<T>, kvmap, qmap, p);
    return;
  }
  if (run_tc) {
    configure_tc<T>();
    dim3 grid(p.Hkv, p.splits, row_tiles);
    launch_k(attn_shared_tc<T>, grid, dim3(kThreadsTC), kSmemBytes, st, kvmap, qmap, p);
  }
  if (run_combine) {
    const int64_t pairs = static_cast<int64_t>(p.M) * p.Hq;
    launch_k(attn_combine_tail<T>, dim3(static_cast<unsigned>((pairs + 3) / 4)), dim3(128), 0, st, p);
  }
}

template <typename T>
static int max_cluster_typed() {
  configure_tc<T>();
  for (int c : {16, 8}) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, c, 1);
    cfg.blockDim = dim3(kThreadsTC);
    cfg.dynamicSmemBytes = kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = c;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_shared_tc<T>, &cfg) == cudaSuccess && n >= 1) return c;
    cudaGetLastError();  // a refused size leaves a sticky error of this query only
  }
  return 8;
}

int attention_max_cluster(bool bf16) {
  static const int v16 = max_cluster_typed<__half>();
  static const int vbf = max_cluster_typed<__nv_bfloat16>();
  return bf16 ? vbf : v16;
}

static unsigned long long* g_phase_buffer = nullptr;

void set_attention_phase_buffer(unsigned long long* buf) { g_phase_buffer = buf; }

void launch_attention(const CUtensorMap& kvmap, const CUtensorMap& qmap, const AttnParams& p_in, bool run_tc,
                      bool run_combine, int row_tiles, cudaStream_t st) {
  AttnParams p = p_in;
  p.phases = g_phase_buffer;
  if (p.bf16)
    launch_typed<__nv_bfloat16>(kvmap, qmap, p, run_tc, run_combine, row_tiles, st);
  else
    launch_typed<__half>(kvmap, qmap, p, run_tc, run_combine, row_tiles, st);
}

}  // namespace atlas
