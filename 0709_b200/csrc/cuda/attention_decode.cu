// Split pass of paged attention for few query rows (decode), on CUDA cores.
//
// With at most kDecodeMaxRows query rows per kv head (tokens x GQA group; one token
// of the 8B geometry is 4 rows), the tensor-core split kernel spends its time
// on a 128-row tile that is nearly all padding and on a long mbarrier/TMEM
// pipeline per 64-key chunk.  This kernel covers the same shared key range
// [0, min(row_full, shared_len)) with plain loads and FMAs and writes the same
// split partials (running max in log2 units, sum, unnormalized O), so the
// merge/tail kernel that follows is unchanged.
//
// Grid (kv heads, splits), 128 threads.  Split s covers keys [s*K, s*K + K)
// with K = ceil(shared_len / splits), processed in chunks of kChunk keys:
//   pass 1  thread t scores key t of the chunk (t < kChunk) against every row
//           (Q rows staged in shared memory as fp32, read as broadcasts), one
//           K row per thread; the chunk's row maxima and sums meet through
//           warp shuffles and a shared-memory step, and the probabilities
//           p = 2^(s - m) go to shared memory;
//   pass 2  warp w owns rows w, w + 4, ...; lane l owns dimensions 4l..4l+3
//           and accumulates sum_j p[r][j] * V[j] with coalesced V loads.
// Running (max, sum, O) are rescaled when a later chunk raises a row's max.
// Before the programmatic-launch wait the split's K/V rows are prefetched to
// L2 (they are committed prefix keys, not outputs of the preceding kernel).

#include "attention.h"
#include "common.cuh"
#include "launch.h"

namespace atlas {

namespace {
constexpr int kDecThreads = 128;
constexpr int kChunk = 128;       // keys scored per pass (one per thread)
constexpr int kHdD = 128;
constexpr float kLog2eD = 1.4426950408889634f;
}  // namespace

template <typename T>
__global__ void __launch_bounds__(kDecThreads) attn_decode_split(AttnParams p) {
  __shared__ float q_s[kDecodeMaxRows][kHdD];           // 8 KB
  __shared__ float p_s[kDecodeMaxRows][kChunk];          // 8 KB: scores, then probabilities
  __shared__ int64_t off_s[kChunk];                      // element offset of each key's K row (-1: none)
  __shared__ float red_s[kDecThreads / 32][kDecodeMaxRows];
  __shared__ float alpha_s[kDecodeMaxRows];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int h = blockIdx.x;
  const int split = blockIdx.y;
  const int G = p.Hq / p.Hkv;
  const int R = p.M * G;  // <= kDecodeMaxRows (checked on the host)
  const int ps = p.page_size;
  const int64_t kv_head = static_cast<int64_t>(ps) * kHdD;

  const int shared_len = p.dparams[0];
  const int per = (shared_len + p.splits - 1) / max(p.splits, 1);
  const int k0 = min(shared_len, split * per);
  const int k1 = min(shared_len, k0 + per);

  // Committed prefix keys: warm L2 while the preceding kernel finishes.
  for (int x = k0 + tid; x < k1; x += kDecThreads) {
    const int page = p.prefix_pages[x / ps];
    if (page >= 0 && page < p.num_pages) {
      const T* kp = static_cast<const T*>(p.kv) +
                    ((static_cast<int64_t>(p.layer) * p.num_pages + page) * 2 * p.Hkv + h) * kv_head + (x % ps) * kHdD;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kp));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kp + 64));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kp + static_cast<int64_t>(p.Hkv) * kv_head));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kp + static_cast<int64_t>(p.Hkv) * kv_head + 64));
    }
  }
  pdl_wait();
  pdl_trigger();

  // Q rows of this kv head (row r = token r / G, head h * G + r % G) and each row's key limit.
  for (int i = tid; i < R * kHdD; i += kDecThreads) {
    const int r = i / kHdD, d = i % kHdD;
    const int m = r / G, hq = h * G + r % G;
    q_s[r][d] = to_f32(static_cast<const T*>(p.q)[(static_cast<int64_t>(m) * p.Hq + hq) * kHdD + d]);
  }
  const float sl2 = p.scale * kLog2eD;
  // Warp w owns rows w, w + 4, ... in pass 2: its running state lives in registers.
  constexpr int kRowsPerWarp = kDecodeMaxRows / (kDecThreads / 32);
  float l_run[kRowsPerWarp], acc[kRowsPerWarp][4];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    l_run[i] = 0.f;
    acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  }
  __syncthreads();
  __shared__ float mrun_s[kDecodeMaxRows];
  __shared__ int lim_s[kDecodeMaxRows];
  if (tid < kDecodeMaxRows) {
    mrun_s[tid] = -INFINITY;
    lim_s[tid] = tid < R ? min(p.row_full[tid / G], shared_len) : 0;
  }
  __syncthreads();

  const T* kv = static_cast<const T*>(p.kv);
  const int64_t v_step = static_cast<int64_t>(p.Hkv) * kv_head;  // K row -> V row of the same key
  for (int c0 = k0; c0 < k1; c0 += kChunk) {
    const int n = min(kChunk, k1 - c0);
    // ---- pass 1: thread t scores key c0 + t against every row
    const int x = c0 + tid;
    int64_t off = -1;
    if (tid < n) {
      const int page = p.prefix_pages[x / ps];
      if (page < 0 || page >= p.num_pages) {
        set_error(p.err, kErrBadIndex);
      } else {
        off = ((static_cast<int64_t>(p.layer) * p.num_pages + page) * 2 * p.Hkv + h) * kv_head + (x % ps) * kHdD;
      }
    }
    off_s[tid] = off;
    float sc[kDecodeMaxRows];
#pragma unroll
    for (int r = 0; r < kDecodeMaxRows; ++r) sc[r] = 0.f;
    if (off >= 0) {
      const uint4* kp4 = reinterpret_cast<const uint4*>(kv + off);
#pragma unroll 4
      for (int c = 0; c < kHdD / 8; ++c) {
        const uint4 raw = kp4[c];
        const T* e = reinterpret_cast<const T*>(&raw);
        float kf[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) kf[j] = to_f32(e[j]);
#pragma unroll
        for (int r = 0; r < kDecodeMaxRows; ++r) {
          if (r < R) {
            const float4 qa = *reinterpret_cast<const float4*>(&q_s[r][c * 8]);
            const float4 qb = *reinterpret_cast<const float4*>(&q_s[r][c * 8 + 4]);
            sc[r] += qa.x * kf[0] + qa.y * kf[1] + qa.z * kf[2] + qa.w * kf[3] + qb.x * kf[4] + qb.y * kf[5] +
                     qb.z * kf[6] + qb.w * kf[7];
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kDecodeMaxRows; ++r) {
      if (r < R) {
        const float s = (off >= 0 && x < lim_s[r]) ? sc[r] * sl2 : -INFINITY;
        p_s[r][tid] = s;
        const float wm = warp_max(s);
        if (lane == 0) red_s[warp][r] = wm;
      }
    }
    __syncthreads();
    if (tid < R) {
      float cm = red_s[0][tid];
#pragma unroll
      for (int w = 1; w < kDecThreads / 32; ++w) cm = fmaxf(cm, red_s[w][tid]);
      const float mold = mrun_s[tid];
      const float mnew = fmaxf(mold, cm);
      alpha_s[tid] = mold == -INFINITY ? 0.f : exp2f(mold - mnew);  // nothing accumulated yet: 0
      mrun_s[tid] = mnew;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kDecodeMaxRows; ++r) {
      if (r < R) {
        const float s = p_s[r][tid];
        const float mr = mrun_s[r];
        p_s[r][tid] = (s == -INFINITY || mr == -INFINITY) ? 0.f : exp2f(s - mr);
      }
    }
    __syncthreads();
    // ---- pass 2: warp w accumulates its rows; lane l owns dimensions 4l..4l+3
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int r = warp + i * (kDecThreads / 32);
      if (r < R) {
        const float a = alpha_s[r];
        l_run[i] *= a;
        acc[i][0] *= a;
        acc[i][1] *= a;
        acc[i][2] *= a;
        acc[i][3] *= a;
      }
    }
    for (int j = 0; j < n; ++j) {
      const int64_t o = off_s[j];
      if (o < 0) continue;  // block-uniform
      const float2 raw = *reinterpret_cast<const float2*>(kv + o + v_step + lane * 4);
      const T* e = reinterpret_cast<const T*>(&raw);
      const float v0 = to_f32(e[0]), v1 = to_f32(e[1]), v2 = to_f32(e[2]), v3 = to_f32(e[3]);
#pragma unroll
      for (int i = 0; i < kRowsPerWarp; ++i) {
        const int r = warp + i * (kDecThreads / 32);
        if (r < R) {
          const float pj = p_s[r][j];
          l_run[i] += pj;
          acc[i][0] += pj * v0;
          acc[i][1] += pj * v1;
          acc[i][2] += pj * v2;
          acc[i][3] += pj * v3;
        }
      }
    }
    __syncthreads();  // p_s, off_s and alpha_s are rewritten by the next chunk
  }

  // ---- split partials in the tensor-core kernel's format (max in log2 units, sum, unnormalized O)
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    const int r = warp + i * (kDecThreads / 32);
    if (r < R) {
      const int m = r / G, hq = h * G + r % G;
      const int64_t rowi = static_cast<int64_t>(split) * p.M * p.Hq + static_cast<int64_t>(m) * p.Hq + hq;
      const float l = l_run[i];
      if (l > 0.f) {
        *reinterpret_cast<float4*>(p.part_o + rowi * kHdD + lane * 4) =
            make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      }
      if (lane == 0) p.part_ml[rowi] = make_float2(l > 0.f ? mrun_s[r] : -INFINITY, l);
    }
  }
}

cudaError_t launch_attention_decode(const AttnParams& p, cudaStream_t st) {
  if (p.M * (p.Hq / p.Hkv) > kDecodeMaxRows) return cudaErrorInvalidValue;
  const dim3 grid(p.Hkv, p.splits);
  if (p.bf16) return launch_k(attn_decode_split<__nv_bfloat16>, grid, dim3(kDecThreads), 0, st, p);
  return launch_k(attn_decode_split<__half>, grid, dim3(kDecThreads), 0, st, p);
}

}  // namespace atlas
