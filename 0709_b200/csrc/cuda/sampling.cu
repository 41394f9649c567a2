// Vocabulary-wide reductions on fp32 logits rows:
//  * log-softmax + top-k (k <= 8), greedy or keyed Gumbel-top-k sampling:
//    pass 1 splits every row into vocabulary chunks (one block each) that
//    produce the chunk's max / sum-exp and top-k; pass 2 (one warp per row)
//    merges them.  Ties prefer the smaller token id, so the order is
//    deterministic.
//    Gumbel noise for token v is a pure function of the row key and v
//    (SplitMix64-style mix; the same arithmetic as the PyTorch path).
//  * per-row log-sum-exp and a gather of (row, token) log-probabilities for
//    target path scoring.
// Parity: reference fp/sampling.py:108-156 and fp/frontier.py:145-189 (top-k
// candidates), src/atlas_0709/target_runtime.py:722-765 (path scoring).

#include "common.cuh"
#include "kernels.h"
#include "launch.h"

namespace atlas {

namespace {
constexpr int kMaxK = 8;
constexpr int kThreads = 512;

__device__ __forceinline__ float keyed_gumbel(uint64_t key, uint32_t v) {
  uint64_t x = key + static_cast<uint64_t>(v + 1) * 0x9E3779B97F4A7C15ull;
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  const float u = (static_cast<float>(x >> 40) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

__device__ __forceinline__ bool better(float s1, int i1, float s2, int i2) {
  return s1 > s2 || (s1 == s2 && i1 < i2);
}
}  // namespace

// Block-wide: pop the best head among all threads' sorted lists, k times.
// Thread lists are (score, id, logit) triples sorted by `better`.
template <int NT>
__device__ void block_topk_merge(float* ts, int* ti, float* tl, int k, float* out_s, int* out_i, float* out_l) {
  __shared__ float bs[NT / 32];
  __shared__ int bi[NT / 32], bt[NT / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int head = 0;
  for (int r = 0; r < k; ++r) {
    float s = head < k ? ts[head] : -INFINITY;
    int id = head < k ? ti[head] : 0x7fffffff;
    int owner = threadIdx.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, id, o);
      const int w2 = __shfl_xor_sync(0xffffffffu, owner, o);
      if (better(s2, i2, s, id)) {
        s = s2;
        id = i2;
        owner = w2;
      }
    }
    if (lane == 0) {
      bs[warp] = s;
      bi[warp] = id;
      bt[warp] = owner;
    }
    __syncthreads();
    if (warp == 0) {
      float s3 = lane < NT / 32 ? bs[lane] : -INFINITY;
      int i3 = lane < NT / 32 ? bi[lane] : 0x7fffffff;
      int w3 = lane < NT / 32 ? bt[lane] : -1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float s2 = __shfl_xor_sync(0xffffffffu, s3, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, i3, o);
        const int w2 = __shfl_xor_sync(0xffffffffu, w3, o);
        if (better(s2, i2, s3, i3)) {
          s3 = s2;
          i3 = i2;
          w3 = w2;
        }
      }
      if (lane == 0) {
        bt[0] = w3;
        bi[0] = i3;
        bs[0] = s3;
      }
    }
    __syncthreads();
    const int win = bt[0];
    if (threadIdx.x == win) {
      out_s[r] = ts[head];
      out_i[r] = ti[head];
      out_l[r] = tl[head];
      ++head;
    }
    __syncthreads();
  }
}

// Pass 1: grid (chunks, rows).  Each block scans one vocabulary chunk of one
// row: online max / sum-exp and the chunk's top-k (score, id, logit).
constexpr int kChunkThreads = 256;

__global__ void __launch_bounds__(kChunkThreads) topk_chunk_kernel(const float* __restrict__ logits, int V, int k,
                                                                   int chunk, const int64_t* __restrict__ keys,
                                                                   float inv_temp, float* __restrict__ part) {
  pdl_wait();
  pdl_trigger();
  const int c = blockIdx.x, b = blockIdx.y, C = gridDim.x;
  const float* row = logits + static_cast<int64_t>(b) * V;
  const bool sample = keys != nullptr;
  const uint64_t key = sample ? static_cast<uint64_t>(keys[b]) : 0ull;
  const int v0 = c * chunk, v1 = min(V, v0 + chunk);
  float mx = -INFINITY, sum = 0.f;
  float ts[kMaxK], tl[kMaxK];
  int ti[kMaxK];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    ts[j] = -INFINITY;
    tl[j] = -INFINITY;
    ti[j] = 0x7fffffff;
  }
  for (int v = v0 + threadIdx.x; v < v1; v += kChunkThreads) {
    const float x = row[v];
    if (x > mx) {
      sum = sum * __expf(mx - x) + 1.f;
      mx = x;
    } else {
      sum += __expf(x - mx);
    }
    const float sc = sample ? x * inv_temp + keyed_gumbel(key, static_cast<uint32_t>(v)) : x;
    if (better(sc, v, ts[k - 1], ti[k - 1])) {
      int j = k - 1;
      while (j > 0 && better(sc, v, ts[j - 1], ti[j - 1])) {
        ts[j] = ts[j - 1];
        ti[j] = ti[j - 1];
        tl[j] = tl[j - 1];
        --j;
      }
      ts[j] = sc;
      ti[j] = v;
      tl[j] = x;
    }
  }
  __shared__ float smx[kChunkThreads / 32], ssum[kChunkThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float wmx = warp_max(mx);
  const float wsum = warp_sum(mx == -INFINITY ? 0.f : sum * __expf(mx - wmx));
  if (lane == 0) {
    smx[warp] = wmx;
    ssum[warp] = wsum;
  }
  __syncthreads();
  // record layout per (row, chunk): [max, sum, k scores, k ids (as float bits), k logits]
  float* rec = part + (static_cast<int64_t>(b) * C + c) * (2 + 3 * kMaxK);
  if (warp == 0) {
    const float m2 = lane < kChunkThreads / 32 ? smx[lane] : -INFINITY;
    const float s2 = lane < kChunkThreads / 32 ? ssum[lane] : 0.f;
    const float bm = warp_max(m2);
    const float bsum = warp_sum(m2 == -INFINITY ? 0.f : s2 * __expf(m2 - bm));
    if (lane == 0) {
      rec[0] = bm;
      rec[1] = bsum;
    }
  }
  __shared__ float os[kMaxK], ol[kMaxK];
  __shared__ int oi[kMaxK];
  block_topk_merge<kChunkThreads>(ts, ti, tl, k, os, oi, ol);
  if (threadIdx.x < k) {
    rec[2 + threadIdx.x] = os[threadIdx.x];
    rec[2 + kMaxK + threadIdx.x] = __int_as_float(oi[threadIdx.x]);
    rec[2 + 2 * kMaxK + threadIdx.x] = ol[threadIdx.x];
  }
}

// Pass 2: one warp per row merges the chunk records.
__global__ void topk_merge_kernel(const float* __restrict__ part, int C, int k, int V, float* __restrict__ out_lp,
                                  int64_t* __restrict__ out_id) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const int lane = threadIdx.x;
  const float* recs = part + static_cast<int64_t>(b) * C * (2 + 3 * kMaxK);
  float mx = -INFINITY, sum = 0.f;
  for (int c = lane; c < C; c += 32) {
    const float m2 = recs[c * (2 + 3 * kMaxK)], s2 = recs[c * (2 + 3 * kMaxK) + 1];
    if (m2 == -INFINITY) continue;
    if (m2 > mx) {
      sum = sum * __expf(mx - m2) + s2;
      mx = m2;
    } else {
      sum += s2 * __expf(m2 - mx);
    }
  }
  const float gm = warp_max(mx);
  const float gs = warp_sum(mx == -INFINITY ? 0.f : sum * __expf(mx - gm));
  const float lse = gm + logf(gs);
  // Each lane walks its chunks' sorted lists; k rounds of warp argmax.
  int heads[8];
  const int per = (C + 31) / 32;
  for (int i = 0; i < 8; ++i) heads[i] = 0;
  for (int r = 0; r < k; ++r) {
    float s = -INFINITY;
    int id = 0x7fffffff, src = -1;
    for (int i = 0; i < per && i < 8; ++i) {
      const int c = lane + i * 32;
      if (c >= C || heads[i] >= k) continue;
      const float* rc = recs + c * (2 + 3 * kMaxK);
      const float sc = rc[2 + heads[i]];
      const int ii = __float_as_int(rc[2 + kMaxK + heads[i]]);
      if (better(sc, ii, s, id)) {
        s = sc;
        id = ii;
        src = i;
      }
    }
    int owner = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, id, o);
      const int w2 = __shfl_xor_sync(0xffffffffu, owner, o);
      if (better(s2, i2, s, id)) {
        s = s2;
        id = i2;
        owner = w2;
      }
    }
    if (lane == owner && src >= 0) {
      const float* rc = recs + (lane + src * 32) * (2 + 3 * kMaxK);
      const float logit = rc[2 + 2 * kMaxK + heads[src]];
      const bool valid = id >= 0 && id < V;
      out_id[static_cast<int64_t>(b) * k + r] = valid ? id : 0;
      out_lp[static_cast<int64_t>(b) * k + r] = valid ? logit - lse : -INFINITY;
      ++heads[src];
    }
    __syncwarp();
  }
}

__global__ void __launch_bounds__(kThreads) row_lse_kernel(const float* __restrict__ logits, int V,
                                                           float* __restrict__ lse_out) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const float* row = logits + static_cast<int64_t>(b) * V;
  float mx = -INFINITY, sum = 0.f;
  for (int v = threadIdx.x; v < V; v += kThreads) {
    const float x = row[v];
    if (x > mx) {
      sum = sum * __expf(mx - x) + 1.f;
      mx = x;
    } else {
      sum += __expf(x - mx);
    }
  }
  __shared__ float smx[kThreads / 32], ssum[kThreads / 32];
  const float wmx = warp_max(mx);
  float wsum = warp_sum(sum * (mx == -INFINITY ? 0.f : __expf(mx - wmx)));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    smx[warp] = wmx;
    ssum[warp] = wsum;
  }
  __syncthreads();
  if (warp == 0) {
    const float m2 = lane < kThreads / 32 ? smx[lane] : -INFINITY;
    const float s2 = lane < kThreads / 32 ? ssum[lane] : 0.f;
    const float bm = warp_max(m2);
    const float bsum = warp_sum(m2 == -INFINITY ? 0.f : s2 * __expf(m2 - bm));
    if (lane == 0) lse_out[b] = bm + logf(bsum);
  }
}

__global__ void gather_lp_kernel(const float* __restrict__ logits, int V, int R, const float* __restrict__ lse,
                                 const int* __restrict__ rows, const int* __restrict__ toks, int n,
                                 float* __restrict__ out, int* err) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = rows[i], t = toks[i];
  if (r < 0 || r >= R || t < 0 || t >= V) {
    set_error(err, kErrBadIndex);
    out[i] = -INFINITY;
    return;
  }
  out[i] = logits[static_cast<int64_t>(r) * V + t] - lse[r];
}

cudaError_t launch_topk(const float* logits, int B, int V, int k, const int64_t* keys, float inv_temp, float* out_lp,
                 int64_t* out_id, float* part, int chunks, cudaStream_t st) {
  const int chunk = (V + chunks - 1) / chunks;
  const cudaError_t e = launch_k(topk_chunk_kernel, dim3(chunks, B), dim3(kChunkThreads), 0, st, logits, V, k, chunk, keys, inv_temp, part);
  if (e != cudaSuccess) return e;
  return launch_k(topk_merge_kernel, dim3(B), dim3(32), 0, st, static_cast<const float*>(part), chunks, k, V, out_lp, out_id);
}

int topk_record_floats() { return 2 + 3 * kMaxK; }

void launch_gather_logprobs(const float* logits, int R, int V, const int* rows, const int* toks, int n, float* lse,
                            float* out, int* err, cudaStream_t st) {
  launch_k(row_lse_kernel, dim3(R), dim3(kThreads), 0, st, logits, V, lse);
  launch_k(gather_lp_kernel, dim3((n + 127) / 128), dim3(128), 0, st, logits, V, R, static_cast<const float*>(lse), rows,
           toks, n, out, err);
}

}  // namespace atlas
