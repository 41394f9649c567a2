// Vocabulary-wide reductions on fp32 logits rows:
//  * log-softmax + top-k (k <= 8), greedy or keyed Gumbel-top-k sampling:
//    one block per row computes the row's log-sum-exp and its top-k in one
//    pass; ties prefer the smaller token id, so the order is deterministic.
//    Gumbel noise for token v is a pure function of the row key and v
//    (SplitMix64-style mix; the same arithmetic as the PyTorch path).
//  * per-row log-sum-exp and a gather of (row, token) log-probabilities for
//    target path scoring.
// Parity: reference fp/sampling.py:108-156 and fp/frontier.py:145-189 (top-k
// candidates), src/atlas_0709/target_runtime.py:722-765 (path scoring).

#include "common.cuh"
#include "kernels.h"

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

__global__ void __launch_bounds__(kThreads) topk_kernel(const float* __restrict__ logits, int V, int k,
                                                        const int64_t* __restrict__ keys, float inv_temp,
                                                        float* __restrict__ out_lp, int64_t* __restrict__ out_id) {
  const int b = blockIdx.x;
  const float* row = logits + static_cast<int64_t>(b) * V;
  const bool sample = keys != nullptr;
  const uint64_t key = sample ? static_cast<uint64_t>(keys[b]) : 0ull;
  float mx = -INFINITY, sum = 0.f;
  float ts[kMaxK];
  int ti[kMaxK];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    ts[j] = -INFINITY;
    ti[j] = 0x7fffffff;
  }
  for (int v = threadIdx.x; v < V; v += kThreads) {
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
        --j;
      }
      ts[j] = sc;
      ti[j] = v;
    }
  }
  __shared__ float smx[kThreads / 32], ssum[kThreads / 32];
  __shared__ float bs[kThreads / 32];
  __shared__ int bi[kThreads / 32], bt[kThreads / 32];
  __shared__ float lse_s;
  // log-sum-exp
  const float wmx = warp_max(mx);
  float wsum = sum * (mx == -INFINITY ? 0.f : __expf(mx - wmx));
  wsum = warp_sum(wsum);
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
    if (lane == 0) lse_s = bm + logf(bsum);
  }
  __syncthreads();
  const float lse = lse_s;
  // k rounds of block-wide best-of-heads
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
      float s3 = lane < kThreads / 32 ? bs[lane] : -INFINITY;
      int i3 = lane < kThreads / 32 ? bi[lane] : 0x7fffffff;
      int w3 = lane < kThreads / 32 ? bt[lane] : -1;
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
      }
    }
    __syncthreads();
    const int win = bt[0], wid = bi[0];
    if (threadIdx.x == 0) {
      const bool valid = wid >= 0 && wid < V;
      out_id[static_cast<int64_t>(b) * k + r] = valid ? wid : 0;
      out_lp[static_cast<int64_t>(b) * k + r] = valid ? row[wid] - lse : -INFINITY;
    }
    if (threadIdx.x == win) ++head;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kThreads) row_lse_kernel(const float* __restrict__ logits, int V,
                                                           float* __restrict__ lse_out) {
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

void launch_topk(const float* logits, int B, int V, int k, const int64_t* keys, float inv_temp, float* out_lp,
                 int64_t* out_id, cudaStream_t st) {
  topk_kernel<<<B, kThreads, 0, st>>>(logits, V, k, keys, inv_temp, out_lp, out_id);
}

void launch_gather_logprobs(const float* logits, int R, int V, const int* rows, const int* toks, int n, float* lse,
                            float* out, int* err, cudaStream_t st) {
  row_lse_kernel<<<R, kThreads, 0, st>>>(logits, V, lse);
  gather_lp_kernel<<<(n + 127) / 128, 128, 0, st>>>(logits, V, R, lse, rows, toks, n, out, err);
}

}  // namespace atlas
