// KV-cache maintenance kernels (all layers in one launch):
//  * tail-page copy-on-write: copy the first ntok slots of a shared partial
//    page into a freshly allocated private page;
//  * slot moves for the target's in-place compaction of the selected route:
//    every source is read into shared memory before any destination is
//    written, so overlapping source/destination sets are safe.
// Parity: reference fp/sglang_runtime.py:686-695 (move_kv_cache for COW) and
// src/atlas_0709/target_runtime.py:873-920 (per-layer gather/scatter commit).

#include "common.cuh"
#include "kernels.h"
#include "launch.h"

namespace atlas {

// grid (copies, layers, 2 * Hkv); cache layout [L, pages, 2, Hkv, ps, hd].
__global__ void kv_copy_pages_kernel(uint4* __restrict__ kv, const int* __restrict__ plan, int num_pages, int Hkv,
                                     int ps, int hd, int* err) {
  pdl_wait();
  pdl_trigger();
  const int ci = blockIdx.x;
  const int layer = blockIdx.y;
  const int kvh = blockIdx.z;  // (k|v) * Hkv + head
  const int src = plan[ci * 3 + 0], dst = plan[ci * 3 + 1], ntok = plan[ci * 3 + 2];
  if (src < 0 || src >= num_pages || dst < 0 || dst >= num_pages || ntok < 0 || ntok > ps) {
    if (threadIdx.x == 0) set_error(err, kErrBadIndex);
    return;
  }
  const int64_t head_vec = static_cast<int64_t>(ps) * hd / 8;  // uint4 per (page, kv, head)
  const int64_t page_vec = 2 * Hkv * head_vec;
  const int64_t base = static_cast<int64_t>(layer) * num_pages * page_vec + kvh * head_vec;
  const uint4* s = kv + base + src * page_vec;
  uint4* d = kv + base + dst * page_vec;
  const int n = ntok * hd / 8;
  for (int i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
}

// Copy-on-write inside a captured forward: the plan and its length live in the forward's
// static inputs (written by the one host->device copy of each call), so one graph serves any
// number of copies up to max_n.  grid (layers, 2 * Hkv); each block copies every page.
__global__ void kv_copy_pages_counted_kernel(uint4* __restrict__ kv, const int* __restrict__ plan,
                                             const int* __restrict__ count, int max_n, int num_pages, int Hkv, int ps,
                                             int hd, int* err) {
  pdl_wait();
  pdl_trigger();
  const int n = min(*count, max_n);
  const int layer = blockIdx.x;
  const int kvh = blockIdx.y;  // (k|v) * Hkv + head
  const int64_t head_vec = static_cast<int64_t>(ps) * hd / 8;
  const int64_t page_vec = 2 * Hkv * head_vec;
  const int64_t base = static_cast<int64_t>(layer) * num_pages * page_vec + kvh * head_vec;
  for (int ci = 0; ci < n; ++ci) {
    const int src = plan[ci * 3 + 0], dst = plan[ci * 3 + 1], ntok = plan[ci * 3 + 2];
    if (src < 0 || src >= num_pages || dst < 0 || dst >= num_pages || ntok < 0 || ntok > ps) {
      if (threadIdx.x == 0) set_error(err, kErrBadIndex);
      continue;
    }
    const uint4* sp = kv + base + src * page_vec;
    uint4* dp = kv + base + dst * page_vec;
    const int nv = ntok * hd / 8;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) dp[i] = sp[i];
  }
}

// grid (layers, 2 * Hkv); n <= 64 slots.
__global__ void kv_move_slots_kernel(uint4* __restrict__ kv, const int* __restrict__ src, const int* __restrict__ dst,
                                     int n, int num_pages, int Hkv, int ps, int hd, int* err) {
  extern __shared__ uint4 buf[];
  pdl_wait();
  pdl_trigger();
  const int layer = blockIdx.x;
  const int kvh = blockIdx.y;
  const int per = hd / 8;
  const int64_t head_vec = static_cast<int64_t>(ps) * per;
  const int64_t page_vec = 2 * Hkv * head_vec;
  const int64_t base = static_cast<int64_t>(layer) * num_pages * page_vec + kvh * head_vec;
  for (int i = threadIdx.x; i < n * per; i += blockDim.x) {
    const int j = i / per, c = i % per;
    const int sl = src[j];
    if (sl < 0 || sl / ps >= num_pages) {
      set_error(err, kErrBadIndex);
      buf[i] = make_uint4(0, 0, 0, 0);
      continue;
    }
    buf[i] = kv[base + (sl / ps) * page_vec + (sl % ps) * per + c];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n * per; i += blockDim.x) {
    const int j = i / per, c = i % per;
    const int dl = dst[j];
    if (dl < 0 || dl / ps >= num_pages) {
      set_error(err, kErrBadIndex);
      continue;
    }
    kv[base + (dl / ps) * page_vec + (dl % ps) * per + c] = buf[i];
  }
}

void launch_kv_copy_pages(void* kv, const int* plan, int n, int layers, int num_pages, int Hkv, int ps, int hd,
                          int* err, cudaStream_t st) {
  if (n == 0) return;
  dim3 grid(n, layers, 2 * Hkv);
  launch_k(kv_copy_pages_kernel, grid, dim3(128), 0, st, static_cast<uint4*>(kv), plan, num_pages, Hkv, ps, hd, err);
}

void launch_kv_copy_pages_counted(void* kv, const int* plan, const int* count, int max_n, int layers, int num_pages,
                                  int Hkv, int ps, int hd, int* err, cudaStream_t st) {
  dim3 grid(layers, 2 * Hkv);
  launch_k(kv_copy_pages_counted_kernel, grid, dim3(128), 0, st, static_cast<uint4*>(kv), plan, count, max_n,
           num_pages, Hkv, ps, hd, err);
}

void launch_kv_move_slots(void* kv, const int* src, const int* dst, int n, int layers, int num_pages, int Hkv, int ps,
                          int hd, int* err, cudaStream_t st) {
  if (n == 0) return;
  dim3 grid(layers, 2 * Hkv);
  const size_t smem = static_cast<size_t>(n) * (hd / 8) * sizeof(uint4);
  launch_k(kv_move_slots_kernel, grid, dim3(256), smem, st, static_cast<uint4*>(kv), src, dst, n, num_pages, Hkv, ps,
           hd, err);
}

}  // namespace atlas
