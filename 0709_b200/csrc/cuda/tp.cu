// Tensor-parallel reduction kernels (the consumer half of the fused
// row-parallel GEMM + all-reduce; the producer half is the GEMM's peer
// epilogue, which stores each rank's fp32 partial tile into every rank's
// receive buffer over NVLink and raises a sequence flag).
//
//  tp_reduce_rmsnorm: wait until every rank's flag has reached this rank's own
//    sequence number for the call site, then  h += sum_r partial_r  (ranks
//    summed in rank order, so every rank computes bit-identical residuals)
//    and  x = RMSNorm(h) * gamma  in the activation dtype -- the residual add
//    and the next layer's input norm fused with the reduction.  Each row is
//    spread over a cluster of 8 CTAs (one eighth of the features each).
//  tp_wait: the same wait alone (the root rank before it reads the gathered
//    vocabulary-parallel logits).
//
// All waits are bounded by g_peer_wait_ns (wall time, per device, set from the
// host with set_peer_wait_ns): on timeout the kernel records kErrPeerTimeout
// and carries on with whatever is in the buffers; the host reads the error
// flag with the next result it copies back and stops before using them.

#include "common.cuh"
#include "launch.h"
#include "gemm.h"
#include "tp.h"

namespace atlas {

// Wall-time limit of every cross-GPU wait in this file's kernels, in ns.  Read
// at run time, so graphs captured earlier follow a later set_peer_wait_ns.
static __device__ uint64_t g_peer_wait_ns = kPeerWaitDefaultNs;

__device__ __forceinline__ void wait_all_ranks(const uint32_t* flags, const uint32_t* seq, int nsrc, int* err) {
  if (flags != nullptr && static_cast<int>(threadIdx.x) < nsrc) {
    const uint32_t target = *reinterpret_cast<const volatile uint32_t*>(seq);
    wait_flag_geq(flags + threadIdx.x, target, err, g_peer_wait_ns);
  }
  __syncthreads();
}

constexpr int kReduceThreads = 128;
constexpr int kReduceCluster = 8;  // CTAs per row: each owns H / 8 features
constexpr int kReduceVec = 4;      // float4 per thread kept in registers (H <= 8 * 128 * 4 * 4 = 16384)

// One cluster of 8 CTAs per row: CTA r sums the sources for features
// [r H/8, (r+1) H/8), adds the residual and its part of sum(h^2); the 8
// partial sums meet through distributed shared memory (read in rank order,
// so every CTA -- and every TP rank -- computes the same rstd).
// Sentinel mode: poll one float4 of a receive slot until none of its words is
// the sentinel (bounded by the global timer), then put the sentinel back for
// the slot's next use.
__device__ __forceinline__ float4 take_slot(float* ptr, int* err) {
  float4 v;
  const uint64_t t0 = global_timer_ns();
  const uint64_t limit = g_peer_wait_ns;
  uint32_t polls = 0;
  while (true) {
    asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(ptr)
                 : "memory");
    if (__float_as_uint(v.x) != kPeerSentinel && __float_as_uint(v.y) != kPeerSentinel &&
        __float_as_uint(v.z) != kPeerSentinel && __float_as_uint(v.w) != kPeerSentinel)
      break;
    if ((++polls & 63u) == 0) {
      if (*reinterpret_cast<volatile int*>(err) != 0 || global_timer_ns() - t0 > limit) {
        set_error(err, kErrPeerTimeout);
        break;
      }
    }
  }
  const float s = __uint_as_float(kPeerSentinel);
  *reinterpret_cast<float4*>(ptr) = make_float4(s, s, s, s);
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kReduceThreads)
    tp_reduce_rmsnorm_kernel(const float* __restrict__ recv, int64_t slot_stride, const uint32_t* flags,
                             const uint32_t* seq, int nsrc, int sentinel, float* __restrict__ h,
                             const T* __restrict__ gamma, T* __restrict__ x, int H, float eps, int* err) {
  __shared__ float red[kReduceThreads / 32];
  __shared__ float part_ss;
  pdl_wait();
  pdl_trigger();
  wait_all_ranks(flags, seq, nsrc, err);
  const int m = blockIdx.y;
  const int chunk = H / kReduceCluster;
  const int c0 = static_cast<int>(blockIdx.x) * chunk;
  float* hr = h + static_cast<int64_t>(m) * H;
  const float* pr = recv + static_cast<int64_t>(m) * H;
  float ss = 0.f;
  float4 keep[kReduceVec];
#pragma unroll
  for (int j = 0; j < kReduceVec; ++j) {
    const int i = c0 + (j * kReduceThreads + static_cast<int>(threadIdx.x)) * 4;
    if (i < c0 + chunk) {
      float4 acc;
      if (sentinel) {
        float* slot0 = const_cast<float*>(pr) + i;
        acc = take_slot(slot0, err);
        for (int r = 1; r < nsrc; ++r) {
          const float4 v = take_slot(slot0 + r * slot_stride, err);
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
      } else {
        acc = __ldcg(reinterpret_cast<const float4*>(pr + i));
        for (int r = 1; r < nsrc; ++r) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(pr + r * slot_stride + i));
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
      }
      float4 o = *reinterpret_cast<const float4*>(hr + i);
      o.x += acc.x;
      o.y += acc.y;
      o.z += acc.z;
      o.w += acc.w;
      *reinterpret_cast<float4*>(hr + i) = o;
      ss += o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
      keep[j] = o;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) part_ss = (red[0] + red[1]) + (red[2] + red[3]);
  cluster_sync();
  float tot = 0.f;
#pragma unroll
  for (int r = 0; r < kReduceCluster; ++r) tot += ld_dsmem_f32(&part_ss, r);
  if (gamma != nullptr) {
    const float inv = rsqrtf(tot / static_cast<float>(H) + eps);
    T* xr = x + static_cast<int64_t>(m) * H;
#pragma unroll
    for (int j = 0; j < kReduceVec; ++j) {
      const int i = c0 + (j * kReduceThreads + static_cast<int>(threadIdx.x)) * 4;
      if (i < c0 + chunk) {
        const float4 o = keep[j];
        xr[i] = from_f32<T>(o.x * inv * to_f32(gamma[i]));
        xr[i + 1] = from_f32<T>(o.y * inv * to_f32(gamma[i + 1]));
        xr[i + 2] = from_f32<T>(o.z * inv * to_f32(gamma[i + 2]));
        xr[i + 3] = from_f32<T>(o.w * inv * to_f32(gamma[i + 3]));
      }
    }
  }
  cluster_sync();  // partial sums stay alive until every CTA of the cluster has read them
}

__global__ void tp_wait_kernel(const uint32_t* flags, const uint32_t* seq, int nsrc, int* err) {
  pdl_wait();
  pdl_trigger();
  wait_all_ranks(flags, seq, nsrc, err);
}

void launch_tp_reduce_rmsnorm(const float* recv, int64_t slot_stride, const uint32_t* flags, const uint32_t* seq,
                              int nsrc, int sentinel, float* h, const void* gamma, void* x, int M, int H, float eps,
                              bool bf16, int* err, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kReduceCluster, M);
  cfg.blockDim = dim3(kReduceThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kReduceCluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (bf16)
    cudaLaunchKernelEx(&cfg, tp_reduce_rmsnorm_kernel<__nv_bfloat16>, recv, slot_stride, flags, seq, nsrc, sentinel, h,
                       static_cast<const __nv_bfloat16*>(gamma), static_cast<__nv_bfloat16*>(x), H, eps, err);
  else
    cudaLaunchKernelEx(&cfg, tp_reduce_rmsnorm_kernel<__half>, recv, slot_stride, flags, seq, nsrc, sentinel, h,
                       static_cast<const __half*>(gamma), static_cast<__half*>(x), H, eps, err);
}

void launch_tp_wait(const uint32_t* flags, const uint32_t* seq, int nsrc, int* err, cudaStream_t st) {
  launch_k(tp_wait_kernel, dim3(1), dim3(32), 0, st, flags, seq, nsrc, err);
}

cudaError_t set_peer_wait_ns(uint64_t ns) { return cudaMemcpyToSymbol(g_peer_wait_ns, &ns, sizeof(ns)); }

cudaError_t get_peer_wait_ns(uint64_t* ns) { return cudaMemcpyFromSymbol(ns, g_peer_wait_ns, sizeof(*ns)); }

}  // namespace atlas
