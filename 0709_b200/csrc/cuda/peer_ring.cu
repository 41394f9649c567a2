// Message rings in peer GPU memory: the drafter <-> target handoff across GPUs.
//
// A ring lives in the RECEIVER's device memory (a plain cudaMalloc region that
// the sender maps through CUDA IPC):
//   [0, 4)      sequence flag: the number of the last message published
//   [256, ...)  one message: 16-byte header {nbytes, seq, 0, 0} + payload
// Requests and responses alternate (a sender publishes message n + 1 only
// after the receiver has answered message n), so one message slot per
// direction is enough and no credit flag is needed.
//
//  ring_push: one CTA copies header + payload from the sender's staging
//    (device memory, or pinned host memory, which is mapped into the device's
//    address space) into the peer's slot with 16-byte stores over NVLink;
//    every thread fences its stores at system scope, and after a CTA barrier
//    thread 0 publishes the sequence number with a system-scope release store.
//  ring_pop: thread 0 polls the flag with system-scope acquire loads, bounded
//    by the wall-clock limit (ring errors go to the ring's own flag: an idle
//    wait that runs out is expected while a peer is busy, and the host simply
//    polls again); then the CTA copies the message to the receiver's
//    destination (pinned host memory or device memory) with cache-bypassing
//    loads.  A message longer than the destination is an error, not a copy.
//
// Plain loads and stores only: no TMA, no multicast, no NVLink multicast
// objects.  Parity: replaces the reference's HTTP JSON transport between the
// drafter process and the target server (src/atlas_0709/rpc.py:245-303).

#include "common.cuh"
#include "peer_ring.h"

namespace atlas {

namespace {
constexpr int kRingThreads = 256;
constexpr int kHeaderBytes = 16;

// Plain stream-ordered launch (no programmatic overlap: a push reads data the
// previous kernel wrote); returns the launch's own status.
template <typename... KArgs, typename... Args>
cudaError_t launch_plain(void (*kern)(KArgs...), cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kRingThreads);
  cfg.stream = st;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}
}  // namespace

__global__ void __launch_bounds__(kRingThreads)
    ring_push_kernel(const uint4* __restrict__ src, int n16, uint4* __restrict__ slot, uint32_t* flag, uint32_t seq) {
  for (int i = threadIdx.x; i < n16; i += kRingThreads) slot[i] = src[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) st_release_sys(flag, seq);
}

__global__ void __launch_bounds__(kRingThreads)
    ring_pop_kernel(const uint4* slot, const uint32_t* flag, uint32_t seq, uint4* dst, int64_t dst_bytes,
                    int* out_nbytes, int* err, uint64_t limit_ns) {
  __shared__ int s_n;
  if (threadIdx.x == 0) {
    int n = -1;
    if (wait_flag_geq(flag, seq, err, limit_ns)) {
      const uint32_t* hdr = reinterpret_cast<const uint32_t*>(slot);
      const uint32_t nbytes = __ldcv(hdr);
      const uint32_t got = __ldcv(hdr + 1);
      if (got != seq || static_cast<int64_t>(nbytes) + kHeaderBytes > dst_bytes) {
        set_error(err, kErrBadIndex);
      } else {
        n = static_cast<int>(nbytes);
      }
    }
    s_n = n;
    if (out_nbytes != nullptr) *out_nbytes = n;
  }
  __syncthreads();
  const int n = s_n;
  if (n < 0) return;
  fence_acq_rel_sys();
  const int n16 = (n + kHeaderBytes + 15) / 16;
  for (int i = threadIdx.x; i < n16; i += kRingThreads) dst[i] = __ldcv(slot + i);
}

cudaError_t launch_ring_push(const void* src, int64_t bytes, void* peer_ring, uint32_t seq, cudaStream_t st) {
  if (bytes < kHeaderBytes || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(peer_ring) & 255))
    return cudaErrorInvalidValue;
  const int n16 = static_cast<int>((bytes + 15) / 16);
  uint8_t* base = static_cast<uint8_t*>(peer_ring);
  return launch_plain(ring_push_kernel, st, static_cast<const uint4*>(src), n16,
                      reinterpret_cast<uint4*>(base + kRingSlotOffset), reinterpret_cast<uint32_t*>(base), seq);
}

cudaError_t launch_ring_pop(const void* ring, uint32_t seq, void* dst, int64_t dst_bytes, int* out_nbytes, int* err,
                            uint64_t limit_ns, cudaStream_t st) {
  if ((reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(ring) & 255)) return cudaErrorInvalidValue;
  const uint8_t* base = static_cast<const uint8_t*>(ring);
  return launch_plain(ring_pop_kernel, st, reinterpret_cast<const uint4*>(base + kRingSlotOffset),
                      reinterpret_cast<const uint32_t*>(base), seq, static_cast<uint4*>(dst), dst_bytes, out_nbytes,
                      err, limit_ns);
}

}  // namespace atlas
